// Key moments + Eq. 15 thresholds in one launch (replaces kernels.py:30-64, 211-215).
//
// One CTA per (b, h) and group of kThrQB q-blocks, D threads.  The head's centroid rows stream
// through a ring of kRingStages shared-memory stages of kRingRows rows (16-byte cp.async, several
// stages in flight, so the loads do not serialise with the sums).  Thread d sums kc[b,h,:,d] and
// its squares over all key blocks in block order (FP32, no FMA), giving mean and population
// variance var = max(E[x^2] - E[x]^2, 0) with every block weighted equally (kernels.py:40-47);
// every CTA of a head computes the same moments (the first one writes them out).  The group's
// Q means are staged in shared memory with coalesced loads, then thread j < kThrQB forms
//   cutoff = (sum_d qc*mean + beta * sqrt(sum_d (qc*qc)*var)) * scale
// for q-block j of the group with sequential sums over d (natural-log units; the fused kernel
// compares the unscaled proxy dot times scale against it).  All operations are explicitly
// rounded (__f*_rn) so a CPU restatement in FP32 reproduces the bits.
#include "common.cuh"

namespace solattn {

namespace {

constexpr int kThrQB = 32;      // q-blocks per CTA
constexpr int kRingRows = 16;   // centroid rows per ring stage
constexpr int kRingStages = 6;  // ring stages (kRingStages - 1 in flight)

template <int D>
__global__ void __launch_bounds__(D) threshold_kernel(const __nv_bfloat16* __restrict__ kc,
                                                      const float* __restrict__ qc, int nqb,
                                                      int nkb, const int32_t* __restrict__ tk_b,
                                                      int H, float scale, float beta,
                                                      float* mean_out, float* var_out,
                                                      float* cutoff) {
  __shared__ float s_mean[D];
  __shared__ float s_var[D];
  __shared__ float s_q[kThrQB][D + 1];  // +1: row-wise reads by different threads hit different banks
  const int bh = blockIdx.y;
  const int qb0 = blockIdx.x * kThrQB;
  const int nq = min(kThrQB, nqb - qb0);
  const int d = threadIdx.x;
  for (int i = d; i < nq * D; i += D)
    s_q[i / D][i % D] = qc[((int64_t)bh * nqb + qb0) * D + i];
  __shared__ __align__(16) __nv_bfloat16 s_kc[kRingStages][kRingRows][D];
  const __nv_bfloat16* kc_bh = kc + (int64_t)bh * nkb * D;
  // The batch's own key blocks in a ragged launch (kc rows past them are padding).
  const int nb = tk_b ? min(max((tk_b[bh / H] + kBlock - 1) / kBlock, 1), nkb) : nkb;
  const int nchunks = (nb + kRingRows - 1) / kRingRows;
  // Rows [c * kRingRows, ...) of the head into stage c % kRingStages; one commit group per
  // chunk (empty past the end) so that the wait below always counts the same groups.
  auto issue = [&](int c) {
    if (c < nchunks) {
      for (int i = d; i < kRingRows * (D / 8); i += D) {
        const int r = i / (D / 8), col = 8 * (i % (D / 8));
        const int row = c * kRingRows + r;
        if (row < nb)
          cp_async16(smem_u32(&s_kc[c % kRingStages][r][col]), kc_bh + (int64_t)row * D + col, 16);
      }
    }
    cp_async_commit();
  };
  for (int c = 0; c < kRingStages - 1; ++c) issue(c);
  float s1 = 0.f, s2 = 0.f;
  for (int c = 0; c < nchunks; ++c) {
    cp_async_wait<kRingStages - 2>();  // this thread's copies of chunk c have landed
    __syncthreads();  // everyone's have, and every thread is done with chunk c - 1's stage
    issue(c + kRingStages - 1);  // into the stage chunk c - 1 used
    const int rows = min(kRingRows, nb - c * kRingRows);
    const __nv_bfloat16* col = &s_kc[c % kRingStages][0][d];
    for (int r = 0; r < rows; ++r) {
      const float x = __bfloat162float(col[r * D]);
      s1 = __fadd_rn(s1, x);
      s2 = __fadd_rn(s2, __fmul_rn(x, x));
    }
  }
  cp_async_wait<0>();
  const float n = (float)nb;
  const float mean = __fdiv_rn(s1, n);
  const float var = fmaxf(__fsub_rn(__fdiv_rn(s2, n), __fmul_rn(mean, mean)), 0.f);
  s_mean[d] = mean;
  s_var[d] = var;
  if (blockIdx.x == 0) {
    mean_out[(int64_t)bh * D + d] = mean;
    var_out[(int64_t)bh * D + d] = var;
  }
  __syncthreads();
  if (d < nq) {
    float mu = 0.f, sg = 0.f;
    for (int e = 0; e < D; ++e) {
      const float qv = s_q[d][e];
      mu = __fadd_rn(mu, __fmul_rn(qv, s_mean[e]));
      sg = __fadd_rn(sg, __fmul_rn(__fmul_rn(qv, qv), s_var[e]));
    }
    cutoff[(int64_t)bh * nqb + qb0 + d] =
        __fmul_rn(__fadd_rn(mu, __fmul_rn(beta, __fsqrt_rn(sg))), scale);
  }
}

}  // namespace

cudaError_t launch_threshold(const __nv_bfloat16* kc, const float* qc, int BH, int H, int nqb,
                             int nkb, int D, float scale, float beta, float* mean, float* var,
                             float* cutoff, const int32_t* tk_b, cudaStream_t stream) {
  const dim3 grid((nqb + kThrQB - 1) / kThrQB, BH);
  if (D == 128)
    threshold_kernel<128><<<grid, 128, 0, stream>>>(kc, qc, nqb, nkb, tk_b, H, scale, beta, mean,
                                                    var, cutoff);
  else
    threshold_kernel<64><<<grid, 64, 0, stream>>>(kc, qc, nqb, nkb, tk_b, H, scale, beta, mean,
                                                  var, cutoff);
  return cudaGetLastError();
}

}  // namespace solattn
