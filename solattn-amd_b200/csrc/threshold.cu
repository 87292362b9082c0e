// Key moments + Eq. 15 thresholds in one launch (replaces kernels.py:30-64, 211-215).
//
// One CTA per (b, h) and group of D / 2 q-blocks, 4 * D threads.  Every CTA of a head computes
// the head's key moments itself (no second launch, no cross-CTA exchange):
//   * thread (j, c), slice j = 0..7 and channel pair c, sums rows j, j + 8, j + 16, ... of
//     kc[b, h] for channels 2c and 2c + 1, x and x * x, in row order; the loads of kUnroll
//     rows are in flight at once (a warp reads 128 contiguous bytes of one row per load);
//   * the eight slice sums of a channel are combined as ((s0 + s1) + (s2 + s3)) +
//     ((s4 + s5) + (s6 + s7)); mean = s1 / n and var = max(s2 / n - mean^2, 0) with every
//     block weighted equally (kernels.py:40-47).
// Cutoffs: eight threads per q-block, thread e summing channels e, e + 8, e + 16, ... of
// qc * mean and (qc * qc) * var in order; the eight partial sums are combined in the same tree
// (a butterfly of shuffles, which gives every lane the tree's value because FP32 addition is
// commutative) and
//   cutoff = (mu + beta * sqrt(sg)) * scale
// in natural-log units (the routing pass compares the unscaled proxy dot times scale against
// it).  Every operation is rounded to nearest without contraction (__f*_rn, packed
// add.rn / mul.rn.f32x2), so a CPU restatement in FP32 reproduces the bits.  The slices make
// the longest dependent chain nb / 8 adds instead of nb: at 512 key blocks the launch is a few
// microseconds, where one thread per channel summing all blocks in order took 13-21 us.
#include "sm100.cuh"

namespace solattn {

namespace {

constexpr int kSlices = 8;   // row slices of the moment sums (and partial sums of the cutoffs)
constexpr int kUnroll = 16;  // rows per slice in flight

__device__ __forceinline__ float tree8(const float* p) {
  return __fadd_rn(__fadd_rn(__fadd_rn(p[0], p[1]), __fadd_rn(p[2], p[3])),
                   __fadd_rn(__fadd_rn(p[4], p[5]), __fadd_rn(p[6], p[7])));
}

template <int D>
__global__ void __launch_bounds__(4 * D) threshold_kernel(const __nv_bfloat16* __restrict__ kc,
                                                          const float* __restrict__ qc, int nqb,
                                                          int nkb, const int32_t* __restrict__ tk_b,
                                                          int H, float scale, float beta,
                                                          float* mean_out, float* var_out,
                                                          float* cutoff) {
  constexpr int kPairs = D / 2;            // channel pairs
  constexpr int kQB = 4 * D / kSlices;     // q-blocks per CTA (eight threads each)
  __shared__ float s_part[2][kSlices][D];  // slice sums of x and x * x
  __shared__ float s_mean[D];
  __shared__ float s_var[D];
  const int bh = blockIdx.y;
  const int t = threadIdx.x;
  // The batch's own key blocks in a ragged launch (kc rows past them are padding).
  const int nb = tk_b ? min(max((tk_b[bh / H] + kBlock - 1) / kBlock, 1), nkb) : nkb;

  {
    const int c = t % kPairs, j = t / kPairs;
    const __nv_bfloat162* col =
        reinterpret_cast<const __nv_bfloat162*>(kc + (int64_t)bh * nkb * D) + c;
    uint64_t s1 = 0ull, s2 = 0ull;  // channels (2c, 2c + 1)
    for (int r0 = j; r0 < nb; r0 += kSlices * kUnroll) {
      __nv_bfloat162 x[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int r = r0 + kSlices * u;
        x[u] = r < nb ? __ldg(col + (int64_t)r * kPairs) : __float2bfloat162_rn(0.f);
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        if (r0 + kSlices * u < nb) {
          const float2 f = __bfloat1622float2(x[u]);
          const uint64_t v = sm100::f2_pack(f.x, f.y);
          s1 = sm100::f2_add(s1, v);
          s2 = sm100::f2_add(s2, sm100::f2_mul(v, v));
        }
      }
    }
    sm100::f2_unpack(s1, s_part[0][j][2 * c], s_part[0][j][2 * c + 1]);
    sm100::f2_unpack(s2, s_part[1][j][2 * c], s_part[1][j][2 * c + 1]);
  }
  __syncthreads();
  if (t < D) {
    float a[kSlices], b[kSlices];
#pragma unroll
    for (int j = 0; j < kSlices; ++j) {
      a[j] = s_part[0][j][t];
      b[j] = s_part[1][j][t];
    }
    const float n = (float)nb;
    const float mean = __fdiv_rn(tree8(a), n);
    const float var = fmaxf(__fsub_rn(__fdiv_rn(tree8(b), n), __fmul_rn(mean, mean)), 0.f);
    s_mean[t] = mean;
    s_var[t] = var;
    if (blockIdx.x == 0) {
      mean_out[(int64_t)bh * D + t] = mean;
      var_out[(int64_t)bh * D + t] = var;
    }
  }
  __syncthreads();

  const int e = t % kSlices;
  const int qb = blockIdx.x * kQB + t / kSlices;  // eight consecutive lanes per q-block
  const bool valid = qb < nqb;
  const float* qrow = qc + ((int64_t)bh * nqb + (valid ? qb : 0)) * D;
  float mu = 0.f, sg = 0.f;
  if (valid) {
#pragma unroll
    for (int i = 0; i < D / kSlices; ++i) {
      const int d = kSlices * i + e;
      const float qv = __ldg(qrow + d);
      mu = __fadd_rn(mu, __fmul_rn(qv, s_mean[d]));
      sg = __fadd_rn(sg, __fmul_rn(__fmul_rn(qv, qv), s_var[d]));
    }
  }
#pragma unroll
  for (int o = 1; o < kSlices; o <<= 1) {
    mu = __fadd_rn(mu, __shfl_xor_sync(0xffffffffu, mu, o));
    sg = __fadd_rn(sg, __shfl_xor_sync(0xffffffffu, sg, o));
  }
  if (valid && e == 0)
    cutoff[(int64_t)bh * nqb + qb] = __fmul_rn(__fadd_rn(mu, __fmul_rn(beta, __fsqrt_rn(sg))), scale);
}

}  // namespace

cudaError_t launch_threshold(const __nv_bfloat16* kc, const float* qc, int BH, int H, int nqb,
                             int nkb, int D, float scale, float beta, float* mean, float* var,
                             float* cutoff, const int32_t* tk_b, cudaStream_t stream) {
  const int per_cta = 4 * D / kSlices;
  const dim3 grid((nqb + per_cta - 1) / per_cta, BH);
  if (D == 128)
    threshold_kernel<128><<<grid, 4 * 128, 0, stream>>>(kc, qc, nqb, nkb, tk_b, H, scale, beta,
                                                        mean, var, cutoff);
  else
    threshold_kernel<64><<<grid, 4 * 64, 0, stream>>>(kc, qc, nqb, nkb, tk_b, H, scale, beta,
                                                      mean, var, cutoff);
  return cudaGetLastError();
}

}  // namespace solattn
