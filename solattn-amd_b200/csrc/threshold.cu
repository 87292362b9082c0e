// Key moments + Eq. 15 thresholds in one launch (replaces kernels.py:30-64, 211-215), for the
// stage-by-stage entry point solattn_threshold; the full forward folds the same work into the
// pooling kernel (pool.cu).  The arithmetic and its order are threshold.cuh's.
//
// One CTA per (b, h) and group of D / 2 q-blocks, 4 * D threads.  Every CTA of a head computes
// the head's key moments itself (one slice/pair assignment per thread), then eight threads per
// q-block form its cutoff.  The slices make the longest dependent chain nb / 8 adds instead of
// nb: at 512 key blocks the launch takes about 11 us at 3 heads and 15 us at 24, where one
// thread per channel summing all blocks in order took 13-21 us.
#include "threshold.cuh"

namespace solattn {

namespace {

template <int D>
__global__ void __launch_bounds__(4 * D) threshold_kernel(const __nv_bfloat16* __restrict__ kc,
                                                          const float* __restrict__ qc, int nqb,
                                                          int nkb, const int32_t* __restrict__ tk_b,
                                                          int H, float scale, float beta,
                                                          float* mean_out, float* var_out,
                                                          float* cutoff) {
  constexpr int kQB = 4 * D / kThrSlices;  // q-blocks per CTA (eight threads each)
  __shared__ float s_part[2][kThrSlices][D];
  __shared__ float s_mean[D];
  __shared__ float s_var[D];
  const int bh = blockIdx.y;
  // The batch's own key blocks in a ragged launch (kc rows past them are padding).
  const int nb = tk_b ? min(max((tk_b[bh / H] + kBlock - 1) / kBlock, 1), nkb) : nkb;
  head_moments<D, 4 * D>(kc + (int64_t)bh * nkb * D, nb, s_part, s_mean, s_var,
                         blockIdx.x == 0 ? mean_out + (int64_t)bh * D : nullptr,
                         blockIdx.x == 0 ? var_out + (int64_t)bh * D : nullptr);
  const int qb = blockIdx.x * kQB + (int)threadIdx.x / kThrSlices;
  const bool valid = qb < nqb;
  const float cut = qblock_cutoff<D>(qc + ((int64_t)bh * nqb + (valid ? qb : 0)) * D, s_mean,
                                     s_var, valid, scale, beta);
  if (valid && threadIdx.x % kThrSlices == 0) cutoff[(int64_t)bh * nqb + qb] = cut;
}

}  // namespace

cudaError_t launch_threshold(const __nv_bfloat16* kc, const float* qc, int BH, int H, int nqb,
                             int nkb, int D, float scale, float beta, float* mean, float* var,
                             float* cutoff, const int32_t* tk_b, cudaStream_t stream) {
  const int per_cta = 4 * D / kThrSlices;
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
