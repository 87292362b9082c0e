// Key moments and Eq. 15 cutoffs of one (b, h) (kernels.py:30-64): the arithmetic shared by the
// threshold kernel (threshold.cu, one launch over every head) and the pooling kernel's per-head
// tail (pool.cu, the last pooling CTA of a head), so that both produce the same bits.
//
// Order (restated in oracle/kernel_order.py):
//   * moments: slice j = 0..7 of channel pair c sums rows j, j + 8, j + 16, ... of kc[b, h]
//     (x and x * x, packed f32x2, row order); the eight slice sums of a channel are combined as
//     ((s0 + s1) + (s2 + s3)) + ((s4 + s5) + (s6 + s7)); mean = s1 / n,
//     var = max(s2 / n - mean^2, 0) with every block weighted equally (kernels.py:40-47);
//   * cutoff of a q-block: eight lanes, lane e summing channels e, e + 8, ... of qc * mean and
//     (qc * qc) * var in order, the partial sums combined in the same tree (a butterfly of
//     shuffles: every lane gets the tree's value because FP32 addition is commutative), then
//     cutoff = (mu + beta * sqrt(sg)) * scale in natural-log units.
// Every operation is rounded to nearest without contraction.  Loads go through L2 (ld.global.cg):
// the pooling kernel's tail reads rows that other CTAs of the same launch wrote.
#pragma once

#include "sm100.cuh"

namespace solattn {

constexpr int kThrSlices = 8;   // row slices of the moment sums, partial sums of the cutoffs
constexpr int kThrUnroll = 16;  // rows per slice in flight

__device__ __forceinline__ float tree8(const float* p) {
  return __fadd_rn(__fadd_rn(__fadd_rn(p[0], p[1]), __fadd_rn(p[2], p[3])),
                   __fadd_rn(__fadd_rn(p[4], p[5]), __fadd_rn(p[6], p[7])));
}

// Moments of kc_bh (nb valid rows of D channels) with kThreads threads (thread index t):
// thread t takes the slice/pair assignments a = t + kThreads * k, k < kPer, and sums them side
// by side; then threads t < D combine the slices into s_mean / s_var (and mean_out / var_out
// when given).  Ends with a __syncthreads; every thread of the block must call it.
template <int D, int kThreads>
__device__ __forceinline__ void head_moments(const __nv_bfloat16* kc_bh, int nb,
                                             float (*s_part)[kThrSlices][D], float* s_mean,
                                             float* s_var, float* mean_out, float* var_out) {
  constexpr int kPairs = D / 2;
  constexpr int kPer = kThrSlices * kPairs / kThreads;
  static_assert(kPer * kThreads == kThrSlices * kPairs, "threads must divide the assignments");
  const int t = threadIdx.x;
  const __nv_bfloat162* base = reinterpret_cast<const __nv_bfloat162*>(kc_bh);
  uint64_t s1[kPer], s2[kPer];
#pragma unroll
  for (int k = 0; k < kPer; ++k) s1[k] = s2[k] = 0ull;
  for (int m0 = 0; m0 * kThrSlices < nb; m0 += kThrUnroll) {
    __nv_bfloat162 x[kPer][kThrUnroll];
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      const int a = t + kThreads * k, c = a % kPairs, j = a / kPairs;
#pragma unroll
      for (int u = 0; u < kThrUnroll; ++u) {
        const int r = (m0 + u) * kThrSlices + j;
        x[k][u] = r < nb ? __ldcg(base + (int64_t)r * kPairs + c) : __float2bfloat162_rn(0.f);
      }
    }
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      const int j = (t + kThreads * k) / kPairs;
#pragma unroll
      for (int u = 0; u < kThrUnroll; ++u) {
        if ((m0 + u) * kThrSlices + j < nb) {
          const float2 f = __bfloat1622float2(x[k][u]);
          const uint64_t v = sm100::f2_pack(f.x, f.y);
          s1[k] = sm100::f2_add(s1[k], v);
          s2[k] = sm100::f2_add(s2[k], sm100::f2_mul(v, v));
        }
      }
    }
  }
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    const int a = t + kThreads * k, c = a % kPairs, j = a / kPairs;
    sm100::f2_unpack(s1[k], s_part[0][j][2 * c], s_part[0][j][2 * c + 1]);
    sm100::f2_unpack(s2[k], s_part[1][j][2 * c], s_part[1][j][2 * c + 1]);
  }
  __syncthreads();
  if (t < D) {
    float a[kThrSlices], b[kThrSlices];
#pragma unroll
    for (int j = 0; j < kThrSlices; ++j) {
      a[j] = s_part[0][j][t];
      b[j] = s_part[1][j][t];
    }
    const float n = (float)nb;
    const float mean = __fdiv_rn(tree8(a), n);
    const float var = fmaxf(__fsub_rn(__fdiv_rn(tree8(b), n), __fmul_rn(mean, mean)), 0.f);
    s_mean[t] = mean;
    s_var[t] = var;
    if (mean_out) {
      mean_out[t] = mean;
      var_out[t] = var;
    }
  }
  __syncthreads();
}

// The cutoff of the q-block whose means start at qrow (global memory, or shared memory when
// kSharedRow), from the eight lanes e = lane % 8 of an aligned lane octet (all 32 lanes of the
// warp must call it; `valid` false gives a lane zero partial sums, and its octet's result is
// not used).
template <int D, bool kSharedRow = false>
__device__ __forceinline__ float qblock_cutoff(const float* qrow, const float* s_mean,
                                               const float* s_var, bool valid, float scale,
                                               float beta) {
  const int e = threadIdx.x % kThrSlices;
  float mu = 0.f, sg = 0.f;
  if (valid) {
    float qv[D / kThrSlices];
#pragma unroll
    for (int i = 0; i < D / kThrSlices; ++i)
      qv[i] = kSharedRow ? qrow[kThrSlices * i + e] : __ldcg(qrow + kThrSlices * i + e);
#pragma unroll
    for (int i = 0; i < D / kThrSlices; ++i) {
      const int d = kThrSlices * i + e;
      mu = __fadd_rn(mu, __fmul_rn(qv[i], s_mean[d]));
      sg = __fadd_rn(sg, __fmul_rn(__fmul_rn(qv[i], qv[i]), s_var[d]));
    }
  }
#pragma unroll
  for (int o = 1; o < kThrSlices; o <<= 1) {
    mu = __fadd_rn(mu, __shfl_xor_sync(0xffffffffu, mu, o));
    sg = __fadd_rn(sg, __shfl_xor_sync(0xffffffffu, sg, o));
  }
  return __fmul_rn(__fadd_rn(mu, __fmul_rn(beta, __fsqrt_rn(sg))), scale);
}

}  // namespace solattn
