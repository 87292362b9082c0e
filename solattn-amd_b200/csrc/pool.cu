// Block pooling of Q, K and V in one launch (replaces kernels.py:16-27 and 185-190).
//
// Work unit = (tensor, b, block, h).  A unit is handled by D threads laid out as 8 row
// groups x D/8 chunk lanes; lane c of group g loads 16 bytes (8 channels) of rows
// g, g+8, ..., g+56 (all eight 128-bit loads issued before any add), accumulating in FP32.
// The 8 group partials are combined through shared memory in group order, then divided by
// the valid row count min(64, T - 64*block) with IEEE division.  K/V means are rounded to
// BF16 (nearest even), Q means stay FP32.  Output layout is [B, H, blocks, D].  In a ragged
// launch batch b has its own key count (K/V blocks past it hold zeros).
//
// The pass is HBM-bound: it reads every Q/K/V element once (the 64 rows of a unit are
// strided by sT, each row a contiguous 2*D-byte segment) and writes 1/64 of that back.
#include "sm100.cuh"

namespace solattn {

template <int D>
__global__ void __launch_bounds__(256) pool_kernel(PoolParams p) {
  constexpr int kChunks = D / 8;          // 16-byte chunks per row
  constexpr int kUnitsPerCta = 256 / D;   // D threads per unit
  __shared__ float part[kUnitsPerCta][8][D];

  const int local_unit = threadIdx.x / D;
  const int lt = threadIdx.x % D;
  const int g = lt / kChunks;  // row group 0..7
  const int c = lt % kChunks;  // chunk lane

  int64_t unit = (int64_t)blockIdx.x * kUnitsPerCta + local_unit;
  int which = 0;
  while (which < 3 && unit >= p.units[which]) {
    unit -= p.units[which];
    ++which;
  }
  const bool active = which < 3;
  int b = 0, blk = 0, h = 0, n = 0;
  // Sums of channels (2j, 2j + 1) in packed f32x2 pairs: each lane of add.rn.f32x2 rounds like
  // __fadd_rn, so the sums are those of the scalar order with half the adds.
  uint64_t acc2[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) acc2[j] = 0ull;
  if (active) {
    const TensorView& x = p.x[which];
    const int T = p.T[which];
    // Unit indices fit 32 bits (the launcher checks), so the decode uses 32-bit division.
    const int u32 = (int)unit;
    h = u32 % p.H;
    const int r = u32 / p.H;
    blk = r % p.nb[which];
    b = r / p.nb[which];
    const int Tv = (which > 0 && p.tk_b) ? clamp_key_count(__ldg(p.tk_b + b), T, p.status)
                                         : T;  // valid rows of this batch
    n = min(kBlock, Tv - blk * kBlock);
    uint4 raw[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int row = g + 8 * i;
      if (row < n) {
        const __nv_bfloat16* src = row_ptr(x, T, b, h, blk * kBlock + row, p.status) + c * 8;
        raw[i] = __ldg(reinterpret_cast<const uint4*>(src));
      }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int row = g + 8 * i;
      if (row < n) {
        const __nv_bfloat162* v2 = reinterpret_cast<const __nv_bfloat162*>(&raw[i]);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = __bfloat1622float2(v2[j]);
          acc2[j] = sm100::f2_add(acc2[j], sm100::f2_pack(f.x, f.y));
        }
      }
    }
  }
#pragma unroll
  for (int j = 0; j < 4; ++j)
    sm100::f2_unpack(acc2[j], part[local_unit][g][c * 8 + 2 * j], part[local_unit][g][c * 8 + 2 * j + 1]);
  __syncthreads();
  if (!active) return;
  // Thread lt now owns channel lt of the unit.
  float s = 0.f;
#pragma unroll
  for (int gg = 0; gg < 8; ++gg) s = __fadd_rn(s, part[local_unit][gg][lt]);
  const float mean = n > 0 ? __fdiv_rn(s, (float)n) : 0.f;
  const int nb = p.nb[which];
  const int64_t o = (((int64_t)b * p.H + h) * nb + blk) * D + lt;
  if (which == 0) {
    reinterpret_cast<float*>(p.y[0])[o] = mean;
  } else {
    reinterpret_cast<__nv_bfloat16*>(p.y[which])[o] = __float2bfloat16_rn(mean);
  }
}

cudaError_t launch_pool(const PoolParams& p, int D, cudaStream_t stream) {
  const int64_t total = p.units[0] + p.units[1] + p.units[2];
  if (total == 0) return cudaSuccess;
  for (int i = 0; i < 3; ++i)
    if (p.units[i] > 0x7fffffff) return cudaErrorInvalidValue;  // 32-bit unit decode
  const int per_cta = 256 / D;
  const int64_t grid = (total + per_cta - 1) / per_cta;
  if (D == 128)
    pool_kernel<128><<<(unsigned)grid, 256, 0, stream>>>(p);
  else
    pool_kernel<64><<<(unsigned)grid, 256, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace solattn
