// Block pooling of Q, K and V in one launch (replaces kernels.py:16-27 and 185-190), and in the
// full forward the key moments of each head (kernels.py:30-49).
//
// Work unit = (tensor, b, block, h).  A unit is handled by D threads laid out as 8 row
// groups x D/8 chunk lanes; lane c of group g loads 16 bytes (8 channels) of rows
// g, g+8, ..., g+56 (all eight 128-bit loads issued before any add), accumulating in FP32.
// The 8 group partials are combined through shared memory in group order, then divided by
// the valid row count min(64, T - 64*block) with IEEE division.  K/V means are rounded to
// BF16 (nearest even), Q means stay FP32.  Output layout is [B, H, blocks, D].  In a ragged
// launch batch b has its own key count (K/V blocks past it hold zeros).  A CTA pools
// 256 / D consecutive blocks of one (b, h); grid row y is one tensor, K first.
//
// The pass reads every Q/K/V element once (the 64 rows of a unit are strided by sT, each row
// a contiguous 2*D-byte segment) and writes 1/64 of that back; non-gathered rows are addressed
// from one base pointer and a stride, so that the kernel is bound by its loads rather than by
// instruction issue.  With fused moments (PoolParams::k_arrive) the CTA that finishes the last
// K block of a head computes that head's mean and variance (threshold.cuh) while the Q and V
// rows still stream.
#include "threshold.cuh"

namespace solattn {

template <int D, bool kGather>
__global__ void __launch_bounds__(256, 4) pool_kernel(PoolParams p) {
  constexpr int kChunks = D / 8;          // 16-byte chunks per row
  constexpr int kUnitsPerCta = 256 / D;   // D threads per unit
  __shared__ float part[kUnitsPerCta][8][D];

  const int which = p.order[blockIdx.y];  // 0: Q, 1: K, 2: V (uniform per CTA)
  const int local_unit = threadIdx.x / D;
  const int lt = threadIdx.x % D;
  const int g = lt / kChunks;  // row group 0..7
  const int c = lt % kChunks;  // chunk lane

  // A CTA takes kUnitsPerCta consecutive blocks of one (b, h); consecutive CTAs take the next
  // head of the same rows (DRAM rows are read whole across a wave of CTAs), and with fused
  // moments the CTA finishing a head's last K block computes that head alone.
  const int nb_t = p.nb[which];
  const int groups = (nb_t + kUnitsPerCta - 1) / kUnitsPerCta;  // block groups per (b, h)
  const int cta = (int)blockIdx.x;  // < B * H * groups (the launcher checks 32 bits)
  const int hh = cta % p.H, rr = cta / p.H;
  const int bb = rr / groups, blk0 = (rr % groups) * kUnitsPerCta;
  const bool active = bb < p.B && blk0 + local_unit < nb_t && p.units[which] > 0;
  int b = 0, blk = 0, h = 0, n = 0;
  // Sums of channels (2j, 2j + 1) in packed f32x2 pairs: each lane of add.rn.f32x2 rounds like
  // __fadd_rn, so the sums are those of the scalar order with half the adds.
  uint64_t acc2[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) acc2[j] = 0ull;
  auto add_row = [&](const uint4& raw) {
    const __nv_bfloat162* v2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __bfloat1622float2(v2[j]);
      acc2[j] = sm100::f2_add(acc2[j], sm100::f2_pack(f.x, f.y));
    }
  };
  if (active) {
    const TensorView& x = p.x[which];
    const int T = p.T[which];
    h = hh;
    b = bb;
    blk = blk0 + local_unit;
    const int Tv = (which > 0 && p.tk_b) ? clamp_key_count(__ldg(p.tk_b + b), T, p.status)
                                         : T;  // valid rows of this batch
    n = min(kBlock, Tv - blk * kBlock);
    uint4 raw[8];
    if constexpr (!kGather) {
      // Rows g, g + 8, ... of the block are one stride apart: one base address, no per-row
      // index arithmetic (the kernel is bound by instruction issue, not by its loads).
      const __nv_bfloat16* base = x.ptr + (int64_t)b * x.sB +
                                  (int64_t)(blk * kBlock + g) * x.sT + (int64_t)h * x.sH + c * 8;
      const int64_t step = 8 * x.sT;
      if (n == kBlock) {
#pragma unroll
        for (int i = 0; i < 8; ++i) raw[i] = __ldg(reinterpret_cast<const uint4*>(base + i * step));
#pragma unroll
        for (int i = 0; i < 8; ++i) add_row(raw[i]);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i)
          if (g + 8 * i < n) raw[i] = __ldg(reinterpret_cast<const uint4*>(base + i * step));
#pragma unroll
        for (int i = 0; i < 8; ++i)
          if (g + 8 * i < n) add_row(raw[i]);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int row = g + 8 * i;
        if (row < n) {
          const __nv_bfloat16* src = row_ptr(x, T, b, h, blk * kBlock + row, p.status) + c * 8;
          raw[i] = __ldg(reinterpret_cast<const uint4*>(src));
        }
      }
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (g + 8 * i < n) add_row(raw[i]);
    }
  }
#pragma unroll
  for (int j = 0; j < 4; ++j)
    sm100::f2_unpack(acc2[j], part[local_unit][g][c * 8 + 2 * j], part[local_unit][g][c * 8 + 2 * j + 1]);
  __syncthreads();
  if (active) {
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
  if (!p.k_arrive || which != 1) return;  // uniform: moments are fused for K CTAs only
  // The CTA that finishes the last K unit of a head computes the head's key moments
  // (threshold.cuh) while the V units are still being pooled.
  __shared__ int s_head[1];
  __shared__ float s_mean[D];
  __shared__ float s_var[D];
  // The CTA's rows are written (barrier), then one thread makes them visible device-wide
  // (a cumulative fence) and counts the CTA's blocks in; a fence in every thread would hold
  // each K CTA until all of its stores had drained.
  __syncthreads();
  if (threadIdx.x == 0) {
    int n_active = 0;
    for (int u = 0; u < kUnitsPerCta; ++u) n_active += (blk0 + u < nb_t) ? 1 : 0;
    int head = -1;
    if (bb < p.B) {
      const int bh = bb * p.H + hh;
      __threadfence();
      if (atomicAdd(p.k_arrive + bh, n_active) + n_active == p.nb[1]) head = bh;
    }
    s_head[0] = head;
  }
  __syncthreads();
  // The shape [2][kThrSlices][D] of the moment partials fits in the unit partials' storage.
  static_assert(sizeof(part) >= sizeof(float) * 2 * kThrSlices * D, "moment partials");
  auto* s_part = reinterpret_cast<float (*)[kThrSlices][D]>(&part[0][0][0]);
  {
    const int bh = s_head[0];
    if (bh < 0) return;
    __threadfence();  // every other CTA's rows of the head are visible
    const int nkb = p.nb[1];
    const int tk = p.tk_b ? clamp_key_count(__ldg(p.tk_b + bh / p.H), p.T[1], p.status) : p.T[1];
    const int nbk = min(max((tk + kBlock - 1) / kBlock, 1), nkb);
    head_moments<D, 256>(reinterpret_cast<const __nv_bfloat16*>(p.y[1]) + (int64_t)bh * nkb * D,
                         nbk, s_part, s_mean, s_var, p.mean + (int64_t)bh * D,
                         p.var + (int64_t)bh * D);
  }
}

cudaError_t launch_pool(const PoolParams& p, int D, cudaStream_t stream) {
  const int per_cta = 256 / D;
  // x: CTAs of one tensor (per_cta consecutive blocks of one head each); y: the tensors pooled,
  // K first (CTAs past a tensor's blocks return at once).  Grid rows are dispatched in order,
  // so with the key moments fused the last K blocks -- and the moments they start -- overlap
  // the Q and V rows.
  PoolParams q = p;
  int rows = 0;
  int64_t most = 0;
  for (int t : {1, 0, 2}) {
    if (p.units[t] <= 0) continue;
    q.order[rows++] = t;
    const int64_t ctas = (int64_t)p.B * p.H * ((p.nb[t] + per_cta - 1) / per_cta);
    if (ctas > 0x7fffffff) return cudaErrorInvalidValue;  // 32-bit CTA decode
    most = ctas > most ? ctas : most;
  }
  if (rows == 0) return cudaSuccess;
  const dim3 grid((unsigned)most, (unsigned)rows);
  const bool gather = p.x[0].idx || p.x[1].idx || p.x[2].idx;
  if (D == 128) {
    if (gather) pool_kernel<128, true><<<grid, 256, 0, stream>>>(q);
    else pool_kernel<128, false><<<grid, 256, 0, stream>>>(q);
  } else {
    if (gather) pool_kernel<64, true><<<grid, 256, 0, stream>>>(q);
    else pool_kernel<64, false><<<grid, 256, 0, stream>>>(q);
  }
  return cudaGetLastError();
}

}  // namespace solattn
