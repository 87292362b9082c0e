// Routing pass: the exact-block bitmask of every (b, h, q-block) (kernels.py:130-143,
// reference.py:41-51), written before the fused attention kernel runs so that the attention
// CTAs start on their tiles at once.
//
// One CTA per (b, h) and group of kRouteQB q-blocks, 256 threads.  A warp stages its 32
// centroid rows in shared memory with coalesced 16-byte cp.async copies (double-buffered: the
// next 64 dims or the next 32 rows are in flight while these are used), then lane kb forms the proxies
// of all the group's q-blocks from row kb,
// with exactly the arithmetic of common.cuh:routing_dot (eight partial sums over d = 8i + j,
// one fused multiply-add per term, combined pairwise), so the decisions are bit-identical to the
// per-CTA routing of the mma.sync kernel.  One ballot per q-block per 32 key blocks gives a
// mask word: masks[((b * H + h) * nqb + qb) * nwords + kb / 32], bit kb % 32.  The word after
// the last mask word is the fused attention kernel's work counter; the pass zeroes it.  When a
// list buffer is given the pass also builds every q-block pair's tile list for the fused kernel
// (common.cuh: build_item_list) and writes the exact-block counts, so that no attention CTA
// spends time on either between two items.  With at least two items per attention CTA (the
// launcher leaves AttnParams::arrive null otherwise) the last CTA of a head to finish its lists
// then sorts the head's q-block pairs (after the sink pairs) by tile count, longest first, for
// the fused kernel's work claims (AttnParams::order): handed out longest first within each head,
// the last items of a launch are its shortest, which shortens the tail in which some CTAs
// still run their last item while the others have none left.  Ties keep no fixed order; the
// results do not depend on the order in which items run.
#include "threshold.cuh"

namespace solattn {

namespace {

constexpr int kRouteQB = 4;
constexpr int kRouteThreads = 256;
constexpr int kRowBytes = 144;                // staged centroid row (64 dims) + 16 bytes of skew
constexpr int kStageBytes = 32 * kRowBytes;   // one warp's 32 rows
constexpr int kRouteSmem = (kRouteThreads / 32) * 2 * kStageBytes;  // double-buffered, dynamic
// The head sort reuses the staging memory: keys of up to kMaxOrderItems pairs and a histogram of
// up to kMaxOrderBins tile counts (item_list_capacity(4096) + 1 = 4169 bins).  A head with more
// pairs keeps the natural order.
constexpr int kMaxOrderItems = 8192;
constexpr int kMaxOrderBins = 4352;
static_assert(4 * (kMaxOrderItems + kMaxOrderBins) <= kRouteSmem, "sort buffers exceed staging");

// Block-wide exclusive scan of hist[0, bins) taken from the top bin down: afterwards hist[b]
// holds the number of entries in bins above b (256 threads).
__device__ __forceinline__ void scan_descending(int* hist, int bins, int* warp_sums) {
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int per = (bins + kRouteThreads - 1) / kRouteThreads;
  const int r0 = t * per, r1 = min(bins, r0 + per);  // reversed positions r: bin bins - 1 - r
  int local = 0;
  for (int r = r0; r < r1; ++r) local += hist[bins - 1 - r];
  int incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) warp_sums[warp] = incl;
  __syncthreads();
  int before = 0;
  for (int w = 0; w < warp; ++w) before += warp_sums[w];
  int run = before + incl - local;
  for (int r = r0; r < r1; ++r) {
    const int c = hist[bins - 1 - r];
    hist[bins - 1 - r] = run;
    run += c;
  }
}

// Called by every thread of a routing CTA after its tile lists are written: the last CTA of the
// head sorts the head's pairs and resets the head's arrival counter.
__device__ __forceinline__ void order_head_items(const AttnParams& p, int bh, uint8_t* smem) {
  __shared__ int s_last;
  __shared__ int s_warp_sums[kRouteThreads / 32];
  __syncthreads();  // this CTA's lists and headers are written; one thread makes them visible
                    // device-wide (a cumulative fence) before the CTA counts itself in
  if (threadIdx.x == 0) {
    __threadfence();
    s_last = atomicAdd(p.arrive + bh, 1) == (int)gridDim.x - 1;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();  // every other CTA's headers are visible
  const int npairs = (p.nqb + 1) / 2;
  const int sink = min(npairs, (p.q_sink_blocks + 1) / 2);
  const int rest = npairs - sink;
  const int bins = item_list_capacity(p.nkb) + 1;  // tile counts 0 .. capacity
  if (rest > 0 && rest <= kMaxOrderItems && bins <= kMaxOrderBins) {
    int* key = reinterpret_cast<int*>(smem);
    int* hist = key + kMaxOrderItems;
    const int64_t stride = item_list_stride(p.nkb);
    const uint8_t* head = p.lists + (int64_t)bh * npairs * stride;
    // Each key is read once (a stale header still yields a permutation of the pairs).
    for (int i = threadIdx.x; i < rest; i += kRouteThreads)
      key[i] = min(max(__ldcg(reinterpret_cast<const int*>(head + (int64_t)(sink + i) * stride)), 0),
                   bins - 1);
    for (int b = threadIdx.x; b < bins; b += kRouteThreads) hist[b] = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < rest; i += kRouteThreads) atomicAdd(&hist[key[i]], 1);
    __syncthreads();
    scan_descending(hist, bins, s_warp_sums);
    __syncthreads();
    int32_t* order = p.order + (int64_t)bh * npairs;
    for (int i = threadIdx.x; i < rest; i += kRouteThreads)
      order[atomicAdd(&hist[key[i]], 1)] = sink + i;
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence();
      p.stamp[bh] = p.epoch;
    }
  }
  if (threadIdx.x == 0) p.arrive[bh] = 0;  // every CTA of the head has arrived
}

template <int D>
__global__ void __launch_bounds__(kRouteThreads, 2) route_kernel(const AttnParams p) {
  __shared__ __align__(16) float sq[kRouteQB][D];
  __shared__ float scut[kRouteQB];
  const int bh = blockIdx.y;
  const int b = bh / p.H;
  const int qb_lo = blockIdx.x * kRouteQB;
  const int nq = min(kRouteQB, p.nqb - qb_lo);
  const int nwords = (p.nkb + 31) / 32;
  const int nkb_b = (key_count(p, b) + kBlock - 1) / kBlock;  // this batch's key blocks
  constexpr int kMaxWords = 4096 / 32;  // the fused kernel's limit of 4096 key blocks
  __shared__ uint32_t smask[kRouteQB][kMaxWords];
  if (blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0)
    p.masks[(int64_t)p.B * p.H * p.nqb * nwords] = 0u;
  for (int i = threadIdx.x; i < kRouteQB * D; i += kRouteThreads) {
    const int j = i / D;
    sq[j][i % D] =
        (p.force == 0 && j < nq) ? p.qc[((int64_t)bh * p.nqb + qb_lo + j) * D + (i % D)] : 0.f;
  }
  // Threshold mode reads the cutoffs, or (fused threshold) forms them below from the key
  // moments staged here.
  const bool fused_cut = p.force == 0 && p.mean != nullptr;
  __shared__ float s_mean[D];
  __shared__ float s_var[D];
  if (fused_cut) {
    for (int d = threadIdx.x; d < D; d += kRouteThreads) {
      s_mean[d] = p.mean[(int64_t)bh * D + d];
      s_var[d] = p.var[(int64_t)bh * D + d];
    }
  } else if (threadIdx.x < kRouteQB) {
    scut[threadIdx.x] = (p.force == 0 && (int)threadIdx.x < nq)
                            ? p.cutoff[(int64_t)bh * p.nqb + qb_lo + threadIdx.x]
                            : 0.f;
  }
  __syncthreads();

  // Per-warp staging of its 32 centroid rows, 64 dims at a time, double-buffered: the 16-byte
  // cp.async copies of the next chunk (next half, or next word) are in flight while this one is
  // computed.  Rows are 144 bytes apart so that the lanes' 16-byte reads of 32 different rows
  // take the minimum 4 wavefronts.
  extern __shared__ __align__(16) uint8_t route_smem[];
  const __nv_bfloat16* kc_bh = p.kc + (int64_t)bh * p.nkb * D;
  const int lane = threadIdx.x & 31, warp_id = threadIdx.x >> 5;
  uint8_t* my_stage = route_smem + warp_id * 2 * kStageBytes;
  constexpr int kHalves = D / 64;
  // This warp's chunks: t = m * kHalves + half for its m-th word w = warp_id + 8 m.
  const int my_words = nwords > warp_id ? (nwords - warp_id + 7) / 8 : 0;
  const int nchunks = p.force == 0 ? my_words * kHalves : 0;
  auto issue = [&](int t) {
    if (t < nchunks) {
      const int w = warp_id + (kRouteThreads / 32) * (t / kHalves), half = t % kHalves;
      uint8_t* dst = my_stage + (t & 1) * kStageBytes;
#pragma unroll
      for (int u = 0; u < 8; ++u) {  // 8 consecutive lanes copy one row's 128 bytes
        const int idx = 32 * u + lane, r = idx >> 3, c = idx & 7;
        const int kr = min(32 * w + r, nkb_b - 1);  // clamped: every address stays in range
        cp_async16(smem_u32(dst + r * kRowBytes + 16 * c), kc_bh + (int64_t)kr * D + 64 * half + 8 * c,
                   16);
      }
    }
    cp_async_commit();
  };
  issue(0);
  // The cutoffs this warp compares against, in registers.  Fused threshold: every warp forms
  // the group's four cutoffs itself from the q-block means already staged in shared memory
  // (eight lanes per q-block, threshold.cuh) while its first centroid chunk is in flight, so
  // that no warp waits for another.
  float cut[kRouteQB];
  if (fused_cut) {
    static_assert(kRouteQB * kThrSlices == 32, "one warp forms the group's cutoffs");
    const int j = lane / kThrSlices;
    const bool valid = j < nq;
    const float c = qblock_cutoff<D, true>(&sq[valid ? j : 0][0], s_mean, s_var, valid, p.scale,
                                           p.beta);
#pragma unroll
    for (int i = 0; i < kRouteQB; ++i) cut[i] = __shfl_sync(0xffffffffu, c, kThrSlices * i);
    if (warp_id == 0 && valid && lane % kThrSlices == 0 && p.cutoff_out)
      p.cutoff_out[(int64_t)bh * p.nqb + qb_lo + j] = c;
  } else {
#pragma unroll
    for (int i = 0; i < kRouteQB; ++i) cut[i] = scut[i];
  }
  int t = 0;
  // Warp-uniform loop over 32-block words.
  for (int w = warp_id; w < nwords; w += kRouteThreads / 32) {
    const int kb = 32 * w + lane;
    // Partial sums of dims 8i + e in pairs (e, e + 1) of packed f32x2 registers: each lane of
    // fma.rn.f32x2 is one fused multiply-add rounded once, exactly like fmaf, so the sums are
    // those of the scalar order with a quarter of the instructions of separate multiplies and
    // adds.
    uint64_t part2[kRouteQB][4];
#pragma unroll
    for (int j = 0; j < kRouteQB; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) part2[j][e] = 0ull;
    if (p.force == 0) {
#pragma unroll 1
      for (int half = 0; half < kHalves; ++half, ++t) {
        issue(t + 1);
        cp_async_wait<1>();  // this lane's copies of chunk t have landed
        __syncwarp();        // and every lane's
        const uint8_t* cur = my_stage + (t & 1) * kStageBytes;
#pragma unroll 4
      for (int ii = 0; ii < 8; ++ii) {
        const int i = 8 * half + ii;
        const uint4 raw = *reinterpret_cast<const uint4*>(cur + lane * kRowBytes + 16 * ii);
        const __nv_bfloat162* k2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
        uint64_t kf2[4];  // dims (8i + 2e, 8i + 2e + 1)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(k2[e]);
          kf2[e] = sm100::f2_pack(f.x, f.y);
        }
#pragma unroll
        for (int j = 0; j < kRouteQB; ++j) {
          // The q-block means of dims 8i..8i+7 as four packed pairs: two 16-byte broadcast reads.
          const ulonglong2 qa = *reinterpret_cast<const ulonglong2*>(&sq[j][8 * i]);
          const ulonglong2 qb4 = *reinterpret_cast<const ulonglong2*>(&sq[j][8 * i + 4]);
          part2[j][0] = sm100::f2_fma(qa.x, kf2[0], part2[j][0]);
          part2[j][1] = sm100::f2_fma(qa.y, kf2[1], part2[j][1]);
          part2[j][2] = sm100::f2_fma(qb4.x, kf2[2], part2[j][2]);
          part2[j][3] = sm100::f2_fma(qb4.y, kf2[3], part2[j][3]);
        }
      }
        __syncwarp();  // every lane is done with this stage before chunk t + 2 overwrites it
      }
    }
#pragma unroll
    for (int j = 0; j < kRouteQB; ++j) {
      if (j >= nq) break;
      const int qb = qb_lo + j;
      float part[8];
#pragma unroll
      for (int e = 0; e < 4; ++e) sm100::f2_unpack(part2[j][e], part[2 * e], part[2 * e + 1]);
      const float dot = __fadd_rn(__fadd_rn(__fadd_rn(part[0], part[1]),
                                            __fadd_rn(part[2], part[3])),
                                  __fadd_rn(__fadd_rn(part[4], part[5]),
                                            __fadd_rn(part[6], part[7])));
      bool sel = false;
      if (kb < nkb_b) sel = route_rules(p, p.force == 0 && __fmul_rn(dot, p.scale) > cut[j], b, qb, kb);
      const uint32_t bal = __ballot_sync(0xffffffffu, sel);
      if (lane == 0) {
        p.masks[((int64_t)bh * p.nqb + qb) * nwords + w] = bal;
        if (nwords <= kMaxWords) smask[j][w] = bal;
      }
    }
  }
  cp_async_wait<0>();  // (only empty groups can be pending here)
  if (!p.lists || nwords > kMaxWords) return;
  __syncthreads();
  // Warp j: the tile list of the group's q-block pair j (q-blocks qb_lo + 2j, qb_lo + 2j + 1).
  const int warp = threadIdx.x >> 5;
  const int qb0 = qb_lo + 2 * warp;
  if (warp < kRouteQB / 2 && qb0 < p.nqb) {
    const bool has1 = qb0 + 1 < p.nqb;
    uint8_t* item =
        p.lists + ((int64_t)bh * ((p.nqb + 1) / 2) + (qb0 >> 1)) * item_list_stride(p.nkb);
    int real;
    const int n = build_item_list(smask[2 * warp], smask[2 * warp + 1], has1, nwords, nkb_b,
                                  p.force, reinterpret_cast<int16_t*>(item + 16), lane, real);
    if (lane == 0) *reinterpret_cast<int4*>(item) = make_int4(n, real, 0, 0);
    if (lane < 2 && p.counts && qb0 + lane < p.nqb) {
      int c = 0;
      for (int i = 0; i < nwords; ++i) c += __popc(smask[2 * warp + lane][i]);
      p.counts[((int64_t)b * p.nqb + qb0 + lane) * p.H + bh % p.H] = c;
    }
  }
  if (p.arrive) order_head_items(p, bh, route_smem);
}

}  // namespace

cudaError_t launch_route(const AttnParams& p, int D, cudaStream_t stream) {
  dim3 grid((p.nqb + kRouteQB - 1) / kRouteQB, p.B * p.H);
  cudaError_t err;
  if (D == 128) {
    err = cudaFuncSetAttribute(route_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               kRouteSmem);
    if (err != cudaSuccess) return err;
    route_kernel<128><<<grid, kRouteThreads, kRouteSmem, stream>>>(p);
  } else {
    err = cudaFuncSetAttribute(route_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               kRouteSmem);
    if (err != cudaSuccess) return err;
    route_kernel<64><<<grid, kRouteThreads, kRouteSmem, stream>>>(p);
  }
  return cudaGetLastError();
}

}  // namespace solattn
