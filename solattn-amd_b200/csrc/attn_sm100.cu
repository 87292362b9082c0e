// Fused routed attention on the Blackwell data path (replaces `_sol`, kernels.py:101-182).
//
// One CTA = one 128-row query tile = two 64-row q-blocks (qb0 = 2*y, qb0 + 1) of one (b, h),
// 128 threads, two CTAs per SM (256 TMEM columns and ~104 KB of shared memory each) so that one
// CTA's softmax overlaps the other CTA's tensor-core work.
//
// Per CTA:
//   1. Prologue: TMEM allocation (warp 0), routing of every key block for both q-blocks into
//      shared bitmasks (common.cuh:route_selected, bit-identical to the CPU restatement), and a
//      tile list in shared memory built by warp 0:
//        - centroid tiles (128 pooled keys kc/vc) holding a block unselected by either q-block:
//          entry -(t + 1);
//        - exact tiles: the union of both q-blocks' exact blocks, two blocks per tile in
//          increasing order: entry a | (b << 16), b = kNoBlock (0x7FFF) when the tile has one
//          block.  Every exact entry is non-negative (block ids < kMaxKeyBlocks < 0x7FFF), so
//          the sign alone tells the two kinds apart.
//   2. Tile loop, all four warps in lockstep (warp w owns TMEM lanes / rows 32w..32w+31),
//      thread 0 issuing TMA and tcgen05.mma:
//        S = Q K^T  (SMEM x SMEM -> TMEM, FP32)      -> S_FULL
//        next K tile TMA (the S MMA has released the K buffer)
//        softmax per row: column mask/bias for the row's q-block, FP32 online softmax with lazy
//        rescaling, P (BF16) written over S in TMEM
//        O += P V  (TMEM x SMEM -> TMEM)               -> O_DONE, then the next V tile TMA
//   3. Epilogue O / l -> BF16 global stores; TMEM released.
#include <cudaTypedefs.h>

#include "sm100.cuh"

namespace solattn {

namespace {

using namespace sm100;

constexpr int kRows = 128;     // query rows per CTA
constexpr int kKeys = 128;     // keys per tile
constexpr int kThreads = 128;  // 4 warps
constexpr uint32_t kTmemCols = 256;
constexpr int kBoxBytes = kRows * 128;  // one 128-row x 64-column BF16 box (16 KB)
constexpr int kMaxKeyBlocks = 4096;     // tile list capacity (T <= 262144 keys)
constexpr int kNoBlock = 0x7FFF;        // second half of a one-block exact tile

enum Bar { Q_FULL, K_FULL, V_FULL, S_FULL, O_DONE, DRAIN, NBARS };

template <int D>
struct Layout {
  static constexpr int kTile = kRows * D * 2;  // bytes of a 128 x D BF16 tile
  static constexpr int kQ = 0;
  static constexpr int kK = kTile;
  static constexpr int kV = 2 * kTile;
  static constexpr int kBars = 3 * kTile;
  static constexpr int kMisc = kBars + NBARS * 8;  // [0] TMEM address [1] abort [2] tiles
  static constexpr int kQbar = kMisc + 16;         // float [2][D]
  static constexpr int kMask = kQbar + 2 * D * 4;  // uint32 [2][nwords]
  __host__ __device__ static int tiles_offset(int nwords) { return kMask + 2 * nwords * 4; }
  __host__ __device__ static int max_tiles(int nkb) { return (nkb + kKeys - 1) / kKeys + (nkb + 1) / 2; }
  static size_t bytes(int nkb) {
    const int nwords = (nkb + 31) / 32;
    size_t n = 1024 + (size_t)tiles_offset(nwords) + (size_t)max_tiles(nkb) * 4;
    // At most two CTAs per SM: each holds 256 of the SM's 512 TMEM columns.
    return n < 80 * 1024 ? 80 * 1024 : n;
  }
};

__device__ __forceinline__ uint32_t valid_word(int w, int nkb) {
  const int lo = 32 * w;
  if (lo + 32 <= nkb) return 0xffffffffu;
  if (lo >= nkb) return 0u;
  return (1u << (nkb - lo)) - 1u;
}

// Bounded wait that ignores the abort flag (drains in-flight copies / MMAs on exit).
__device__ __forceinline__ void mbar_wait_quiet(uint32_t bar, uint32_t parity) {
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > kWaitLimitCycles) return;
  }
}

}  // namespace

namespace {

// Issues the TMA loads of one K or V tile (tile-list entry `e`) into `dst` on barrier `full`.
// Centroid tiles read 128 pooled rows as two 64-row boxes (a second half starting past the
// last centroid repeats the first; its columns are masked).  Exact tiles read two 64-key blocks
// (a one-block tile repeats its block; the repeat is masked).  All rows are inside the tensors.
static_assert(kMaxKeyBlocks < kNoBlock, "block ids must stay below the one-block sentinel");
template <int D>
__device__ __forceinline__ void load_kv_tile(uint32_t dst, const CUtensorMap* tile_map,
                                             const CUtensorMap* cent_map, uint32_t full, int e,
                                             int nkb, int h, int b) {
  mbar_expect_tx(full, (uint32_t)(kKeys * D * 2));
  if (e < 0) {
    const int c0 = kKeys * (-e - 1);
    const int c1 = c0 + kBlock < nkb ? c0 + kBlock : c0;
#pragma unroll
    for (int j = 0; j < D / 64; ++j) {
      tma_load_4d(dst + j * kBoxBytes, cent_map, full, 64 * j, c0, h, b);
      tma_load_4d(dst + j * kBoxBytes + kBlock * 128, cent_map, full, 64 * j, c1, h, b);
    }
  } else {
    const int a = e & 0xffff;
    const int hi = (e >> 16) & 0xffff;
    const int bb = hi == kNoBlock ? a : hi;
#pragma unroll
    for (int j = 0; j < D / 64; ++j) {
      tma_load_4d(dst + j * kBoxBytes, tile_map, full, 64 * j, kBlock * a, h, b);
      tma_load_4d(dst + j * kBoxBytes + kBlock * 128, tile_map, full, 64 * j, kBlock * bb, h, b);
    }
  }
}

// Every lane waits; the warp agrees on the outcome (false after a timeout or an abort).
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                          int32_t* status) {
  const bool ok = mbar_wait(bar, parity, abort_flag, status);
  return __all_sync(0xffffffffu, ok);
}

}  // namespace

template <int D>
__global__ void __launch_bounds__(kThreads, 2)
    attn_sm100_kernel(const AttnParams p, const __grid_constant__ CUtensorMap tmQ,
                      const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                      const __grid_constant__ CUtensorMap tmKC,
                      const __grid_constant__ CUtensorMap tmVC) {
  using L = Layout<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t sQ = sbase + L::kQ, sK = sbase + L::kK, sV = sbase + L::kV;
  const uint32_t bar0 = sbase + L::kBars;
  uint32_t* misc = reinterpret_cast<uint32_t*>(smem + L::kMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(misc + 1);
  float* sQbar = reinterpret_cast<float*>(smem + L::kQbar);
  uint32_t* sMask = reinterpret_cast<uint32_t*>(smem + L::kMask);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // Query tiles of one head are adjacent in launch order so that the CTAs resident at any time
  // share that head's K/V (16 MB at T=32k) in L2.
  const int bh = blockIdx.y;
  const int b = bh / p.H, h = bh % p.H;
  const int qb0 = 2 * blockIdx.x;
  const bool has1 = qb0 + 1 < p.nqb;
  const int nwords = (p.nkb + 31) / 32;
  int* sTiles = reinterpret_cast<int*>(smem + L::tiles_offset(nwords));

  if (tid == 0) {
    mbar_init(bar0 + 8 * Q_FULL, 1);
    mbar_init(bar0 + 8 * K_FULL, 1);
    mbar_init(bar0 + 8 * V_FULL, 1);
    mbar_init(bar0 + 8 * S_FULL, 1);
    mbar_init(bar0 + 8 * O_DONE, 1);
    mbar_init(bar0 + 8 * DRAIN, 1);
    misc[1] = 0;
    misc[2] = 0;
    mbar_fence_init();
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(misc), kTmemCols);
    // Give up the allocation permit at once: while a CTA holds it, no further CTA that needs
    // TMEM is launched on this SM, and two CTAs per SM are what hides the softmax.
    tmem_relinquish();
  }
  if (p.force == 0) {
    for (int i = tid; i < 2 * D; i += kThreads) {
      const int qb = qb0 + i / D;
      sQbar[i] = qb < p.nqb ? p.qc[((int64_t)bh * p.nqb + qb) * D + (i % D)] : 0.f;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = misc[0];

  if (tid == 0) {
    tma_prefetch(&tmQ);
    tma_prefetch(&tmK);
    tma_prefetch(&tmV);
    tma_prefetch(&tmKC);
    tma_prefetch(&tmVC);
    mbar_expect_tx(bar0 + 8 * Q_FULL, L::kTile);
    for (int j = 0; j < D / 64; ++j)
      tma_load_4d(sQ + j * kBoxBytes, &tmQ, bar0 + 8 * Q_FULL, 64 * j, qb0 * kBlock, h, b);
  }

  // ---- routing of both q-blocks into shared bitmasks ----
  // Lane kb of a warp reads centroid row kb once and forms both q-blocks' proxies from it (the
  // arithmetic of common.cuh:route_selected, bit for bit); one ballot per q-block per 32 blocks.
  const __nv_bfloat16* kc_bh = p.kc + (int64_t)bh * p.nkb * D;
  for (int wi = warp; wi < nwords; wi += kThreads / 32) {
    const int kb = wi * 32 + lane;
    const int kbc = kb < p.nkb ? kb : p.nkb - 1;  // clamped: every address stays in range
    bool sel[2] = {false, false};
    if (p.force == 0) {
      float d0, d1;
      routing_dot2(sQbar, sQbar + D, kc_bh + (int64_t)kbc * D, D, d0, d1);
      const float cut0 = p.cutoff[(int64_t)bh * p.nqb + qb0];
      const float cut1 = has1 ? p.cutoff[(int64_t)bh * p.nqb + qb0 + 1] : 0.f;
      sel[0] = __fmul_rn(d0, p.scale) > cut0;
      sel[1] = __fmul_rn(d1, p.scale) > cut1;
    }
#pragma unroll
    for (int qsel = 0; qsel < 2; ++qsel) {
      const int qb = qb0 + qsel;
      bool s_ = false;
      if (kb < p.nkb && qb < p.nqb) s_ = route_rules(p, sel[qsel], b, qb, kb);
      const uint32_t bal = __ballot_sync(0xffffffffu, s_);
      if (lane == 0) {
        sMask[qsel * nwords + wi] = bal;
        if (p.debug_mask && qb < p.nqb) p.debug_mask[((int64_t)bh * p.nqb + qb) * nwords + wi] = bal;
      }
    }
  }
  __syncthreads();

  // ---- tile list (warp 0) and exact-block counts ----
  if (warp == 0) {
    const uint32_t* m0 = sMask;
    const uint32_t* m1 = sMask + nwords;
    int n = 0;
    const int nct = p.force == 1 ? 0 : (p.nkb + kKeys - 1) / kKeys;
    for (int t0 = 0; t0 < nct; t0 += 32) {
      const int t = t0 + lane;
      bool useful = false;
      if (t < nct) {
        for (int wi = 4 * t; wi < 4 * t + 4 && wi < nwords; ++wi) {
          const uint32_t v = valid_word(wi, p.nkb);
          const uint32_t w0 = m0[wi], w1 = m1[wi];
          if ((~w0 & v) || (has1 && (~w1 & v))) useful = true;
        }
      }
      const uint32_t bal = __ballot_sync(0xffffffffu, useful);
      if (useful) sTiles[n + __popc(bal & ((1u << lane) - 1u))] = -(t + 1);
      n += __popc(bal);
    }
    // Exact blocks of the union in increasing order; block of rank r goes to the low (r even)
    // or high (r odd) 16 bits of entry n + r/2.
    uint16_t* half = reinterpret_cast<uint16_t*>(sTiles + n);
    int r = 0;
    for (int w0 = 0; w0 < nwords; w0 += 32) {
      const int wi = w0 + lane;
      uint32_t bits = 0u;
      if (wi < nwords) bits = m0[wi] | (has1 ? m1[wi] : 0u);
      const int cnt = __popc(bits);
      int incl = cnt;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      int rank = r + incl - cnt;
      while (bits) {
        const int bit = __ffs(bits) - 1;
        bits &= bits - 1u;
        half[rank++] = (uint16_t)(32 * wi + bit);
      }
      r += __shfl_sync(0xffffffffu, incl, 31);
    }
    __syncwarp();
    if (lane == 0) {
      if (r & 1) half[r] = (uint16_t)kNoBlock;  // one-block last tile
      misc[2] = (uint32_t)(n + (r + 1) / 2);
    }
    if (lane < 2 && p.counts && qb0 + lane < p.nqb) {
      int c = 0;
      for (int i = 0; i < nwords; ++i) c += __popc(sMask[lane * nwords + i]);
      p.counts[((int64_t)b * p.nqb + qb0 + lane) * p.H + h] = c;
    }
  }
  __syncthreads();
  const int ntiles = (int)misc[2];

  // ---- tile loop ----
  const uint32_t lane_base = (uint32_t)(warp * 32) << 16;  // warp w reads TMEM lanes 32w..32w+31
  const uint32_t tS = tmem, tO = tmem + kKeys;
  const uint32_t tSr = tS + lane_base, tOr = tO + lane_base;
  const int row = warp * 32 + lane;
  const int qsel = row >> 6;
  const bool row_ok = qsel == 0 || has1;
  const uint32_t* mymask = sMask + qsel * nwords;
  const float sl2 = p.scale_log2;
  const float last_bias = log2f((float)(p.Tk - (p.nkb - 1) * kBlock));
  const int last_word = (p.nkb - 1) >> 5;
  constexpr uint32_t idS = idesc_bf16(kRows, kKeys, false);
  constexpr uint32_t idO = idesc_bf16(kRows, D, true);

  int k_issued = 0, v_issued = 0;  // thread 0 only
  if (tid == 0 && ntiles > 0) {
    load_kv_tile<D>(sK, &tmK, &tmKC, bar0 + 8 * K_FULL, sTiles[0], p.nkb, h, b);
    load_kv_tile<D>(sV, &tmV, &tmVC, bar0 + 8 * V_FULL, sTiles[0], p.nkb, h, b);
    k_issued = v_issued = 1;
  }
  float m_run = -INFINITY, l_run = 0.f;
  int done = 0;
  for (int i = 0; i < ntiles; ++i) {
    const int entry = sTiles[i];
    // -- thread 0: S = Q K^T --
    if (tid == 0 && !*abort_flag) {
      bool ok = true;
      if (i == 0) ok = mbar_wait(bar0 + 8 * Q_FULL, 0, abort_flag, p.status);
      if (ok && i > 0) {
        // P V of the previous tile is complete: S/P columns and the V buffer are free.
        ok = mbar_wait(bar0 + 8 * O_DONE, (i - 1) & 1, abort_flag, p.status);
        if (ok) {
          load_kv_tile<D>(sV, &tmV, &tmVC, bar0 + 8 * V_FULL, entry, p.nkb, h, b);
          ++v_issued;
        }
      }
      if (ok) ok = mbar_wait(bar0 + 8 * K_FULL, i & 1, abort_flag, p.status);
      if (ok) {
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const uint32_t off = (uint32_t)((k >> 2) * kBoxBytes + (k & 3) * 32);
          mma_ss(tS, smem_desc_sw128(sQ + off, 16, 1024), smem_desc_sw128(sK + off, 16, 1024), idS,
                 k > 0 ? 1u : 0u);
        }
        mma_commit(bar0 + 8 * S_FULL);
      }
    }
    // -- all: softmax of this tile --
    if (warp_wait(bar0 + 8 * S_FULL, i & 1, abort_flag, p.status)) {
      tc_fence_after();
      if (tid == 0 && i + 1 < ntiles) {  // the S MMA has released the K buffer
        load_kv_tile<D>(sK, &tmK, &tmKC, bar0 + 8 * K_FULL, sTiles[i + 1], p.nkb, h, b);
        ++k_issued;
      }
      uint32_t s[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(tSr + 32 * c, s[c]);
      tmem_wait_ld();
      float mt = -INFINITY;
      if (entry < 0) {
        const int t = -entry - 1;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int wi = 4 * t + c;
          const uint32_t word = mymask[wi < nwords ? wi : nwords - 1];  // index kept in range
          const uint32_t approx = row_ok ? (~word & valid_word(wi, p.nkb)) : 0u;
          const int last_j = wi == last_word ? ((p.nkb - 1) & 31) : 32;
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const float bias = j == last_j ? last_bias : 6.f;  // log2(valid length)
            const float v =
                ((approx >> j) & 1u) ? fmaf(__uint_as_float(s[c][j]), sl2, bias) : -INFINITY;
            s[c][j] = __float_as_uint(v);
            mt = fmaxf(mt, v);
          }
        }
      } else {
        const int a = entry & 0xffff;
        const int hi = (entry >> 16) & 0xffff;
        const bool single = hi == kNoBlock;
        const int bb = single ? a : hi;
        const uint32_t wa = mymask[a >> 5], wb = mymask[bb >> 5];
        const bool va = row_ok && ((wa >> (a & 31)) & 1u);
        const bool vb = row_ok && !single && ((wb >> (bb & 31)) & 1u);
        const int la = va ? min(kBlock, p.Tk - a * kBlock) : 0;
        const int lb = vb ? min(kBlock, p.Tk - bb * kBlock) : 0;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int lim = c < 2 ? la : lb;
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const float v = ((c & 1) * 32 + j) < lim ? __uint_as_float(s[c][j]) * sl2 : -INFINITY;
            s[c][j] = __float_as_uint(v);
            mt = fmaxf(mt, v);
          }
        }
      }
      // Lazy rescaling: the running max only moves when a row's max grows by more than 8
      // (a factor 256), so P stays <= 256 and O is rarely touched; O and l share the max.
      const float m_new = fmaxf(m_run, mt);
      bool need = false;
      float alpha = 1.f;
      if (m_run == -INFINITY) {
        m_run = m_new;  // nothing accumulated yet: O and l are zero for this row
      } else if (m_new > m_run + 8.f) {
        need = true;
        alpha = fast_exp2(m_run - m_new);
        m_run = m_new;
      }
      if (__any_sync(0xffffffffu, need)) {
        // P V of the previous tile completed before this tile's S was issued.
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          uint32_t o[32];
          tmem_ld32(tOr + 32 * c, o);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; ++j) o[j] = __float_as_uint(__uint_as_float(o[j]) * alpha);
          tmem_st32(tOr + 32 * c, o);
        }
        l_run *= alpha;
      }
      const float m_use = m_run == -INFINITY ? 0.f : m_run;
      float sum = 0.f;
      uint32_t pk[2][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          const float p0 = fast_exp2(__uint_as_float(s[c][j]) - m_use);
          const float p1 = fast_exp2(__uint_as_float(s[c][j + 1]) - m_use);
          sum += p0 + p1;
          pk[c >> 1][(c & 1) * 16 + j / 2] = pack_bf16(p0, p1);
        }
      }
      l_run += sum;
      tmem_st32(tSr, pk[0]);  // P (BF16 pairs) overwrites S columns 0..63
      tmem_st32(tSr + 32, pk[1]);
      tmem_wait_st();
    }
    tc_fence_before();
    __syncthreads();
    if (*abort_flag) break;  // read by every thread after the same barrier: uniform
    // -- thread 0: O += P V --
    if (tid == 0) {
      tc_fence_after();
      if (mbar_wait(bar0 + 8 * V_FULL, i & 1, abort_flag, p.status)) {
#pragma unroll
        for (int k = 0; k < kKeys / 16; ++k)
          mma_ts(tO, tS + (uint32_t)(k * 8),
                 smem_desc_sw128(sV + (uint32_t)(k * 16 * 128), kBoxBytes, 1024), idO,
                 (i > 0 || k > 0) ? 1u : 0u);
        mma_commit(bar0 + 8 * O_DONE);
      }
    }
    done = i + 1;
  }

  // ---- epilogue ----
  if (ntiles > 0 && done == ntiles &&
      warp_wait(bar0 + 8 * O_DONE, (ntiles - 1) & 1, abort_flag, p.status)) {
    tc_fence_after();
    const float inv = 1.f / l_run;
    const int grow = qb0 * kBlock + row;
    __nv_bfloat16* dst = p.out + (((int64_t)b * p.Tq + grow) * p.H + h) * D;
#pragma unroll 1
    for (int c = 0; c < D / 32; ++c) {
      uint32_t o[32];
      tmem_ld32(tOr + 32 * c, o);
      tmem_wait_ld();
      if (grow < p.Tq) {
        uint4 v4[4];
        uint32_t* w32 = reinterpret_cast<uint32_t*>(v4);
#pragma unroll
        for (int j = 0; j < 16; ++j)
          w32[j] = pack_bf16(__uint_as_float(o[2 * j]) * inv, __uint_as_float(o[2 * j + 1]) * inv);
        uint4* d4 = reinterpret_cast<uint4*>(dst + 32 * c);
#pragma unroll
        for (int j = 0; j < 4; ++j) d4[j] = v4[j];
      }
    }
  }

  // ---- drain and release ----
  if (tid == 0) {
    mma_commit(bar0 + 8 * DRAIN);  // every MMA of this CTA has completed once this fires
    mbar_wait_quiet(bar0 + 8 * DRAIN, 0);
    if (*abort_flag) {  // never leave while a bulk copy may still write shared memory
      mbar_wait_quiet(bar0 + 8 * Q_FULL, 0);
      if (k_issued > 0) mbar_wait_quiet(bar0 + 8 * K_FULL, (k_issued - 1) & 1);
      if (v_issued > 0) mbar_wait_quiet(bar0 + 8 * V_FULL, (v_issued - 1) & 1);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------- host side
namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

// BF16 tensor map with 128-byte swizzle; dims/strides listed innermost first (strides in
// bytes for dims 1..rank-1).
bool make_map(CUtensorMap* map, const void* base, uint32_t rank, const cuuint64_t* dims,
              const cuuint64_t* strides, const cuuint32_t* box) {
  PFN_cuTensorMapEncodeTiled_v12000 fn = encode_fn();
  if (!fn) return false;
  const cuuint32_t elem[5] = {1, 1, 1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, const_cast<void*>(base), dims, strides,
            box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 4-D map over a BTHD view [B, T, H, D] with box {64, rows, 1, 1}.
bool make_bthd_map(CUtensorMap* map, const TensorView& x, int B, int T, int H, int D,
                   uint32_t rows) {
  cuuint64_t sb = (cuuint64_t)x.sB * 2;
  if (B == 1 || sb == 0) sb = ((cuuint64_t)x.sT * 2 * (cuuint64_t)T + 15) & ~cuuint64_t(15);
  const cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)T, (cuuint64_t)H, (cuuint64_t)B};
  const cuuint64_t strides[3] = {(cuuint64_t)x.sT * 2, (cuuint64_t)x.sH * 2, sb};
  const cuuint32_t box[4] = {64, rows, 1, 1};
  return make_map(map, x.ptr, 4, dims, strides, box);
}

// 4-D map over the pooled [B, H, nkb, D] statistics with box {64, 64, 1, 1}.
bool make_pooled_map(CUtensorMap* map, const __nv_bfloat16* base, int B, int H, int nkb, int D) {
  const cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)nkb, (cuuint64_t)H, (cuuint64_t)B};
  const cuuint64_t strides[3] = {(cuuint64_t)D * 2, (cuuint64_t)nkb * D * 2,
                                 (cuuint64_t)H * nkb * D * 2};
  const cuuint32_t box[4] = {64, (cuuint32_t)kBlock, 1, 1};
  return make_map(map, base, 4, dims, strides, box);
}

template <int D>
cudaError_t launch_sm100(const AttnParams& p, cudaStream_t stream) {
  if (p.nkb > kMaxKeyBlocks) return cudaErrorInvalidValue;
  CUtensorMap tmQ, tmK, tmV, tmKC, tmVC;
  if (!make_bthd_map(&tmQ, p.q, p.B, p.Tq, p.H, D, kRows) ||
      !make_bthd_map(&tmK, p.k, p.B, p.Tk, p.H, D, kBlock) ||
      !make_bthd_map(&tmV, p.v, p.B, p.Tk, p.H, D, kBlock) ||
      !make_pooled_map(&tmKC, p.kc, p.B, p.H, p.nkb, D) ||
      !make_pooled_map(&tmVC, p.vc, p.B, p.H, p.nkb, D))
    return cudaErrorInvalidValue;
  const size_t smem = Layout<D>::bytes(p.nkb);
  cudaError_t err = cudaFuncSetAttribute(attn_sm100_kernel<D>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (err != cudaSuccess) return err;
  dim3 grid((p.nqb + 1) / 2, p.B * p.H);
  attn_sm100_kernel<D><<<grid, kThreads, smem, stream>>>(p, tmQ, tmK, tmV, tmKC, tmVC);
  return cudaGetLastError();
}

}  // namespace

bool attn_sm100_supported(const AttnParams& p) { return p.nkb <= kMaxKeyBlocks; }

cudaError_t launch_attn_sm100(const AttnParams& p, int D, cudaStream_t stream) {
  return D == 128 ? launch_sm100<128>(p, stream) : launch_sm100<64>(p, stream);
}

}  // namespace solattn
