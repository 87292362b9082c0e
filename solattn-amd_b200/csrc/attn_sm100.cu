// Fused routed attention on the Blackwell data path (replaces `_sol`, kernels.py:101-182).
//
// One CTA = one 128-row query tile = two 64-row q-blocks (qb0 = 2*x, qb0 + 1) of one (b, h);
// 192 threads, two CTAs per SM (256 TMEM columns and ~100 KB of shared memory each).
//
// Tiles hold 64 keys: one exact key block, or 64 pooled centroids.  The tile list (shared
// memory, built by warp 0 after routing) holds first every 64-centroid group that still has a
// block unselected by either q-block (entry -(t + 1)), then every block of the union of both
// q-blocks' exact sets in increasing order (entry kb >= 0).  A row whose q-block did not select
// an exact block sees it as -inf; a centroid whose block is exact for the row's q-block too.
//
// Warp roles:
//   warps 0-3  softmax: warp w owns TMEM lanes / tile rows 32w..32w+31 (warps 0-1 q-block qb0,
//              warps 2-3 qb0 + 1).  Per tile: wait S_FULL, tcgen05.ld S, mask/bias, FP32 online
//              softmax with lazy rescaling, P (BF16) written over its S buffer, arrive P_FULL.
//              A warp whose q-block does not use the tile writes P = 0 without reading S.
//              Epilogue O / l -> BF16.
//   warp 4     S issue (the whole warp runs the loop, lane 0 issues): S_i = Q K_i^T into TMEM
//              buffer i % 2 once P_{i-2} V_{i-2} has freed it; refills the K ring (2 slots)
//              when S_{i-1} has completed (K_EMPTY).
//   warp 5     P V issue: O += P_i V_i once the softmax warps have written P_i; loads Q and
//              refills the V ring when P_i V_i has completed (PV_DONE).
//   One thread can issue a tcgen05.mma only about every 100 cycles, so S (8 MMAs of N=64 per
//   tile) and P V (4 MMAs of N=D) come from two threads; the tensor core works on S_{i+1} and
//   P_{i-1} V_{i-1} while the softmax warps work on tile i.
// TMEM: S buffers at columns [0, 64) and [64, 128) (P packed into the first 32 columns of its
// buffer), O at [128, 128 + D).
#include <cudaTypedefs.h>

#include "sm100.cuh"

namespace solattn {

namespace {

using namespace sm100;

constexpr int kRows = 128;         // query rows per CTA
constexpr int kKeys = 64;          // keys per tile
constexpr int kSoftmaxWarps = 4;
constexpr int kSWarp = 4;   // S = Q K^T issue and the K ring
constexpr int kPVWarp = 5;  // O += P V issue, the V ring and Q
constexpr int kThreads = 192;
constexpr uint32_t kTmemCols = 256;
constexpr int kQBox = kRows * 128;   // one 128-row x 64-column BF16 box of Q (16 KB)
constexpr int kKVBox = kKeys * 128;  // one 64-row x 64-column BF16 box of K or V (8 KB)
constexpr int kMaxKeyBlocks = 4096;  // tile list capacity (T <= 262144 keys)

// Barriers: slot-indexed pairs for the 2-deep rings.
enum Bar {
  Q_FULL,
  K_FULL0, K_FULL1, K_EMPTY0, K_EMPTY1, V_FULL0, V_FULL1,
  S_FULL0, S_FULL1, P_FULL0, P_FULL1, PV_DONE0, PV_DONE1,
  DRAIN_S, DRAIN_PV, NBARS
};

template <int D>
struct Layout {
  static constexpr int kQTile = kRows * D * 2;   // 128 x D BF16
  static constexpr int kKVTile = kKeys * D * 2;  // 64 x D BF16
  static constexpr int kQ = 0;
  static constexpr int kK = kQTile;                 // 2 slots
  static constexpr int kV = kK + 2 * kKVTile;       // 2 slots
  static constexpr int kBars = kV + 2 * kKVTile;
  static constexpr int kMisc = kBars + NBARS * 8;   // [0] TMEM address [1] abort [2] tiles
  static constexpr int kQbar = kMisc + 16;          // float [2][D]
  static constexpr int kMask = kQbar + 2 * D * 4;   // uint32 [2][nwords]
  __host__ __device__ static int tiles_offset(int nwords) { return kMask + 2 * nwords * 4; }  // int16
  __host__ __device__ static int max_tiles(int nkb) { return (nkb + kKeys - 1) / kKeys + nkb; }
  static size_t bytes(int nkb) {
    const int nwords = (nkb + 31) / 32;
    size_t n = 1024 + (size_t)tiles_offset(nwords) + (size_t)max_tiles(nkb) * 2;
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

// Every lane waits; the warp agrees on the outcome (false after a timeout or an abort).
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                          int32_t* status) {
  const bool ok = mbar_wait(bar, parity, abort_flag, status);
  return __all_sync(0xffffffffu, ok);
}

// TMA loads of one K or V tile (tile-list entry e) into `dst` on barrier `full`: 64 centroid rows
// of the pooled map (e < 0) or the 64 rows of key block e.  Rows past the end of a tensor are
// filled with zeros by the TMA unit and masked by the softmax.
template <int D>
__device__ __forceinline__ void load_kv_tile(uint32_t dst, const CUtensorMap* tile_map,
                                             const CUtensorMap* cent_map, uint32_t full, int e,
                                             int h, int b) {
  mbar_expect_tx(full, (uint32_t)(kKeys * D * 2));
  const bool cent = e < 0;
  const int row = cent ? kKeys * (-e - 1) : kBlock * e;
#pragma unroll
  for (int j = 0; j < D / 64; ++j)
    tma_load_4d(dst + j * kKVBox, cent ? cent_map : tile_map, full, 64 * j, row, h, b);
}

// Row max of 64 scores with three-input max instructions: eight independent chains.
__device__ __forceinline__ float row_max64(const uint32_t (&s)[2][32]) {
  float m[8];
#pragma unroll
  for (int g = 0; g < 8; ++g) {
    const int c = g >> 2, j = (g & 3) * 8;
    const float a = fmax3(__uint_as_float(s[c][j]), __uint_as_float(s[c][j + 1]),
                          __uint_as_float(s[c][j + 2]));
    const float b2 = fmax3(__uint_as_float(s[c][j + 3]), __uint_as_float(s[c][j + 4]),
                           __uint_as_float(s[c][j + 5]));
    m[g] = fmax3(a, b2, fmaxf(__uint_as_float(s[c][j + 6]), __uint_as_float(s[c][j + 7])));
  }
  return fmax3(fmax3(m[0], m[1], m[2]), fmax3(m[3], m[4], m[5]), fmaxf(m[6], m[7]));
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
  auto bar = [bar0](int i) { return bar0 + 8u * (uint32_t)i; };
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
  int16_t* sTiles = reinterpret_cast<int16_t*>(smem + L::tiles_offset(nwords));

  if (tid == 0) {
    for (int i = 0; i < NBARS; ++i)
      mbar_init(bar(i), (i == P_FULL0 || i == P_FULL1) ? kSoftmaxWarps : 1);
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

  if (tid == kPVWarp * 32) {  // Q starts loading before the routing prologue
    tma_prefetch(&tmQ);
    tma_prefetch(&tmK);
    tma_prefetch(&tmV);
    tma_prefetch(&tmKC);
    tma_prefetch(&tmVC);
    mbar_expect_tx(bar(Q_FULL), L::kQTile);
    for (int j = 0; j < D / 64; ++j)
      tma_load_4d(sQ + j * kQBox, &tmQ, bar(Q_FULL), 64 * j, qb0 * kBlock, h, b);
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
        for (int wi = 2 * t; wi < 2 * t + 2 && wi < nwords; ++wi) {
          const uint32_t v = valid_word(wi, p.nkb);
          const uint32_t w0 = m0[wi], w1 = m1[wi];
          if ((~w0 & v) || (has1 && (~w1 & v))) useful = true;
        }
      }
      const uint32_t bal = __ballot_sync(0xffffffffu, useful);
      if (useful) sTiles[n + __popc(bal & ((1u << lane) - 1u))] = (int16_t)(-(t + 1));
      n += __popc(bal);
    }
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
      int rank = n + r + incl - cnt;
      while (bits) {
        const int bit = __ffs(bits) - 1;
        bits &= bits - 1u;
        sTiles[rank++] = (int16_t)(32 * wi + bit);
      }
      r += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) misc[2] = (uint32_t)(n + r);
    if (lane < 2 && p.counts && qb0 + lane < p.nqb) {
      int c = 0;
      for (int i = 0; i < nwords; ++i) c += __popc(sMask[lane * nwords + i]);
      p.counts[((int64_t)b * p.nqb + qb0 + lane) * p.H + h] = c;
    }
  }
  __syncthreads();
  const int ntiles = (int)misc[2];

  if (warp == kSWarp) {
    // ------------------------------------------------------------------ S issue + K ring
    // The whole warp runs the loop so that descriptors and addresses stay warp-uniform; lane 0
    // issues every copy, MMA and commit (a commit tracks the MMAs of its own thread).  S and
    // P V are issued by two different warps: one thread can issue a tcgen05.mma only every
    // ~100 cycles, more than an M=128 N=64 MMA computes.
    constexpr uint32_t idS = idesc_bf16(kRows, kKeys, false);
    constexpr uint64_t kSlotStep = (uint64_t)(L::kKVTile >> 4);
    const uint64_t dQ = smem_desc_sw128(sQ, 16, 1024);
    const uint64_t dK = smem_desc_sw128(sK, 16, 1024);
    int k_loads0 = 0, k_loads1 = 0;  // copies issued per slot (for the drain after an abort)
    if (lane == 0) {
      for (int t = 0; t < 2 && t < ntiles; ++t) {
        load_kv_tile<D>(sK + t * L::kKVTile, &tmK, &tmKC, bar(K_FULL0 + t), sTiles[t], h, b);
        if (t) ++k_loads1; else ++k_loads0;
      }
    }
    bool ok = warp_wait(bar(Q_FULL), 0, abort_flag, p.status);
    for (int i = 0; ok && i < ntiles; ++i) {
      const int sl = i & 1;
      const uint32_t ph = (uint32_t)(i >> 1) & 1u;
      if (i >= 1 && i + 1 < ntiles) {
        // K slot (i + 1) % 2 is free once S_{i-1} has completed.
        const int fs = (i - 1) & 1;
        ok = warp_wait(bar(K_EMPTY0 + fs), (uint32_t)((i - 1) >> 1) & 1u, abort_flag, p.status);
        if (!ok) break;
        if (lane == 0) {
          load_kv_tile<D>(sK + fs * L::kKVTile, &tmK, &tmKC, bar(K_FULL0 + fs), sTiles[i + 1], h, b);
          if (fs) ++k_loads1; else ++k_loads0;
        }
      }
      // S_i = Q K_i^T into S buffer i % 2, once K_i has landed and P_{i-2} V_{i-2} (the last
      // reader of that buffer) has completed.
      ok = warp_wait(bar(K_FULL0 + sl), ph, abort_flag, p.status) &&
           (i < 2 || warp_wait(bar(PV_DONE0 + sl), ph ^ 1u, abort_flag, p.status));
      if (!ok) break;
      tc_fence_after();
      if (lane == 0) {
        const uint64_t kd = dK + (uint64_t)sl * kSlotStep;
        const uint32_t tS = tmem + (uint32_t)(kKeys * sl);
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const uint64_t off = (uint64_t)(((k >> 2) * kQBox + (k & 3) * 32) >> 4);
          const uint64_t offk = (uint64_t)(((k >> 2) * kKVBox + (k & 3) * 32) >> 4);
          mma_ss(tS, dQ + off, kd + offk, idS, k > 0 ? 1u : 0u);
        }
        mma_commit(bar(S_FULL0 + sl));
        mma_commit(bar(K_EMPTY0 + sl));
      }
      __syncwarp();
    }
    if (lane == 0) {
      // Every MMA of this thread has completed once DRAIN_S fires; no copy may still be writing
      // shared memory when the CTA leaves.
      mma_commit(bar(DRAIN_S));
      mbar_wait_quiet(bar(DRAIN_S), 0);
      if (*abort_flag) {
        if (k_loads0) mbar_wait_quiet(bar(K_FULL0), (uint32_t)(k_loads0 - 1) & 1u);
        if (k_loads1) mbar_wait_quiet(bar(K_FULL1), (uint32_t)(k_loads1 - 1) & 1u);
      }
    }
    __syncwarp();
  } else if (warp == kPVWarp) {
    // ------------------------------------------------------------------ P V issue + V ring + Q
    constexpr uint32_t idO = idesc_bf16(kRows, D, true);
    constexpr uint64_t kSlotStep = (uint64_t)(L::kKVTile >> 4);
    const uint64_t dV = smem_desc_sw128(sV, kKVBox, 1024);
    const uint32_t tO = tmem + 128;
    int v_loads0 = 0, v_loads1 = 0;
    if (lane == 0) {
      for (int t = 0; t < 2 && t < ntiles; ++t) {
        load_kv_tile<D>(sV + t * L::kKVTile, &tmV, &tmVC, bar(V_FULL0 + t), sTiles[t], h, b);
        if (t) ++v_loads1; else ++v_loads0;
      }
    }
    bool ok = true;
    for (int i = 0; i < ntiles; ++i) {
      // O += P_i V_i
      const int sl = i & 1;
      const uint32_t ph = (uint32_t)(i >> 1) & 1u;
      ok = warp_wait(bar(P_FULL0 + sl), ph, abort_flag, p.status) &&
           warp_wait(bar(V_FULL0 + sl), ph, abort_flag, p.status);
      if (!ok) break;
      tc_fence_after();
      if (lane == 0) {
        const uint64_t vd = dV + (uint64_t)sl * kSlotStep;
        const uint32_t tP = tmem + (uint32_t)(kKeys * sl);
#pragma unroll
        for (int k = 0; k < kKeys / 16; ++k)
          mma_ts(tO, tP + (uint32_t)(8 * k), vd + (uint64_t)((k * 16 * 128) >> 4), idO,
                 (i > 0 || k > 0) ? 1u : 0u);
        mma_commit(bar(PV_DONE0 + sl));
      }
      __syncwarp();
      if (i + 2 < ntiles) {
        // V slot i % 2 is free once P_i V_i has completed.
        ok = warp_wait(bar(PV_DONE0 + sl), ph, abort_flag, p.status);
        if (!ok) break;
        if (lane == 0) {
          load_kv_tile<D>(sV + sl * L::kKVTile, &tmV, &tmVC, bar(V_FULL0 + sl), sTiles[i + 2], h, b);
          if (sl) ++v_loads1; else ++v_loads0;
        }
      }
    }
    if (lane == 0) {
      mma_commit(bar(DRAIN_PV));
      mbar_wait_quiet(bar(DRAIN_PV), 0);
      if (*abort_flag) {
        mbar_wait_quiet(bar(Q_FULL), 0);
        if (v_loads0) mbar_wait_quiet(bar(V_FULL0), (uint32_t)(v_loads0 - 1) & 1u);
        if (v_loads1) mbar_wait_quiet(bar(V_FULL1), (uint32_t)(v_loads1 - 1) & 1u);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ softmax warps
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;  // warp w reads TMEM lanes 32w..
    const uint32_t tOr = tmem + 128 + lane_base;
    const int row = warp * 32 + lane;
    const int qsel = warp >> 1;                    // warps 0-1: qb0, warps 2-3: qb0 + 1
    const bool warp_rows = qsel == 0 || has1;      // the warp's q-block exists
    const uint32_t* mymask = sMask + qsel * nwords;
    const float sl2 = p.scale_log2;
    const uint64_t sl2x2 = f2_pack(sl2, sl2);
    const uint64_t six2 = f2_pack(6.f, 6.f);       // log2(64): bias of a full block's centroid
    const int last_len = p.Tk - (p.nkb - 1) * kBlock;
    const float last_bias = log2f((float)last_len);
    const int last_col = (p.nkb - 1) & 63;         // column of the last centroid in its group
    const int last_group = (p.nkb - 1) >> 6;
    float m_run = -INFINITY, l_run = 0.f;
    int i = 0;
    bool ok = true;
    for (; i < ntiles; ++i) {
      const int sl = i & 1;
      // Tile metadata first: these shared-memory reads overlap the wait for S.  Every value
      // below is warp-uniform (one q-block per warp).
      const int entry = sTiles[i];
      const bool centroid = entry < 0;
      uint32_t approx0 = 0u, approx1 = 0u;  // centroid columns this q-block uses
      int len = 0;                          // valid keys of an exact block it selected
      if (centroid) {
        const int t = -entry - 1;  // 2t < nwords since t <= (nkb - 1) / 64
        if (warp_rows) {
          approx0 = ~mymask[2 * t] & valid_word(2 * t, p.nkb);
          if (2 * t + 1 < nwords) approx1 = ~mymask[2 * t + 1] & valid_word(2 * t + 1, p.nkb);
        }
      } else if (warp_rows && ((mymask[entry >> 5] >> (entry & 31)) & 1u)) {
        len = min(kBlock, p.Tk - entry * kBlock);
      }
      const bool active = centroid ? (approx0 | approx1) != 0u : len > 0;
      if (!warp_wait(bar(S_FULL0 + sl), (uint32_t)(i >> 1) & 1u, abort_flag, p.status)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t tSr = tmem + (uint32_t)(kKeys * sl) + lane_base;
      if (!active) {
        // The tile contributes nothing to these rows: P = 0, the running max and sum stay.
        uint32_t z[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) z[j] = 0u;
        tmem_st32(tSr, z);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(P_FULL0 + sl));
        continue;
      }
      uint32_t s[2][32];
      tmem_ld32(tSr, s[0]);
      tmem_ld32(tSr + 32, s[1]);
      tmem_wait_ld();
      float m_tile, k_mul;
      if (centroid) {
        // Centroid logits in log2 units, s * scale_log2 + log2(len), and -inf where the block is
        // exact for this q-block (or past the last block).
        const int t = -entry - 1;
        if (t == last_group && last_len != kBlock) {
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            const uint32_t approx = c ? approx1 : approx0;
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const float bias = (32 * c + j) == last_col ? last_bias : 6.f;
              const float v = ((approx >> j) & 1u) ? fmaf(__uint_as_float(s[c][j]), sl2, bias)
                                                   : -INFINITY;
              s[c][j] = __float_as_uint(v);
            }
          }
        } else {
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            const uint32_t approx = c ? approx1 : approx0;
#pragma unroll
            for (int j = 0; j < 32; j += 2) {
              float v0, v1;
              f2_unpack(f2_fma(f2_pack(__uint_as_float(s[c][j]), __uint_as_float(s[c][j + 1])),
                               sl2x2, six2),
                        v0, v1);
              s[c][j] = __float_as_uint(((approx >> j) & 1u) ? v0 : -INFINITY);
              s[c][j + 1] = __float_as_uint(((approx >> (j + 1)) & 1u) ? v1 : -INFINITY);
            }
          }
        }
        m_tile = row_max64(s);
        k_mul = 1.f;
      } else {
        // Exact tiles keep raw scores: max(s) * scale_log2 equals max(s * scale_log2) bit for
        // bit (the scale is positive) and the scale is folded into the exponent's FMA.
        if (len < kBlock) {
#pragma unroll
          for (int c = 0; c < 2; ++c)
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (32 * c + j >= len) s[c][j] = __float_as_uint(-INFINITY);
        }
        m_tile = row_max64(s) * sl2;
        k_mul = sl2;
      }
      // Lazy rescaling: the running max only moves when a row's max grows by more than 8
      // (a factor 256), so P stays <= 256 and O is rarely touched; O and l share the max.
      const float m_new = fmaxf(m_run, m_tile);
      bool need = false;
      float alpha = 1.f;
      if (m_run == -INFINITY) {
        m_run = m_new;  // nothing accumulated yet: O and l are zero for this row
      } else if (m_new > m_run + 8.f) {
        need = true;
        alpha = fast_exp2(m_run - m_new);
        l_run *= alpha;  // before this tile's sum, which uses the new max
        m_run = m_new;
      }
      const float m_use = m_run == -INFINITY ? 0.f : m_run;
      // p = exp2(s * k_mul - m_use), two lanes per FMA; sums in four packed accumulators.
      const uint64_t kmul2 = f2_pack(k_mul, k_mul), negm2 = f2_pack(-m_use, -m_use);
      uint64_t acc[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[j] = 0ull;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t pk[16];
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          const uint64_t x2 =
              f2_fma(f2_pack(__uint_as_float(s[c][j]), __uint_as_float(s[c][j + 1])), kmul2, negm2);
          float x0, x1;
          f2_unpack(x2, x0, x1);
          const float p0 = fast_exp2(x0), p1 = fast_exp2(x1);
          acc[(j >> 1) & 3] = f2_add(acc[(j >> 1) & 3], f2_pack(p0, p1));
          pk[j / 2] = pack_bf16(p0, p1);
        }
        tmem_st16(tSr + 16 * c, pk);  // P (BF16 pairs) over the first 32 columns of the buffer
      }
      {
        const uint64_t a01 = f2_add(acc[0], acc[1]), a23 = f2_add(acc[2], acc[3]);
        float lo, hi;
        f2_unpack(f2_add(a01, a23), lo, hi);
        l_run += lo + hi;
      }
      if (__any_sync(0xffffffffu, need)) {
        // O may only be touched once every P V issued so far (up to tile i-1) has completed;
        // P_i V_i is not issued before this warp arrives on P_FULL below.
        if (!warp_wait(bar(PV_DONE0 + ((i - 1) & 1)), (uint32_t)((i - 1) >> 1) & 1u, abort_flag,
                       p.status)) {
          tmem_wait_st();
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t a2 = f2_pack(alpha, alpha);
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          uint32_t o[32];
          tmem_ld32(tOr + 32 * c, o);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; j += 2) {
            float x0, x1;
            f2_unpack(f2_mul(f2_pack(__uint_as_float(o[j]), __uint_as_float(o[j + 1])), a2), x0, x1);
            o[j] = __float_as_uint(x0);
            o[j + 1] = __float_as_uint(x1);
          }
          tmem_st32(tOr + 32 * c, o);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(P_FULL0 + sl));
    }
    // ---- epilogue: O / l -> BF16 ----
    if (ok && ntiles > 0 &&
        warp_wait(bar(PV_DONE0 + ((ntiles - 1) & 1)), (uint32_t)((ntiles - 1) >> 1) & 1u,
                  abort_flag, p.status)) {
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

// The softmax folds a positive scale into the exponent (max(s) * scale == max(s * scale) and
// masked -inf scores stay -inf), so other scales take the mma.sync kernel.
bool attn_sm100_supported(const AttnParams& p) {
  return p.nkb <= kMaxKeyBlocks && p.scale_log2 > 0.f;
}

cudaError_t launch_attn_sm100(const AttnParams& p, int D, cudaStream_t stream) {
  return D == 128 ? launch_sm100<128>(p, stream) : launch_sm100<64>(p, stream);
}

}  // namespace solattn
