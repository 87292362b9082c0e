// Fused routed attention on the Blackwell data path (replaces `_sol`, kernels.py:101-182).
//
// Persistent kernel: one CTA per SM (it allocates all 512 TMEM columns) works through a list of
// work items in launch order: CTA c starts with item c and takes each further item from the
// launch's work counter while it issues the last tiles of the one before (round robin over the
// grid when there is no counter).  An item is one
// 128-row query tile = two 64-row q-blocks (qb0, qb0 + 1) of one (b, h).  Launch order: first
// the q-block pairs holding query-sink blocks of all heads (every key block exact: the longest
// items), then each head's remaining pairs head by head (the items in flight at one time share
// one head's K/V in L2), within a head most tiles first (the routing pass sorts them), so that
// the launch ends on its shortest items.  384 threads.
//
// Tiles hold 64 keys: one exact key block, or 64 pooled centroids.  The routing pass
// (route.cu) has already written every q-block's exact-block bitmask; an item's tile list
// (shared memory) holds first every 64-centroid group that still has a block unselected by
// either q-block (entry -(t + 1)), then every block of the union of both q-blocks' exact sets
// in increasing order (entry kb >= 0).  A row whose q-block did not select an exact block sees
// it as -inf; a centroid whose block is exact for the row's q-block too.
//
// The tiles of all of a CTA's items form one sequence: tile g (counted over the CTA's items)
// uses ring slot / S buffer g % kStages and softmax group g % 2, so the rings and the tensor
// core run on from one item into the next.  Two independent online softmaxes run side by side:
// group x (softmax warps 4x..4x+3) takes the tiles with g % 2 == x into its own accumulator O_x
// with its own running max and sum; the item's epilogue merges the two.
//
// TMEM (512 columns): O_0 at [0, 128), O_1 at [128, 256), and kStages S buffers of 64 columns
// at [256, 512); P (BF16 pairs) is written over the first 32 columns of its S buffer.
// Shared memory: two Q buffers (items alternate), K and V rings of kStages 64-row tiles, and two
// sets of routing bitmasks and tile lists (items alternate).
//
// Warp roles:
//   warps 0-7  softmax: warp w owns TMEM lanes 32(w%4)..+31 for the tiles of group w/4.  Per
//              tile: tcgen05.ld S, mask/bias, FP32 online softmax with lazy rescaling, P
//              written over the S buffer, arrive P_FULL.  A warp whose q-block does not use
//              the tile writes P = 0 without reading S.  Item epilogue: merge O_0 and O_1 ->
//              BF16, then O_FREE (the next item's P V may overwrite O).
//   warps 8-9  S issue for even / odd tiles (the whole warp runs the loop so that operands stay
//              warp-uniform; one elected lane issues): S_g = Q K_g^T once P_{g-kStages} V has
//              freed the buffer and K_g has landed; two issuers keep the 8 MMAs (N = 64) per tile
//              flowing.
//   warp 10    P V issue (likewise warp-uniform): O_{g%2} += P_g V_g once the group's four warps
//              have written P_g.
//   warp 11    producer: per item, the routing bitmasks, the tile list and the exact-block
//              counts (built one item ahead), Q; then the K ring (slot refilled when S has
//              completed) and the V ring (slot refilled when P V has completed), by TMA, or by
//              gathering rows with cp.async for indexed inputs.
#include <cudaTypedefs.h>

#include <cstring>

#include "sm100.cuh"

namespace solattn {

namespace {

using namespace sm100;

constexpr int kRows = 128;         // query rows per item
constexpr int kKeys = 64;          // keys per tile
constexpr int kStages = 4;         // S buffers = K slots = V slots
constexpr int kGroupWarps = 4;     // softmax warps per group (one per TMEM lane quarter)
constexpr int kSoftmaxWarps = 8;
constexpr int kSWarp0 = 8;         // S issue, even tiles (kSWarp0 + 1: odd tiles)
constexpr int kPVWarp = 10;        // P V issue
constexpr int kKWarp = 11;         // producer
constexpr int kThreads = 384;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemO = 0, kTmemS = 256;  // O_x at kTmemO + 128 x
constexpr int kQBox = kRows * 128;   // one 128-row x 64-column BF16 box of Q (16 KB)
constexpr int kKVBox = kKeys * 128;  // one 64-row x 64-column BF16 box of K or V (8 KB)
constexpr int kMaxKeyBlocks = 4096;  // tile list capacity (T <= 262144 keys)
constexpr int kClaimTiles = 8;       // late claim: the next item this many tiles before the end
constexpr int kEarlyClaimItems = 16; // items per CTA from which the next items are claimed early
constexpr int kOrderItemsPerCta = 2;  // items per CTA from which the routing pass sorts them
// Tile-list entry that pads an item to an even tile count, so that every item starts at an even
// position of the CTA's tile sequence and its tiles split between the two softmax groups by
// their item-local parity: the result of an item then does not depend on which CTA ran it
// after which other items (bitwise repeatable under the dynamic schedule).  No keys, no loads,
// no MMAs, P = 0.  Centroid entries are -(t + 1) >= -64.
constexpr int kDummyTile = kPadTile;
// Readers of an item's tile list that must be done before the producer overwrites it two items
// later: the softmax warps, the two S issuers and the P V issuer.
constexpr int kListReaders = kSoftmaxWarps + 3;

// Barriers; ring barriers are indexed by slot, item barriers by item parity.
enum Bar {
  Q_FULL, Q_EMPTY = Q_FULL + 2, LIST_FULL = Q_EMPTY + 2, LIST_EMPTY = LIST_FULL + 2,
  O_FREE = LIST_EMPTY + 2,
  K_FULL, K_EMPTY = K_FULL + kStages, V_FULL = K_EMPTY + kStages, S_FULL = V_FULL + kStages,
  P_FULL = S_FULL + kStages, PV_DONE = P_FULL + kStages,
  MERGE = PV_DONE + kStages,  // [4 lane quarters], two arrivals each: the epilogue exchange
  DRAIN_S0 = MERGE + 4, DRAIN_S1, DRAIN_PV, NBARS
};

template <int D>
struct Layout {
  static constexpr int kQTile = kRows * D * 2;   // 128 x D BF16
  static constexpr int kKVTile = kKeys * D * 2;  // 64 x D BF16
  static constexpr int kQ = 0;                   // two Q buffers
  static constexpr int kK = 2 * kQTile;
  static constexpr int kV = kK + kStages * kKVTile;
  static constexpr int kBars = kV + kStages * kKVTile;
  // uint32 [0] TMEM address [1] abort flag; of list buffer j: [2 + j] tiles (even), [4 + j]
  // item, [6 + j] tiles with keys (the rest is one padding tile), [8 + j] the item's key count
  // Rounded up to 16 bytes: the tile lists behind it are filled by cp.async.bulk, whose shared
  // destination must be 16-byte aligned whatever the number of barriers.
  static constexpr int kMisc = (kBars + NBARS * 8 + 15) & ~15;
  static constexpr int kMerge = kMisc + 48;  // float [2 items][8 warps][2][32 lanes]: m, l
  static constexpr int kMask = kMerge + 2 * 8 * 2 * 32 * 4;  // uint32 [2 items][2 q-blocks][nwords]
  static_assert(kMisc % 16 == 0 && kMerge % 16 == 0 && kMask % 16 == 0,
                "tile lists must start on 16-byte boundaries (bulk-copy destination)");
  __host__ __device__ static int tiles_offset(int nwords) { return kMask + 4 * nwords * 4; }
  __host__ __device__ static int max_tiles(int nkb) { return item_list_capacity(nkb); }
  static size_t bytes(int nkb) {  // int16 tile lists [2 items][max_tiles]
    const int nwords = (nkb + 31) / 32;
    return 1024 + (size_t)tiles_offset(nwords) + 2 * (size_t)max_tiles(nkb) * 2;
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

// Loads issued into ring slot s after `issued` loads in total (loads go to slots 0, 1, ...).
__device__ __forceinline__ int loads_into(int issued, int s) {
  return issued > s ? (issued - s + kStages - 1) / kStages : 0;
}

// TMA loads of one K or V tile (tile-list entry e) into `dst` on barrier `full`: 64 centroid rows
// of the pooled map (e < 0) or the 64 rows of key block e.  Rows past the end of a tensor are
// filled with zeros by the TMA unit and masked by the softmax.
template <int D>
__device__ __forceinline__ void load_kv_tile(uint32_t dst, const CUtensorMap* tile_map,
                                             const CUtensorMap* cent_map, uint32_t full, int e,
                                             int h, int b) {
  if (e == kDummyTile) {  // a padding tile loads nothing
    mbar_arrive(full);
    return;
  }
  mbar_expect_tx(full, (uint32_t)(kKeys * D * 2));
  const bool cent = e < 0;
  const int row = cent ? kKeys * (-e - 1) : kBlock * e;
#pragma unroll
  for (int j = 0; j < D / 64; ++j)
    tma_load_4d(dst + j * kKVBox, cent ? cent_map : tile_map, full, 64 * j, row, h, b);
}

// Row indices of a gathered tile, loaded ahead into registers: lane l holds the token index of
// rows l, l + 32, ... (ROWS / 32 of them), row r taken from idx[min(r, valid - 1)].  An index
// outside [0, x.rows) is reported (kStatusBadIndex) and replaced by 0, so every address
// computed from it stays in range.
template <int ROWS>
struct RowIdx {
  int64_t t[ROWS / 32];
};
template <int ROWS>
__device__ __forceinline__ RowIdx<ROWS> load_row_idx(const TensorView& x, const int64_t* idx,
                                                     int valid, int lane, int32_t* status) {
  RowIdx<ROWS> ri;
#pragma unroll
  for (int k = 0; k < ROWS / 32; ++k) {
    int64_t tok = __ldg(idx + min(32 * k + lane, valid - 1));
    if (tok < 0 || tok >= x.rows) {
      report(status, kStatusBadIndex);
      tok = 0;
    }
    ri.t[k] = tok;
  }
  return ri;
}

// Gathered rows (indexed inputs): the ROWS rows of head h named by `ri`, copied from the NHD
// tensor x with 16-byte cp.async into a 128-byte-swizzled K-major tile at `dst` (64-column
// boxes `box_bytes` apart; 16-byte chunk c of row r lands at chunk c ^ (r % 8), the layout a
// tiled TMA load produces).  D/8 consecutive lanes cover one row, so every warp instruction
// reads whole rows.  The calling lane then arms `full` for one arrival when its copies have
// landed.
template <int D, int ROWS>
__device__ __forceinline__ void gather_tile(uint32_t dst, uint32_t box_bytes, const TensorView& x,
                                            const RowIdx<ROWS>& ri, int h, int lane,
                                            uint32_t full) {
  constexpr int kChunks = D / 8;              // 16-byte chunks per row
  constexpr int kRowsPerPass = 32 / kChunks;  // rows one warp instruction covers (2 or 4)
  const int q = lane % kChunks, j = q >> 3, c = q & 7;
  const __nv_bfloat16* base = x.ptr + (int64_t)h * x.sH + 8 * q;
#pragma unroll
  for (int r0 = 0; r0 < ROWS; r0 += kRowsPerPass) {
    const int r = r0 + lane / kChunks;
    const int64_t tok = __shfl_sync(0xffffffffu, ri.t[r0 / 32], r & 31);
    cp_async16(dst + (uint32_t)j * box_bytes + (uint32_t)(r * 128 + ((c ^ (r & 7)) * 16)),
               base + tok * x.sT, 16);
  }
  cp_async_mbar_arrive_noinc(full);
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


// A work item is a q-block pair, identified by its pair id bh * npairs + pair.
struct ItemPos {
  int b, h, bh, qb0;
};
__device__ __forceinline__ ItemPos item_at(int pid, int nqb, int H) {
  const int npairs = (nqb + 1) / 2;
  ItemPos ip;
  ip.bh = pid / npairs;
  ip.b = ip.bh / H;
  ip.h = ip.bh % H;
  ip.qb0 = 2 * (pid % npairs);
  return ip;
}

// The pair id of the launch's claim number `claim`: first the pairs holding query-sink blocks
// of every head (the longest items: every key block exact, so none of them may start last),
// then each head's remaining pairs, head by head (the items in flight at one time share one
// head's K/V in L2), within a head in the routing pass's order, most tiles first, where it
// wrote one for this call (stamp == epoch), else in q-block order.
__device__ __forceinline__ int claim_pair(const AttnParams& p, int claim) {
  const int npairs = (p.nqb + 1) / 2;
  const int sink = min(npairs, (p.q_sink_blocks + 1) / 2);
  const int sink_items = sink * p.B * p.H;
  if (claim < sink_items) return (claim / sink) * npairs + claim % sink;
  const int r = claim - sink_items, rest = npairs - sink;
  if (rest <= 0) return 0;  // (claims stop below sink_items then)
  const int bh = r / rest, j = r % rest;
  int pair = sink + j;
  if (p.order) {
    const uint32_t st = __ldg(p.stamp + bh);
    const int o = __ldg(p.order + (int64_t)bh * npairs + j);
    if (st == p.epoch && o >= sink && o < npairs) pair = o;
  }
  return bh * npairs + pair;
}

// An item's routing mask words (both q-blocks, 2 nwords <= 256 words), loaded into registers one
// item ahead so that the load latency is off the producer's path: lane l holds word l + 32 j.
constexpr int kMaskRegs = 2 * (kMaxKeyBlocks / 32) / 32;
struct MaskWords {
  uint32_t w[kMaskRegs];
  int ntiles, real;  // from the item's precomputed list header (when the routing pass built it)
  int pid;           // the claimed item's pair id
};
__device__ __forceinline__ MaskWords load_mask_words(const AttnParams& p, int claim, int total,
                                                     int nwords, int lane) {
  MaskWords mw;
#pragma unroll
  for (int j = 0; j < kMaskRegs; ++j) mw.w[j] = 0u;
  mw.ntiles = mw.real = 0;
  mw.pid = claim < total ? claim_pair(p, claim) : 0;
  if (!p.masks || claim >= total) return mw;
  const ItemPos ip = item_at(mw.pid, p.nqb, p.H);
  if (p.lists) {
    const int2 hdr = __ldg(reinterpret_cast<const int2*>(
        p.lists + ((int64_t)ip.bh * ((p.nqb + 1) / 2) + (ip.qb0 >> 1)) * item_list_stride(p.nkb)));
    mw.ntiles = hdr.x;
    mw.real = hdr.y;
  }
#pragma unroll
  for (int j = 0; j < kMaskRegs; ++j) {
    const int i = 32 * j + lane;
    if (i < 2 * nwords) {
      const int qb = ip.qb0 + i / nwords;
      if (qb < p.nqb) mw.w[j] = __ldg(p.masks + ((int64_t)ip.bh * p.nqb + qb) * nwords + (i % nwords));
    }
  }
  return mw;
}

// One warp: both q-blocks' exact-block bitmasks of an item into m[0, 2 nwords) -- the routing
// pass's words (loaded ahead into `mw`), or (force modes without a mask buffer) the force /
// local / sink / protected rules alone.  Then, without a precomputed list, the item's tile list
// into `tiles` (build_item_list) and the per-q-block exact counts when requested; returns the
// number of tiles (warp-uniform) and the count without the padding entry in `real`.
__device__ __forceinline__ int build_tile_list(const AttnParams& p, const ItemPos& ip,
                                               const MaskWords& mw, uint32_t* m, int16_t* tiles,
                                               int nwords, int tk, int lane, int& real) {
  const bool has1 = ip.qb0 + 1 < p.nqb;
  const int nkb_b = (tk + kBlock - 1) / kBlock;  // this batch's key blocks
  if (p.masks) {
#pragma unroll
    for (int j = 0; j < kMaskRegs; ++j)
      if (32 * j + lane < 2 * nwords) m[32 * j + lane] = mw.w[j];
  } else {
    for (int i = 0; i < 2 * nwords; ++i) {
      const int qb = ip.qb0 + i / nwords, kb = 32 * (i % nwords) + lane;
      const bool sel = qb < p.nqb && kb < nkb_b && route_rules(p, false, ip.b, qb, kb);
      const uint32_t bal = __ballot_sync(0xffffffffu, sel);
      if (lane == 0) m[i] = bal;
    }
  }
  __syncwarp();
  if (p.lists) {  // the routing pass built the list (and wrote the counts)
    real = mw.real;
    return mw.ntiles;
  }
  const int n = build_item_list(m, m + nwords, has1, nwords, nkb_b, p.force, tiles, lane, real);
  if (lane < 2 && p.counts && ip.qb0 + lane < p.nqb) {
    int c = 0;
    for (int i = 0; i < nwords; ++i) c += __popc(m[lane * nwords + i]);
    p.counts[((int64_t)ip.b * p.nqb + ip.qb0 + lane) * p.H + ip.h] = c;
  }
  return n;
}

// Item epilogue of one softmax warp: wait for the group's last P V, exchange the running max
// and sum with the partner warp (same TMEM lanes, other group; the exchange buffer alternates
// with the items, so a warp that has run ahead never overwrites values not yet read), merge O_0
// and O_1 for the warp's 32 rows and half of the head dims into BF16, releasing both
// accumulators (the next item's P V may start) as soon as they are read, then the item's tile
// list.  Returns false after an abort.
template <int D>
__device__ __forceinline__ bool item_epilogue(uint32_t tmem, uint32_t bar0, int warp, int lane, int k,
                                           int last, float m_run, float l_run, int ntiles, int g,
                                           int pid, float* sMerge, volatile int* abort_flag,
                                           int32_t* status, __nv_bfloat16* out,
                                           const int64_t* out_idx, int64_t out_rows, int Tq, int H,
                                           int nqb) {
  auto bar = [bar0](int i) { return bar0 + 8u * (uint32_t)i; };
  const int quarter = warp & 3, grp = warp >> 2, lb = k & 1;
  const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
  if (last >= 0 &&
      !warp_wait(bar(PV_DONE + last % kStages), (uint32_t)(last / kStages) & 1u, abort_flag, status))
    return false;
  const float m_me = last >= 0 ? m_run : -INFINITY;
  float* mg = sMerge + lb * (8 * 2 * 32);
  mg[(warp * 2) * 32 + lane] = m_me;
  mg[(warp * 2 + 1) * 32 + lane] = l_run;
  __syncwarp();
  if (lane == 0) mbar_arrive(bar(MERGE + quarter));
  if (!warp_wait(bar(MERGE + quarter), (uint32_t)k & 1u, abort_flag, status)) return false;
  tc_fence_after();
  const float m_o = mg[((warp ^ 4) * 2) * 32 + lane];
  const float l_o = mg[((warp ^ 4) * 2 + 1) * 32 + lane];
  const float m0 = grp == 0 ? m_me : m_o, m1 = grp == 0 ? m_o : m_me;
  const float l0 = grp == 0 ? l_run : l_o, l1 = grp == 0 ? l_o : l_run;
  const float m = fmaxf(m0, m1);
  const float f0 = m0 == -INFINITY ? 0.f : fast_exp2(m0 - m);
  const float f1 = m1 == -INFINITY ? 0.f : fast_exp2(m1 - m);
  const float inv = 1.f / (l0 * f0 + l1 * f1);
  // A group without tiles in this item holds another item's accumulator: it is skipped.
  const bool has0 = ntiles >= 2 || (ntiles == 1 && (g & 1) == 0);
  const bool has1 = ntiles >= 2 || (ntiles == 1 && (g & 1) == 1);
  const ItemPos ip = item_at(pid, nqb, H);
  const int grow = ip.qb0 * kBlock + quarter * 32 + lane;
  // This warp writes head dims [grp * D / 2, (grp + 1) * D / 2) of its 32 rows: row grow of
  // batch b, or (scatter) output row out_idx[b * Tq + grow].
  bool store = grow < Tq;
  int64_t orow = (int64_t)ip.b * Tq + grow;
  if (out_idx && store) {
    orow = __ldg(out_idx + orow);
    if (orow < 0 || orow >= out_rows) {
      report(status, kStatusBadIndex);
      store = false;
    }
  }
  __nv_bfloat16* dst = out + (orow * H + ip.h) * D + grp * (D / 2);
#pragma unroll 1
  for (int c = 0; c < D / 32; ++c) {  // 16 columns at a time
    const uint32_t col = (uint32_t)(grp * (D / 2) + 16 * c);
    uint32_t o0[16], o1[16];
    if (has0) tmem_ld16(tmem + kTmemO + lane_base + col, o0);
    if (has1) tmem_ld16(tmem + kTmemO + 128 + lane_base + col, o1);
    tmem_wait_ld();
    if (c == D / 32 - 1) {
      // Both accumulators read: the next item's P V may start.
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(O_FREE));
    }
    if (store) {
      uint32_t w[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float a0 = 0.f, a1 = 0.f;
        if (has0) {
          a0 = __uint_as_float(o0[2 * j]) * f0;
          a1 = __uint_as_float(o0[2 * j + 1]) * f0;
        }
        if (has1) {
          a0 = fmaf(__uint_as_float(o1[2 * j]), f1, a0);
          a1 = fmaf(__uint_as_float(o1[2 * j + 1]), f1, a1);
        }
        w[j] = pack_bf16(a0 * inv, a1 * inv);
      }
      uint4* d4 = reinterpret_cast<uint4*>(dst + 16 * c);
      d4[0] = make_uint4(w[0], w[1], w[2], w[3]);
      d4[1] = make_uint4(w[4], w[5], w[6], w[7]);
    }
  }
  __syncwarp();
  if (lane == 0) mbar_arrive(bar(LIST_EMPTY + lb));
  return true;
}

}  // namespace


template <int D, bool kLateClaim>
__global__ void __launch_bounds__(kThreads, 1)
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
  volatile uint32_t* vmisc = misc;  // the list words are rewritten while the kernel runs
  volatile int* abort_flag = reinterpret_cast<volatile int*>(misc + 1);
  float* sMerge = reinterpret_cast<float*>(smem + L::kMerge);
  const int nwords = (p.nkb + 31) / 32;
  const int max_tiles = L::max_tiles(p.nkb);
  uint32_t* sMask = reinterpret_cast<uint32_t*>(smem + L::kMask);                // [2][2][nwords]
  int16_t* sTiles = reinterpret_cast<int16_t*>(smem + L::tiles_offset(nwords));  // [2][max_tiles]

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int total = ((p.nqb + 1) / 2) * p.B * p.H;  // work items

  if (tid == 0) {
    for (int i = 0; i < NBARS; ++i) {
      uint32_t count = 1;
      // Gathered loads arrive once per producer lane (cp.async completions).
      if (i >= Q_FULL && i < Q_FULL + 2 && p.q.idx) count = 32;
      if (((i >= K_FULL && i < K_FULL + kStages) || (i >= V_FULL && i < V_FULL + kStages)) && p.k.idx)
        count = 32;
      if (i >= Q_EMPTY && i < Q_EMPTY + 2) count = 2;  // both S issuers
      if (i >= LIST_EMPTY && i < LIST_EMPTY + 2) count = kListReaders;
      if (i == O_FREE) count = kSoftmaxWarps;
      if (i >= P_FULL && i < P_FULL + kStages) count = kGroupWarps;
      if (i >= MERGE && i < MERGE + 4) count = 2;
      mbar_init(bar(i), count);
    }
    misc[1] = 0;
    mbar_fence_init();
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(misc), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = misc[0];

  if (warp == kKWarp) {
    // ------------------------------------------------------------------ producer
    // Per item: the tile list into list buffer k % 2 once the item two back has released it,
    // Q into Q buffer k % 2 once both S issuers' MMAs of that item have completed, then the
    // item's K and V tiles into the rings.  Slot s of the K ring is free once S_{g - kStages}
    // has completed, slot s of the V ring once P_{g - kStages} V_{g - kStages} has; S_g itself
    // waits for the latter, so loading K_g before that wait delays nothing.  Without gathers
    // lane 0 alone issues the TMA loads; gathered rows are copied by the whole warp.
    if (lane == 0) {
      if (!p.q.idx) tma_prefetch(&tmQ);
      if (!p.k.idx) {
        tma_prefetch(&tmK);
        tma_prefetch(&tmV);
      }
      tma_prefetch(&tmKC);
      tma_prefetch(&tmVC);
    }
    // Items after the first come from the launch's work counter (the word after the routing
    // masks, zeroed by the routing pass) when there is one, else round robin over the grid.
    unsigned int* counter =
        p.masks ? p.masks + (int64_t)p.B * p.H * p.nqb * nwords : nullptr;
    // When to claim the next item.  With many items per CTA (early): the item after next is
    // claimed when an item starts, and the next item's mask words load while the current
    // item's tiles stream, so that no latency falls between two items.  With few items per CTA
    // (late): the next item is claimed while the producer issues the current item's last
    // kClaimTiles tiles, about kClaimTiles + kStages tiles before the consumers can start it.
    // A CTA then commits to an item only shortly before it is free for it, and the counter
    // balances the CTAs' work up to the last items; claimed early, the last rounds of items
    // are handed out by the state of the CTAs two items before, which leaves a tail of about
    // one item (measured at 3 heads of the bench workload, 5 items per CTA: 7 % of the
    // kernel's time).  The two modes are two instantiations (kLateClaim) and the early one
    // carries none of the late-claim code: the kernel's speed at many items per CTA changed by
    // several per cent with changes to producer code that it does not execute (code placement
    // and register allocation follow the whole kernel).
    constexpr bool early = !kLateClaim;
    int item = (int)blockIdx.x;
    int next = item + (int)gridDim.x;
    if constexpr (early) {
      if (counter && lane == 0) next = (int)gridDim.x + (int)atomicAdd(counter, 1u);
      next = __shfl_sync(0xffffffffu, next, 0);
    }
    MaskWords mw = load_mask_words(p, item, total, nwords, lane);
    int g = 0;  // tiles of this CTA's earlier items
    int k_issued = 0, v_issued = 0, q_issued = 0;
    bool ok = true;
    for (int k = 0; ok; ++k) {
      const int lb = k & 1;
      if (item >= total) {  // no more work: the consumers leave their loops
        if (k >= 2 && !warp_wait(bar(LIST_EMPTY + lb), (uint32_t)((k >> 1) - 1) & 1u,
                                 abort_flag, p.status))
          break;
        if (lane == 0) {
          misc[4 + lb] = 0xffffffffu;
          mbar_arrive(bar(LIST_FULL + lb));
        }
        break;
      }
      const int pid = mw.pid;  // the claimed item (mw holds its words until the next load)
      const ItemPos ip = item_at(pid, p.nqb, p.H);
      // Q of the item first: it does not depend on the tile list.
      if (k >= 2 && !warp_wait(bar(Q_EMPTY + lb), (uint32_t)((k >> 1) - 1) & 1u, abort_flag,
                               p.status)) {
        ok = false;
        break;
      }
      const uint32_t dq = sQ + (uint32_t)(lb * L::kQTile);
      if (p.q.idx) {
        const RowIdx<kRows> ri = load_row_idx<kRows>(
            p.q, p.q.idx + (int64_t)ip.b * p.Tq + (int64_t)ip.qb0 * kBlock,
            p.Tq - ip.qb0 * kBlock, lane, p.status);
        gather_tile<D, kRows>(dq, kQBox, p.q, ri, ip.h, lane, bar(Q_FULL + lb));
      } else if (lane == 0) {
        mbar_expect_tx(bar(Q_FULL + lb), L::kQTile);
        for (int j = 0; j < D / 64; ++j)
          tma_load_4d(dq + j * kQBox, &tmQ, bar(Q_FULL + lb), 64 * j, ip.qb0 * kBlock, ip.h, ip.b);
      }
      ++q_issued;
      // Early claim: the item after next, used two items on.
      int next2 = next + (int)gridDim.x;
      if constexpr (early) {
        if (counter && lane == 0) next2 = (int)gridDim.x + (int)atomicAdd(counter, 1u);
      }
      // The tile list, once the item two back has released the buffer.
      if (k >= 2 && !warp_wait(bar(LIST_EMPTY + lb), (uint32_t)((k >> 1) - 1) & 1u, abort_flag,
                               p.status)) {
        ok = false;
        break;
      }
      int16_t* tl = sTiles + lb * max_tiles;
      const int tk = key_count(p, ip.b);  // the item's keys (its window's count if ragged)
      int real;
      const int ntiles =
          build_tile_list(p, ip, mw, sMask + lb * 2 * nwords, tl, nwords, tk, lane, real);
      if (lane == 0) {
        misc[2 + lb] = (uint32_t)ntiles;
        misc[4 + lb] = (uint32_t)pid;
        misc[6 + lb] = (uint32_t)real;
        misc[8 + lb] = (uint32_t)tk;
        if (p.lists) {
          // The routing pass's list for this item: one bulk copy, which completes the barrier.
          const uint32_t bytes = (uint32_t)((2 * ntiles + 15) & ~15);
          const uint8_t* src = p.lists + 16 +
              ((int64_t)ip.bh * ((p.nqb + 1) / 2) + (ip.qb0 >> 1)) * item_list_stride(p.nkb);
          mbar_expect_tx(bar(LIST_FULL + lb), bytes);
          bulk_copy_g2s(smem_u32(tl), src, bytes, bar(LIST_FULL + lb));
        } else {
          mbar_arrive(bar(LIST_FULL + lb));
        }
      }
      if constexpr (early) mw = load_mask_words(p, next, total, nwords, lane);
      // The producer reads the list too (its K/V loads follow the entries).
      if (p.lists && !warp_wait(bar(LIST_FULL + lb), (uint32_t)(k >> 1) & 1u, abort_flag, p.status)) {
        ok = false;
        break;
      }
      if constexpr (early) {
        // K and V tiles of the item
        if (!p.k.idx) {
          if (lane == 0) {
            for (int i = 0; i < ntiles; ++i) {
              const int gi = g + i, s = gi % kStages;
              const uint32_t prev = (uint32_t)(gi / kStages - 1) & 1u;  // parity of the last use
              if (gi >= kStages && !mbar_wait(bar(K_EMPTY + s), prev, abort_flag, p.status)) {
                ok = false;
                break;
              }
              load_kv_tile<D>(sK + s * L::kKVTile, &tmK, &tmKC, bar(K_FULL + s), tl[i], ip.h, ip.b);
              ++k_issued;
              if (gi >= kStages && !mbar_wait(bar(PV_DONE + s), prev, abort_flag, p.status)) {
                ok = false;
                break;
              }
              load_kv_tile<D>(sV + s * L::kKVTile, &tmV, &tmVC, bar(V_FULL + s), tl[i], ip.h, ip.b);
              ++v_issued;
            }
          }
          ok = __shfl_sync(0xffffffffu, ok, 0);
        } else {
          // Gathered K/V rows: the whole warp copies; a tile's 64 row indices (shared by K and
          // V) are loaded one tile ahead.  Centroid tiles still come by TMA (lane 0), the other
          // lanes arriving on the barrier, which counts one arrival per lane in this mode.
          const int64_t* kvidx = p.k.idx + (int64_t)ip.b * p.Tk;
          auto row_idx = [&](int e) {
            RowIdx<kKeys> ri;
            if (e >= 0) {
              ri = load_row_idx<kKeys>(p.k, kvidx + (int64_t)e * kBlock, tk - e * kBlock, lane,
                                       p.status);
            } else {
              ri.t[0] = ri.t[1] = 0;
            }
            return ri;
          };
          RowIdx<kKeys> ri = row_idx(ntiles > 0 ? tl[0] : -1);
          for (int i = 0; i < ntiles; ++i) {
            const int gi = g + i, s = gi % kStages;
            const uint32_t prev = (uint32_t)(gi / kStages - 1) & 1u;
            const int e = tl[i];
            if (gi >= kStages && !warp_wait(bar(K_EMPTY + s), prev, abort_flag, p.status)) {
              ok = false;
              break;
            }
            if (e >= 0) gather_tile<D, kKeys>(sK + s * L::kKVTile, kKVBox, p.k, ri, ip.h, lane, bar(K_FULL + s));
            else if (lane == 0 || e == kDummyTile) load_kv_tile<D>(sK + s * L::kKVTile, &tmK, &tmKC, bar(K_FULL + s), e, ip.h, ip.b);
            else mbar_arrive(bar(K_FULL + s));
            ++k_issued;
            if (gi >= kStages && !warp_wait(bar(PV_DONE + s), prev, abort_flag, p.status)) {
              ok = false;
              break;
            }
            if (e >= 0) gather_tile<D, kKeys>(sV + s * L::kKVTile, kKVBox, p.v, ri, ip.h, lane, bar(V_FULL + s));
            else if (lane == 0 || e == kDummyTile) load_kv_tile<D>(sV + s * L::kKVTile, &tmV, &tmVC, bar(V_FULL + s), e, ip.h, ip.b);
            else mbar_arrive(bar(V_FULL + s));
            ++v_issued;
            if (i + 1 < ntiles) ri = row_idx(tl[i + 1]);
          }
        }
      } else {
        // Late claim of the next item: lane 0 issues the atomicAdd before tile claim_at and goes
        // on issuing tiles; two tiles later, when the result has returned, the warp reads it and
        // loads the item's mask words.
        const int claim_at = max(0, ntiles - kClaimTiles);
        const int read_at = min(ntiles, claim_at + 2);
        int claimed = item + (int)gridDim.x;
        auto claim_issue = [&]() {
          if (counter && lane == 0) claimed = (int)gridDim.x + (int)atomicAdd(counter, 1u);
        };
        auto claim_read = [&]() {
          next = __shfl_sync(0xffffffffu, claimed, 0);
          mw = load_mask_words(p, next, total, nwords, lane);
        };
        // K and V tiles of the item
        if (!p.k.idx) {
          const int bounds[4] = {0, claim_at, read_at, ntiles};
          for (int phase = 0; phase < 3 && ok; ++phase) {
            if (phase == 1) claim_issue();
            if (phase == 2) claim_read();
            if (lane == 0) {
              for (int i = bounds[phase]; i < bounds[phase + 1]; ++i) {
                const int gi = g + i, s = gi % kStages;
                const uint32_t prev = (uint32_t)(gi / kStages - 1) & 1u;  // parity of the last use
                if (gi >= kStages && !mbar_wait(bar(K_EMPTY + s), prev, abort_flag, p.status)) {
                  ok = false;
                  break;
                }
                load_kv_tile<D>(sK + s * L::kKVTile, &tmK, &tmKC, bar(K_FULL + s), tl[i], ip.h, ip.b);
                ++k_issued;
                if (gi >= kStages && !mbar_wait(bar(PV_DONE + s), prev, abort_flag, p.status)) {
                  ok = false;
                  break;
                }
                load_kv_tile<D>(sV + s * L::kKVTile, &tmV, &tmVC, bar(V_FULL + s), tl[i], ip.h, ip.b);
                ++v_issued;
              }
            }
            ok = __shfl_sync(0xffffffffu, ok, 0);
          }
        } else {
          // Gathered K/V rows: the whole warp copies; a tile's 64 row indices (shared by K and
          // V) are loaded one tile ahead.  Centroid tiles still come by TMA (lane 0), the other
          // lanes arriving on the barrier, which counts one arrival per lane in this mode.
          const int64_t* kvidx = p.k.idx + (int64_t)ip.b * p.Tk;
          auto row_idx = [&](int e) {
            RowIdx<kKeys> ri;
            if (e >= 0) {
              ri = load_row_idx<kKeys>(p.k, kvidx + (int64_t)e * kBlock, tk - e * kBlock, lane,
                                       p.status);
            } else {
              ri.t[0] = ri.t[1] = 0;
            }
            return ri;
          };
          RowIdx<kKeys> ri = row_idx(ntiles > 0 ? tl[0] : -1);
          for (int i = 0; i < ntiles; ++i) {
            if (i == claim_at) claim_issue();
            if (i == read_at) claim_read();
            const int gi = g + i, s = gi % kStages;
            const uint32_t prev = (uint32_t)(gi / kStages - 1) & 1u;
            const int e = tl[i];
            if (gi >= kStages && !warp_wait(bar(K_EMPTY + s), prev, abort_flag, p.status)) {
              ok = false;
              break;
            }
            if (e >= 0) gather_tile<D, kKeys>(sK + s * L::kKVTile, kKVBox, p.k, ri, ip.h, lane, bar(K_FULL + s));
            else if (lane == 0 || e == kDummyTile) load_kv_tile<D>(sK + s * L::kKVTile, &tmK, &tmKC, bar(K_FULL + s), e, ip.h, ip.b);
            else mbar_arrive(bar(K_FULL + s));
            ++k_issued;
            if (gi >= kStages && !warp_wait(bar(PV_DONE + s), prev, abort_flag, p.status)) {
              ok = false;
              break;
            }
            if (e >= 0) gather_tile<D, kKeys>(sV + s * L::kKVTile, kKVBox, p.v, ri, ip.h, lane, bar(V_FULL + s));
            else if (lane == 0 || e == kDummyTile) load_kv_tile<D>(sV + s * L::kKVTile, &tmV, &tmVC, bar(V_FULL + s), e, ip.h, ip.b);
            else mbar_arrive(bar(V_FULL + s));
            ++v_issued;
            if (i + 1 < ntiles) ri = row_idx(tl[i + 1]);
          }
          if (ok && read_at == ntiles) {  // fewer than three tiles after claim_at
            if (claim_at == ntiles) claim_issue();
            claim_read();
          }
        }
        if (!ok) break;
      }
      g += ntiles;
      item = next;
      if constexpr (early) next = __shfl_sync(0xffffffffu, next2, 0);
    }
    if (p.q.idx || p.k.idx) cp_async_wait_all();  // no copy may still write shared memory
    if (lane == 0 && *abort_flag) {
      for (int j = 0; j < 2; ++j) {
        const int n = q_issued > j ? (q_issued - j + 1) / 2 : 0;
        if (n) mbar_wait_quiet(bar(Q_FULL + j), (uint32_t)(n - 1) & 1u);
      }
      for (int s = 0; s < kStages; ++s) {
        int n = loads_into(k_issued, s);
        if (n) mbar_wait_quiet(bar(K_FULL + s), (uint32_t)(n - 1) & 1u);
        n = loads_into(v_issued, s);
        if (n) mbar_wait_quiet(bar(V_FULL + s), (uint32_t)(n - 1) & 1u);
      }
    }
    __syncwarp();
  } else if (warp == kPVWarp) {
    // ------------------------------------------------------------------ P V issue
    constexpr uint32_t idO = idesc_bf16(kRows, D, true);
    constexpr uint64_t kSlotStep = (uint64_t)(L::kKVTile >> 4);
    const uint64_t dV = smem_desc_sw128(sV, kKVBox, 1024);
    int g = 0;
    bool ok = true;
    for (int k = 0; ok; ++k) {
      const int lb = k & 1;
      if (!warp_wait(bar(LIST_FULL + lb), (uint32_t)(k >> 1) & 1u, abort_flag, p.status)) break;
      const int item = (int)vmisc[4 + lb];
      const int ntiles = (int)vmisc[2 + lb];
      const int real = (int)vmisc[6 + lb];  // tiles with keys; the rest is a padding tile
      if (item < 0) break;
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(LIST_EMPTY + lb));
      // The previous item's epilogue has read both O accumulators.
      if (k >= 1 && !warp_wait(bar(O_FREE), (uint32_t)(k - 1) & 1u, abort_flag, p.status)) break;
      for (int i = 0; i < ntiles; ++i) {
        const int gi = g + i, s = gi % kStages;
        const uint32_t ph = (uint32_t)(gi / kStages) & 1u;
        if (!warp_wait(bar(P_FULL + s), ph, abort_flag, p.status) ||
            !warp_wait(bar(V_FULL + s), ph, abort_flag, p.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (p.k.idx) fence_proxy_async_smem();  // gathered V rows were written by cp.async
        // Operands are computed by the whole warp (warp-uniform) and one elected lane issues: a
        // tcgen05.mma issued from a branch that only lane 0 runs took up to twice as long.
        const uint64_t vd = dV + (uint64_t)s * kSlotStep;
        const uint32_t tP = tmem + kTmemS + (uint32_t)(kKeys * s);
        const uint32_t tO = tmem + kTmemO + (uint32_t)(128 * (gi & 1));  // the tile's group
        // Local tiles 0 and 1 are each group's first of the item (items start at even tile
        // positions): they start the accumulator.
        const uint32_t acc0 = i > 1 ? 1u : 0u;
        const bool has_keys = i < real;
        if (elect_one()) {
          if (has_keys) {
#pragma unroll
            for (int kk = 0; kk < kKeys / 16; ++kk)
              mma_ts(tO, tP + (uint32_t)(8 * kk), vd + (uint64_t)((kk * 16 * 128) >> 4), idO,
                     kk > 0 ? 1u : acc0);
          }
          mma_commit(bar(PV_DONE + s));  // a padding tile: once the MMAs before it completed
        }
        __syncwarp();
      }
      g += ntiles;
    }
    if (lane == 0) {
      mma_commit(bar(DRAIN_PV));
      mbar_wait_quiet(bar(DRAIN_PV), 0);
    }
    __syncwarp();
  } else if (warp >= kSWarp0) {
    // ------------------------------------------------------------------ S issue (two warps)
    const int par = warp - kSWarp0;  // tiles g with g % 2 == par
    constexpr uint32_t idS = idesc_bf16(kRows, kKeys, false);
    constexpr uint64_t kSlotStep = (uint64_t)(L::kKVTile >> 4);
    const uint64_t dK = smem_desc_sw128(sK, 16, 1024);
    int g = 0;
    bool ok = true;
    for (int k = 0; ok; ++k) {
      const int lb = k & 1;
      const uint32_t iph = (uint32_t)(k >> 1) & 1u;
      if (!warp_wait(bar(LIST_FULL + lb), iph, abort_flag, p.status)) break;
      const int item = (int)vmisc[4 + lb];
      const int ntiles = (int)vmisc[2 + lb];
      const int real = (int)vmisc[6 + lb];  // tiles with keys; the rest is a padding tile
      if (item < 0) break;
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(LIST_EMPTY + lb));
      if (!warp_wait(bar(Q_FULL + lb), iph, abort_flag, p.status)) break;
      if (p.q.idx) fence_proxy_async_smem();  // gathered Q rows were written by cp.async
      const uint64_t dQ = smem_desc_sw128(sQ + (uint32_t)(lb * L::kQTile), 16, 1024);
      for (int i = (par ^ g) & 1; i < ntiles; i += 2) {
        const int gi = g + i, s = gi % kStages;
        const uint32_t ph = (uint32_t)(gi / kStages) & 1u;
        // P_{g - kStages} V_{g - kStages} (the last reader of the buffer) has completed, and
        // K_g has landed.  The order matters: the two issuers run independently, and only once
        // tile g - kStages is finished can K_FULL of this slot not still be a phase behind
        // (a parity wait on a barrier two phases behind would pass at once).
        if (gi >= kStages && !warp_wait(bar(PV_DONE + s), ph ^ 1u, abort_flag, p.status)) {
          ok = false;
          break;
        }
        if (!warp_wait(bar(K_FULL + s), ph, abort_flag, p.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (p.k.idx) fence_proxy_async_smem();  // gathered K rows were written by cp.async
        const uint64_t kd = dK + (uint64_t)s * kSlotStep;
        const uint32_t tS = tmem + kTmemS + (uint32_t)(kKeys * s);
        const bool has_keys = i < real;
        if (elect_one()) {
          if (has_keys) {
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
              const uint64_t off = (uint64_t)(((kk >> 2) * kQBox + (kk & 3) * 32) >> 4);
              const uint64_t offk = (uint64_t)(((kk >> 2) * kKVBox + (kk & 3) * 32) >> 4);
              mma_ss(tS, dQ + off, kd + offk, idS, kk > 0 ? 1u : 0u);
            }
          }
          // (a padding tile: both barriers once the MMAs before it completed)
          mma_commit(bar(S_FULL + s));
          mma_commit(bar(K_EMPTY + s));
        }
        __syncwarp();
      }
      // Q buffer lb is free once this issuer's MMAs of the item have completed.
      if (ok && lane == 0) mma_commit(bar(Q_EMPTY + lb));
      __syncwarp();
      g += ntiles;
    }
    if (lane == 0) {
      mma_commit(bar(DRAIN_S0 + par));
      mbar_wait_quiet(bar(DRAIN_S0 + par), 0);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ softmax warps
    const int quarter = warp & 3, grp = warp >> 2;
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;  // TMEM lanes 32 quarter..
    const uint32_t tOr = tmem + kTmemO + (uint32_t)(128 * grp) + lane_base;
    const int qsel = quarter >> 1;  // lanes 0-63: qb0, lanes 64-127: qb0 + 1
    const float sl2 = p.scale_log2;
    const uint64_t sl2x2 = f2_pack(sl2, sl2);
    const uint64_t six2 = f2_pack(6.f, 6.f);  // log2(64): bias of a full block's centroid
    int g = 0;
    bool ok = true;
    for (int k = 0; ok; ++k) {
      const int lb = k & 1;
      if (!warp_wait(bar(LIST_FULL + lb), (uint32_t)(k >> 1) & 1u, abort_flag, p.status)) break;
      const int item = (int)vmisc[4 + lb];
      if (item < 0) break;
      const int ntiles = (int)vmisc[2 + lb];
      const ItemPos ip = item_at(item, p.nqb, p.H);
      // The warp's q-block exists (only the last pair of a head can lack its second q-block).
      const bool warp_rows = qsel == 0 || ip.qb0 + 1 < p.nqb;
      // The batch's keys (its own count in a ragged launch) and its last, maybe partial, block.
      const int tk = (int)vmisc[8 + lb], nkb_b = (tk + kBlock - 1) / kBlock;
      const int last_len = tk - (nkb_b - 1) * kBlock;
      const float last_bias = log2f((float)last_len);
      const int last_col = (nkb_b - 1) & 63;  // column of the last centroid in its group
      const int last_group = (nkb_b - 1) >> 6;
      const uint32_t* mymask = sMask + (lb * 2 + qsel) * nwords;
      const int16_t* tl = sTiles + lb * max_tiles;
      float m_run = -INFINITY, l_run = 0.f;
      int last = -1;  // this group's previous tile (its P V is the last one into O_grp)
      for (int i = (grp ^ g) & 1; i < ntiles; i += 2) {
        const int gi = g + i, s = gi % kStages;
        // Tile metadata first: these shared-memory reads overlap the wait for S.  Every value
        // below is warp-uniform (one q-block per warp).
        const int entry = tl[i];
        const bool dummy = entry == kDummyTile;
        const bool centroid = entry < 0 && !dummy;
        uint32_t approx0 = 0u, approx1 = 0u;  // centroid columns this q-block uses
        int len = 0;                          // valid keys of an exact block it selected
        if (centroid) {
          const int t = -entry - 1;  // 2t < nwords since t <= (nkb - 1) / 64
          if (warp_rows) {
            approx0 = ~mymask[2 * t] & valid_word(2 * t, nkb_b);
            if (2 * t + 1 < nwords) approx1 = ~mymask[2 * t + 1] & valid_word(2 * t + 1, nkb_b);
          }
        } else if (!dummy && warp_rows && ((mymask[entry >> 5] >> (entry & 31)) & 1u)) {
          len = min(kBlock, tk - entry * kBlock);
        }
        const bool active = centroid ? (approx0 | approx1) != 0u : len > 0;
        if (!warp_wait(bar(S_FULL + s), (uint32_t)(gi / kStages) & 1u, abort_flag, p.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t tSr = tmem + kTmemS + (uint32_t)(kKeys * s) + lane_base;
        if (!active) {
          // The tile contributes nothing to these rows: P = 0, the running max and sum stay.
          uint32_t z[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) z[j] = 0u;
          tmem_st32(tSr, z);
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(bar(P_FULL + s));
          last = gi;
          continue;
        }
        uint32_t sv[2][32];
        tmem_ld32(tSr, sv[0]);
        tmem_ld32(tSr + 32, sv[1]);
        tmem_wait_ld();
        float m_tile, k_mul;
        if (centroid) {
          // Centroid logits in log2 units, s * scale_log2 + log2(len), and -inf where the block
          // is exact for this q-block (or past the last block).  Every full block has
          // log2(64) = 6; a partial last block (column lc of the last group) is patched after.
          const int t = -entry - 1;
          const int lc = (t == last_group && last_len != kBlock) ? last_col : kKeys;
          float raw_lc = 0.f;
          if (lc < kKeys) {
#pragma unroll
            for (int c = 0; c < 2; ++c)
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (32 * c + j == lc) raw_lc = __uint_as_float(sv[c][j]);
          }
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            const uint32_t approx = c ? approx1 : approx0;
#pragma unroll
            for (int j = 0; j < 32; j += 2) {
              float v0, v1;
              f2_unpack(f2_fma(f2_pack(__uint_as_float(sv[c][j]), __uint_as_float(sv[c][j + 1])),
                               sl2x2, six2),
                        v0, v1);
              sv[c][j] = __float_as_uint(((approx >> j) & 1u) ? v0 : -INFINITY);
              sv[c][j + 1] = __float_as_uint(((approx >> (j + 1)) & 1u) ? v1 : -INFINITY);
            }
          }
          if (lc < kKeys && (((lc < 32 ? approx0 : approx1) >> (lc & 31)) & 1u)) {
            const float v = fmaf(raw_lc, sl2, last_bias);
#pragma unroll
            for (int c = 0; c < 2; ++c)
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (32 * c + j == lc) sv[c][j] = __float_as_uint(v);
          }
          m_tile = row_max64(sv);
          k_mul = 1.f;
        } else {
          // Exact tiles keep raw scores: max(s) * scale_log2 equals max(s * scale_log2) bit for
          // bit (the scale is positive) and the scale is folded into the exponent's FMA.
          if (len < kBlock) {
#pragma unroll
            for (int c = 0; c < 2; ++c)
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (32 * c + j >= len) sv[c][j] = __float_as_uint(-INFINITY);
          }
          m_tile = row_max64(sv) * sl2;
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
            float x0, x1;
            f2_unpack(f2_fma(f2_pack(__uint_as_float(sv[c][j]), __uint_as_float(sv[c][j + 1])),
                             kmul2, negm2),
                      x0, x1);
            const float p0 = fast_exp2(x0), p1 = fast_exp2(x1);
            acc[(j >> 1) & 3] = f2_add(acc[(j >> 1) & 3], f2_pack(p0, p1));
            pk[j / 2] = pack_bf16(p0, p1);
          }
          tmem_st16(tSr + (uint32_t)(16 * c), pk);  // P over the first 32 columns of the buffer
        }
        {
          const uint64_t a01 = f2_add(acc[0], acc[1]), a23 = f2_add(acc[2], acc[3]);
          float lo, hi;
          f2_unpack(f2_add(a01, a23), lo, hi);
          l_run += lo + hi;
        }
        if (__any_sync(0xffffffffu, need)) {
          // O_grp may only be touched once the group's previous P V has completed (the P V
          // issue is in order); P_g V_g is not issued before this group arrives on P_FULL below.
          if (!warp_wait(bar(PV_DONE + last % kStages), (uint32_t)(last / kStages) & 1u,
                         abort_flag, p.status)) {
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
              float y0, y1;
              f2_unpack(f2_mul(f2_pack(__uint_as_float(o[j]), __uint_as_float(o[j + 1])), a2), y0, y1);
              o[j] = __float_as_uint(y0);
              o[j + 1] = __float_as_uint(y1);
            }
            tmem_st32(tOr + 32 * c, o);
          }
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(P_FULL + s));
        last = gi;
      }
      if (!ok) break;
      // ---- item epilogue ----
      // Tiles with keys decide which accumulators hold this item.
      if (!item_epilogue<D>(tmem, bar0, warp, lane, k, last, m_run, l_run, (int)vmisc[6 + lb], g,
                            (int)vmisc[4 + lb], sMerge, abort_flag, p.status, p.out, p.out_idx,
                            p.out_rows, p.Tq, p.H, p.nqb))
        break;
      g += ntiles;
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
cudaError_t launch_route(const AttnParams& p, int D, cudaStream_t stream);  // route.cu

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
  if (p.nkb > kMaxKeyBlocks || (p.masks == nullptr && p.force == 0) || (p.tk_b && !p.k.idx))
    return cudaErrorInvalidValue;
  // Gathered (indexed) inputs are copied by the producer warp and need no tensor map.
  CUtensorMap tmQ, tmK, tmV, tmKC, tmVC;
  memset(&tmQ, 0, sizeof(tmQ));
  memset(&tmK, 0, sizeof(tmK));
  memset(&tmV, 0, sizeof(tmV));
  if ((!p.q.idx && !make_bthd_map(&tmQ, p.q, p.B, p.Tq, p.H, D, kRows)) ||
      (!p.k.idx && (!make_bthd_map(&tmK, p.k, p.B, p.Tk, p.H, D, kBlock) ||
                    !make_bthd_map(&tmV, p.v, p.B, p.Tk, p.H, D, kBlock))) ||
      !make_pooled_map(&tmKC, p.kc, p.B, p.H, p.nkb, D) ||
      !make_pooled_map(&tmVC, p.vc, p.B, p.H, p.nkb, D))
    return cudaErrorInvalidValue;
  // Persistent grid: one CTA per SM, each working through items until none are left.
  const int64_t items = (int64_t)((p.nqb + 1) / 2) * p.B * p.H;
  if (items > 0x7fff0000) return cudaErrorInvalidValue;
  int dev = 0, sms = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err == cudaSuccess) err = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (err != cudaSuccess) return err;
  const int64_t ctas = items < sms ? items : sms;
  // With fewer than kOrderItemsPerCta items per CTA every CTA takes one or two items and the
  // order cannot shorten the tail; the routing pass then skips the per-head sort (its counter,
  // fence and the last CTA's sort are pure latency at such sizes).
  AttnParams q = p;
  if (items < (int64_t)kOrderItemsPerCta * ctas) {
    q.arrive = nullptr;
    q.stamp = nullptr;
    q.order = nullptr;
  }
  if (q.masks) {
    err = launch_route(q, D, stream);
    if (err != cudaSuccess) return err;
  }
  const size_t smem = Layout<D>::bytes(q.nkb);
  // Fewer than kEarlyClaimItems items per CTA: the instantiation that claims items late.
  auto* kernel = items < (int64_t)kEarlyClaimItems * ctas ? attn_sm100_kernel<D, true>
                                                          : attn_sm100_kernel<D, false>;
  err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (err != cudaSuccess) return err;
  kernel<<<(unsigned)ctas, kThreads, smem, stream>>>(q, tmQ, tmK, tmV, tmKC, tmVC);
  return cudaGetLastError();
}

}  // namespace

// The int16 tile list holds at most kMaxKeyBlocks key blocks.  Every entry point has already
// rejected scales <= 0 (the softmax folds the positive scale into its exponent FMA) and a
// threshold route without routing masks, so the key-block count is the only limit left.
bool attn_sm100_supported(const AttnParams& p) { return p.nkb <= kMaxKeyBlocks; }

cudaError_t launch_attn_sm100(const AttnParams& p, int D, cudaStream_t stream) {
  return D == 128 ? launch_sm100<128>(p, stream) : launch_sm100<64>(p, stream);
}

}  // namespace solattn
