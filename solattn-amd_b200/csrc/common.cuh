// Shared device helpers for the SOL attention kernels (sm_100a).
// Hand-written PTX wrappers: cp.async, ldmatrix, mma.sync (used by the pooling and
// small-tile paths), ex2, and the launch-parameter structures shared by the host layer.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace solattn {

constexpr int kBlock = 64;  // tokens per routing block (kernels.py:12)

// Device-side error codes written to the caller's status word (first error wins).
constexpr int kStatusWaitTimeout = 1;  // a bounded mbarrier wait ran out
constexpr int kStatusBadIndex = 2;     // a gather index outside its tensor
constexpr int kStatusTmem = 3;         // TMEM allocation returned an unusable address
constexpr int kStatusBadTma = 4;       // a TMA tile coordinate outside its tensor (load skipped)

struct TensorView {
  const __nv_bfloat16* ptr;
  int64_t sB, sT, sH;   // element strides; the head dimension is contiguous
  const int64_t* idx;   // optional gather index [B, T] (indexed NHD inputs), else nullptr
  int64_t rows;         // number of rows of the underlying tensor (bounds for idx)
};

struct AttnParams {
  TensorView q, k, v;
  const __nv_bfloat16* kc;  // [B, H, nkb, D]
  const __nv_bfloat16* vc;  // [B, H, nkb, D]
  const float* qc;          // [B, H, nqb, D]
  const float* cutoff;      // [B, H, nqb] (read by routing unless mean/var are given)
  // The full forward's fused threshold: the pooling kernel wrote the key moments mean / var
  // [B, H, D], and each routing CTA forms its q-blocks' cutoffs from them (threshold.cuh
  // arithmetic) and writes them to cutoff_out [B, H, nqb]; else nullptr.
  const float* mean;
  const float* var;
  float* cutoff_out;
  const uint8_t* protect;   // [B, nqb, nkb] or nullptr
  __nv_bfloat16* out;       // [B, Tq, H, D], or NHD [out_rows, H, D] when out_idx is set
  const int64_t* out_idx;   // optional output rows [B, Tq]: row t of batch b goes to
                            // out[out_idx[b * Tq + t]] (the indexed forms' scatter), else nullptr
  int64_t out_rows;         // rows of `out` when out_idx is set (bounds for out_idx)
  int32_t* counts;          // [B, nqb, H] or nullptr
  int32_t* status;          // device status word or nullptr
  uint32_t* masks;          // [B, H, nqb, ceil(nkb/32)] routing bitmask: written by route.cu
                            // (read by attn_sm100_kernel) or by attn_mma_kernel
  uint8_t* lists;           // per-item tile lists (see item_list_stride) written by route.cu, or
                            // nullptr (the fused kernel then builds them itself)
  // Item order (with lists only; else nullptr): route.cu sorts each head's q-block pairs after
  // the sink pairs by tile count, longest first, and the fused kernel hands them out in that
  // order.  arrive[B * H] counts the routing CTAs of a head that have written their lists (zero
  // when the routing pass starts, and the pass leaves it zero); the last one writes the head's
  // order[B * H, npairs] and stamp[B * H] = epoch.  The order is used only where the stamp
  // equals this call's epoch, so a head without a sorted order keeps the natural one.
  int32_t* arrive;
  uint32_t* stamp;
  int32_t* order;
  uint32_t epoch;
  int B, Tq, Tk, H, nqb, nkb;
  const int32_t* tk_b;  // optional per-batch key counts [B] (ragged indexed plans: batch b has
                        // tk_b[b] <= Tk keys, ceil(tk_b[b] / 64) key blocks), else nullptr
  float scale;       // softmax scale (natural-log units), used by routing
  float beta;        // Eq. 15 beta (the fused threshold's cutoffs)
  float scale_log2;  // scale * log2(e), used by the softmax
  int force, local, kv_sink_blocks, q_sink_blocks;
};

struct PoolParams {
  TensorView x[3];   // q, k, v
  int T[3];          // Tq, Tk, Tk
  int nb[3];         // blocks per tensor
  int64_t units[3];  // units per tensor (B*nb*H); 0 skips the tensor
  const int32_t* tk_b;  // optional per-batch key counts [B] for K and V (ragged), else nullptr
  void* y[3];        // qc (float), kc (bf16), vc (bf16)
  int B, H;
  int order[3];      // tensor of grid row y (set by the launcher: K, then Q, then V)
  // Fused key moments (the full forward in threshold mode, else nullptr): k_arrive[B * H]
  // counts the finished K units of each head (zero at the start of the launch); the CTA that
  // finishes a head's last K unit computes the head's mean / var [B, H, D] (threshold.cuh).
  int32_t* k_arrive;
  float* mean;
  float* var;
  int32_t* status;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void report(int32_t* status, int code) {
  if (status) atomicCAS(status, 0, code);
}

// Address of token row t of (b, h) in a BTHD view, or of the gathered NHD row.
__device__ __forceinline__ const __nv_bfloat16* row_ptr(const TensorView& x, int T, int b, int h,
                                                        int t, int32_t* status) {
  int64_t tok = t;
  if (x.idx) {
    tok = __ldg(x.idx + (int64_t)b * T + t);
    if (tok < 0 || tok >= x.rows) {
      report(status, kStatusBadIndex);
      tok = 0;
    }
  }
  return x.ptr + (int64_t)b * x.sB + tok * x.sT + (int64_t)h * x.sH;
}

// 16-byte async copy global -> shared; src_bytes = 0 zero-fills the destination.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src),
               "r"(src_bytes));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// D = A(16x16 bf16, row) * B(16x8 bf16, col) + D, FP32 accumulate.
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                               uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// 2^x with the hardware approximation (ex2.approx.ftz.f32); ex2(-inf) = +0.
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Row-major [rows][D] bf16 tile in shared memory with 16-byte chunks XOR-swizzled by row:
// chunk c of row r lives at chunk (c ^ (r & 7)).  Conflict-free for ldmatrix.
template <int D>
__device__ __forceinline__ uint32_t swz(uint32_t base, int row, int chunk) {
  return base + (uint32_t)(row * D * 2 + ((chunk ^ (row & 7)) << 4));
}

// Routing proxy dot product sum_d qbar[d] * kc[d] in a fixed order shared by every kernel and
// by its CPU restatement: eight partial sums p_j over d = 8i + j (i increasing), each term one
// fused multiply-add p_j = fma(qbar[d], kc[d], p_j) rounded once to nearest FP32, then
// ((p0 + p1) + (p2 + p3)) + ((p4 + p5) + (p6 + p7)).  kcrow must be 16-byte aligned.
__device__ __forceinline__ float routing_dot(const float* qbar, const __nv_bfloat16* kcrow, int D) {
  float p[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) p[j] = 0.f;
  for (int i = 0; i < D / 8; ++i) {
    const uint4 raw = __ldg(reinterpret_cast<const uint4*>(kcrow) + i);
    const __nv_bfloat162* k2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 kf = __bfloat1622float2(k2[j]);
      p[2 * j] = __fmaf_rn(qbar[8 * i + 2 * j], kf.x, p[2 * j]);
      p[2 * j + 1] = __fmaf_rn(qbar[8 * i + 2 * j + 1], kf.y, p[2 * j + 1]);
    }
  }
  return __fadd_rn(__fadd_rn(__fadd_rn(p[0], p[1]), __fadd_rn(p[2], p[3])),
                   __fadd_rn(__fadd_rn(p[4], p[5]), __fadd_rn(p[6], p[7])));
}

// Two routing dots against one centroid row (same order and rounding as routing_dot).
__device__ __forceinline__ void routing_dot2(const float* qa, const float* qb,
                                             const __nv_bfloat16* kcrow, int D, float& da,
                                             float& db) {
  float pa[8], pb[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) pa[j] = pb[j] = 0.f;
  uint4 rows[16];  // D <= 128: the whole centroid row in flight at once
#pragma unroll
  for (int i = 0; i < 16; ++i)
    if (i < D / 8) rows[i] = __ldg(reinterpret_cast<const uint4*>(kcrow) + i);
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    if (i >= D / 8) break;
    const uint4 raw = rows[i];
    const __nv_bfloat162* k2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 kf = __bfloat1622float2(k2[j]);
      pa[2 * j] = __fmaf_rn(qa[8 * i + 2 * j], kf.x, pa[2 * j]);
      pa[2 * j + 1] = __fmaf_rn(qa[8 * i + 2 * j + 1], kf.y, pa[2 * j + 1]);
      pb[2 * j] = __fmaf_rn(qb[8 * i + 2 * j], kf.x, pb[2 * j]);
      pb[2 * j + 1] = __fmaf_rn(qb[8 * i + 2 * j + 1], kf.y, pb[2 * j + 1]);
    }
  }
  da = __fadd_rn(__fadd_rn(__fadd_rn(pa[0], pa[1]), __fadd_rn(pa[2], pa[3])),
                 __fadd_rn(__fadd_rn(pa[4], pa[5]), __fadd_rn(pa[6], pa[7])));
  db = __fadd_rn(__fadd_rn(__fadd_rn(pb[0], pb[1]), __fadd_rn(pb[2], pb[3])),
                 __fadd_rn(__fadd_rn(pb[4], pb[5]), __fadd_rn(pb[6], pb[7])));
}

// Tile lists of the fused sm_100 kernel, one per item = q-block pair (b, h, pair): a 16-byte
// header {tiles (even), tiles with keys, 0, 0} and item_list_capacity(nkb) int16 entries:
// first every 64-centroid group that still has a block unselected by either q-block (entry
// -(t + 1)), then every block of the union of both q-blocks' exact sets in increasing order
// (entry kb >= 0), then, for an odd count, one padding entry.  Capacities are multiples of 8
// entries so that every list starts on a 16-byte boundary.
constexpr int kPadTile = -32768;  // the padding entry (centroid entries are -(t + 1) >= -64)
__host__ __device__ inline int item_list_capacity(int nkb) {
  return ((nkb + 63) / 64 + nkb + 1 + 7) & ~7;
}
__host__ __device__ inline int64_t item_list_stride(int nkb) {
  return 16 + 2 * (int64_t)item_list_capacity(nkb);
}

// The item-order section of a mask buffer, after the tile lists: arrive and stamp (B * H words
// each, padded to 16 bytes), then order (B * H * npairs words).
__host__ __device__ inline int64_t order_words_padded(int64_t bh) { return (bh + 3) & ~int64_t(3); }
__host__ __device__ inline int64_t order_section_bytes(int64_t bh, int64_t npairs) {
  return 4 * (2 * order_words_padded(bh) + bh * npairs);
}

__device__ __forceinline__ uint32_t valid_bits32(int w, int nkb) {
  const int lo = 32 * w;
  if (lo + 32 <= nkb) return 0xffffffffu;
  if (lo >= nkb) return 0u;
  return (1u << (nkb - lo)) - 1u;
}

// One warp: the tile list of a q-block pair from the two q-blocks' exact-block bitmasks m0 and
// m1 (nwords words each; m1 is ignored when has1 is false) into `tiles` (shared or global
// memory), padded to an even count.  Returns the count (warp-uniform); `real` receives the
// count without the padding entry.  nkb_b: key blocks of the batch; force == 1 (every block
// exact) lists no centroid group.
__device__ __forceinline__ int build_item_list(const uint32_t* m0, const uint32_t* m1, bool has1,
                                               int nwords, int nkb_b, int force, int16_t* tiles,
                                               int lane, int& real) {
  int n = 0;
  const int nct = force == 1 ? 0 : (nkb_b + 63) / 64;
  for (int t0 = 0; t0 < nct; t0 += 32) {
    const int t = t0 + lane;
    bool useful = false;
    if (t < nct) {
      for (int wi = 2 * t; wi < 2 * t + 2 && wi < nwords; ++wi) {
        const uint32_t v = valid_bits32(wi, nkb_b);
        if ((~m0[wi] & v) || (has1 && (~m1[wi] & v))) useful = true;
      }
    }
    const uint32_t bal = __ballot_sync(0xffffffffu, useful);
    if (useful) tiles[n + __popc(bal & ((1u << lane) - 1u))] = (int16_t)(-(t + 1));
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
      tiles[rank++] = (int16_t)(32 * wi + bit);
    }
    r += __shfl_sync(0xffffffffu, incl, 31);
  }
  n += r;
  real = n;
  if (n & 1) {  // even tile counts: every item starts at an even tile position
    if (lane == 0) tiles[n] = (int16_t)kPadTile;
    ++n;
  }
  __syncwarp();
  return n;
}

// Keys of batch b: its own count in a ragged launch (a count outside [1, Tk] is reported and
// clamped, so that every index derived from it stays in range), else Tk.
__device__ __forceinline__ int clamp_key_count(int n, int Tk, int32_t* status) {
  if (n < 1 || n > Tk) {
    report(status, kStatusBadIndex);
    n = n < 1 ? 1 : Tk;
  }
  return n;
}
__device__ __forceinline__ int key_count(const AttnParams& p, int b) {
  return p.tk_b ? clamp_key_count(__ldg(p.tk_b + b), p.Tk, p.status) : p.Tk;
}

// The force modes and the local / sink / protected rules (reference.py:41-51,
// kernels.py:136-143) applied to a threshold decision `sel`.
__device__ __forceinline__ bool route_rules(const AttnParams& p, bool sel, int b, int qb, int kb) {
  if (p.force == 1) sel = true;
  if (p.force == 2) sel = false;
  int diff = kb - qb;
  if (diff < 0) diff = -diff;
  sel = sel || (p.local >= 0 && diff <= p.local) || kb < p.kv_sink_blocks || qb < p.q_sink_blocks;
  if (p.protect) sel = sel || p.protect[((int64_t)b * p.nqb + qb) * p.nkb + kb] != 0;
  return sel;
}

// Routing rule shared by every attention kernel: is key block kb exact for (b, qb, h)?
// Threshold mode: (routing_dot * scale) > cut.  Then the force modes and the local / sink /
// protected rules of reference.py:41-51 (kernels.py:136-143).
__device__ __forceinline__ bool route_selected(const AttnParams& p, const float* qbar,
                                               const __nv_bfloat16* kcrow, float cut, int D,
                                               int b, int qb, int kb) {
  bool sel;
  if (p.force == 1) {
    sel = true;
  } else if (p.force == 2) {
    sel = false;
  } else {
    sel = __fmul_rn(routing_dot(qbar, kcrow, D), p.scale) > cut;
  }
  int diff = kb - qb;
  if (diff < 0) diff = -diff;
  sel = sel || (p.local >= 0 && diff <= p.local) || kb < p.kv_sink_blocks || qb < p.q_sink_blocks;
  if (p.protect) sel = sel || p.protect[((int64_t)b * p.nqb + qb) * p.nkb + kb] != 0;
  return sel;
}

}  // namespace solattn
