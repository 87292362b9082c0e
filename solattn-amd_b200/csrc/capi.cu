// extern "C" entry points of libsolattn.so (declared in include/solattn.h).
// Argument checking here is the C-side contract; the Python layer performs the reference's
// ValueError validation (attention.py:19-44) before it gets this far.
#include <math.h>
#include <stdio.h>

#include <atomic>

#include "../../include/solattn.h"
#include "common.cuh"

namespace solattn {
cudaError_t launch_pool(const PoolParams& p, int D, cudaStream_t stream);
cudaError_t launch_threshold(const __nv_bfloat16* kc, const float* qc, int BH, int H, int nqb,
                             int nkb, int D, float scale, float beta, float* mean, float* var,
                             float* cutoff, const int32_t* tk_b, cudaStream_t stream);
cudaError_t launch_attention(const AttnParams& p, int D, cudaStream_t stream);
}  // namespace solattn

using namespace solattn;

namespace {

constexpr int64_t kMaxTokens = int64_t(1) << 24;  // 16M rows per sequence
constexpr int64_t kMaxBlocks = 16384;             // key blocks the routing bitmask holds

int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }
int64_t align256(int64_t x) { return (x + 255) & ~int64_t(255); }

bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

// Strides are elements; every row start must be 16-byte aligned for the vector loads.
bool strides_ok(int64_t sB, int64_t sT, int64_t sH) {
  return sB >= 0 && sT > 0 && sH > 0 && sB % 8 == 0 && sT % 8 == 0 && sH % 8 == 0;
}

}  // namespace

// Shape contract shared by every entry point (also used by noalloc.cu).
namespace solattn {
int check_shapes(int64_t B, int64_t Tq, int64_t Tk, int64_t H, int64_t D) {
  if (B <= 0 || Tq <= 0 || Tk <= 0 || H <= 0) return SOLATTN_ERR_ARG;
  if (D != 64 && D != 128) return SOLATTN_ERR_UNSUPPORTED;
  if (Tq > kMaxTokens || Tk > kMaxTokens || B * H > (int64_t(1) << 30)) return SOLATTN_ERR_ARG;
  if (cdiv(Tk, kBlock) > kMaxBlocks) return SOLATTN_ERR_UNSUPPORTED;
  if (cdiv(Tq, kBlock) > 65535 * 64 || B * H > 65535) return SOLATTN_ERR_UNSUPPORTED;
  return SOLATTN_OK;
}
}  // namespace solattn

namespace {

TensorView view(const void* ptr, int64_t sB, int64_t sT, int64_t sH, const int64_t* idx,
                int64_t rows) {
  TensorView t;
  t.ptr = static_cast<const __nv_bfloat16*>(ptr);
  t.sB = sB;
  t.sT = sT;
  t.sH = sH;
  t.idx = idx;
  t.rows = rows;
  return t;
}

int from_cuda(cudaError_t e) { return e == cudaSuccess ? SOLATTN_OK : SOLATTN_ERR_LAUNCH; }

struct Layout {
  int64_t kc, vc, qc, mean, var, cutoff, masks, status, total;
};

// Bytes of the routing-mask buffer: the bitmask words, the work counter (padded to 16 bytes),
// one tile list per q-block pair (common.cuh: item_list_stride), then the item-order section
// (common.cuh: order_section_bytes).
int64_t masks_bytes(int64_t B, int64_t Tq, int64_t Tk, int64_t H) {
  const int64_t nqb = cdiv(Tq, kBlock), nkb = cdiv(Tk, kBlock);
  const int64_t words = (B * H * nqb * cdiv(nkb, 32) + 1 + 3) & ~int64_t(3);
  return 4 * words + B * H * cdiv(nqb, 2) * item_list_stride((int)nkb) +
         order_section_bytes(B * H, cdiv(nqb, 2));
}

// The tile lists inside a mask buffer.
uint8_t* lists_of(uint32_t* masks, int64_t B, int64_t Tq, int64_t Tk, int64_t H) {
  if (!masks) return nullptr;
  const int64_t nqb = cdiv(Tq, kBlock), nkb = cdiv(Tk, kBlock);
  const int64_t words = (B * H * nqb * cdiv(nkb, 32) + 1 + 3) & ~int64_t(3);
  return reinterpret_cast<uint8_t*>(masks) + 4 * words;
}

// The item-order section inside a mask buffer (after the tile lists) into p.arrive, p.stamp and
// p.order, with a fresh nonzero epoch.  Epochs come from one process-wide counter, so a stamp
// left by an earlier call never matches.
std::atomic<uint32_t> g_epoch{0};
void set_item_order(AttnParams& p, uint32_t* masks, int64_t B, int64_t Tq, int64_t Tk,
                    int64_t H) {
  p.arrive = nullptr;
  p.stamp = nullptr;
  p.order = nullptr;
  p.epoch = 0;
  if (!masks) return;
  const int64_t nqb = cdiv(Tq, kBlock), nkb = cdiv(Tk, kBlock), bh = B * H;
  uint8_t* sec = lists_of(masks, B, Tq, Tk, H) + bh * cdiv(nqb, 2) * item_list_stride((int)nkb);
  p.arrive = reinterpret_cast<int32_t*>(sec);
  p.stamp = reinterpret_cast<uint32_t*>(sec) + order_words_padded(bh);
  p.order = reinterpret_cast<int32_t*>(sec) + 2 * order_words_padded(bh);
  uint32_t e;
  do {
    e = g_epoch.fetch_add(1u, std::memory_order_relaxed) + 1u;
  } while (e == 0u);
  p.epoch = e;
}

Layout layout(int64_t B, int64_t Tq, int64_t Tk, int64_t H, int64_t D) {
  Layout L;
  const int64_t nqb = cdiv(Tq, kBlock), nkb = cdiv(Tk, kBlock);
  int64_t off = 0;
  // The status word, then (at byte 16) two per-head counter arrays, the routing pass's and the
  // pooling kernel's (finished K units), which solattn_sol_forward zeroes together with the
  // status word before every call.
  L.status = off;
  off = align256(off + 16 + 8 * B * H);
  L.kc = off;
  off = align256(off + B * H * nkb * D * 2);
  L.vc = off;
  off = align256(off + B * H * nkb * D * 2);
  L.qc = off;
  off = align256(off + B * H * nqb * D * 4);
  L.mean = off;
  off = align256(off + B * H * D * 4);
  L.var = off;
  off = align256(off + B * H * D * 4);
  L.cutoff = off;
  off = align256(off + B * H * nqb * 4);
  L.masks = off;
  off = align256(off + masks_bytes(B, Tq, Tk, H));  // + the work counter and tile lists
  L.total = off;
  return L;
}

int pool_impl(const void* q, const void* k, const void* v, int64_t B, int64_t Tq, int64_t Tk,
              int64_t H, int64_t D, int64_t q_sB, int64_t q_sT, int64_t q_sH, int64_t k_sB,
              int64_t k_sT, int64_t k_sH, int64_t v_sB, int64_t v_sT, int64_t v_sH,
              const int64_t* q_idx, const int64_t* kv_idx, int64_t idx_rows, int pool_q, float* qc,
              void* kc, void* vc, const int32_t* key_counts, int32_t* status, int32_t* k_arrive,
              float* mean, float* var, void* stream);

// Rows of the underlying tensor addressed by a gather index (bounds for the device check).
int64_t gather_rows(const int64_t* idx, int64_t idx_rows, int64_t T) { return idx ? idx_rows : T; }

}  // namespace

extern "C" {

const char* solattn_version(void) { return "sol-attn-b200 0.1.0 sm_100a"; }

const char* solattn_strerror(int code) {
  switch (code) {
    case SOLATTN_OK: return "ok";
    case SOLATTN_ERR_ARG: return "invalid argument";
    case SOLATTN_ERR_UNSUPPORTED: return "unsupported configuration";
    case SOLATTN_ERR_LAUNCH: return "kernel launch failed";
    case SOLATTN_ERR_DEVICE: return "device-side error reported by a kernel";
    case SOLATTN_ERR_CUDA: return "CUDA runtime call failed";
    case SOLATTN_ERR_TOO_LARGE: return "problem exceeds the fixed no-allocation scratch array";
    default: return "unknown error";
  }
}

int64_t solattn_workspace_layout(int64_t B, int64_t Tq, int64_t Tk, int64_t H, int64_t D,
                                 int64_t* off_kc, int64_t* off_vc, int64_t* off_qc,
                                 int64_t* off_mean, int64_t* off_var, int64_t* off_cutoff,
                                 int64_t* off_status, int64_t* off_masks) {
  if (check_shapes(B, Tq, Tk, H, D) != SOLATTN_OK) return 0;
  const Layout L = layout(B, Tq, Tk, H, D);
  if (off_kc) *off_kc = L.kc;
  if (off_vc) *off_vc = L.vc;
  if (off_qc) *off_qc = L.qc;
  if (off_mean) *off_mean = L.mean;
  if (off_var) *off_var = L.var;
  if (off_cutoff) *off_cutoff = L.cutoff;
  if (off_status) *off_status = L.status;
  if (off_masks) *off_masks = L.masks;
  return L.total;
}

int64_t solattn_masks_bytes(int64_t B, int64_t Tq, int64_t Tk, int64_t H) {
  if (B <= 0 || Tq <= 0 || Tk <= 0 || H <= 0) return 0;
  return masks_bytes(B, Tq, Tk, H);
}

int solattn_pool_qkv(const void* q, const void* k, const void* v, int64_t B, int64_t Tq,
                     int64_t Tk, int64_t H, int64_t D, int64_t q_sB, int64_t q_sT, int64_t q_sH,
                     int64_t k_sB, int64_t k_sT, int64_t k_sH, int64_t v_sB, int64_t v_sT,
                     int64_t v_sH, const int64_t* q_idx, const int64_t* kv_idx, int64_t idx_rows,
                     int pool_q, float* qc, void* kc, void* vc, int32_t* status, void* stream) {
  return pool_impl(q, k, v, B, Tq, Tk, H, D, q_sB, q_sT, q_sH, k_sB, k_sT, k_sH, v_sB, v_sT, v_sH,
                   q_idx, kv_idx, idx_rows, pool_q, qc, kc, vc, nullptr, status, nullptr, nullptr, nullptr, stream);
}

int solattn_threshold(const void* kc, const float* qc, int64_t B, int64_t H, int64_t nqb,
                      int64_t nkb, int64_t D, float scale, float beta, float* mean, float* var,
                      float* cutoff, void* stream) {
  if (B <= 0 || H <= 0 || nqb <= 0 || nkb <= 0 || nkb > kMaxBlocks) return SOLATTN_ERR_ARG;
  if (D != 64 && D != 128) return SOLATTN_ERR_UNSUPPORTED;
  if (!kc || !qc || !mean || !var || !cutoff) return SOLATTN_ERR_ARG;
  if (!(scale > 0.f) || !isfinite(scale) || !isfinite(beta)) return SOLATTN_ERR_ARG;
  return from_cuda(launch_threshold(static_cast<const __nv_bfloat16*>(kc), qc, (int)(B * H),
                                    (int)H, (int)nqb, (int)nkb, (int)D, scale, beta, mean, var,
                                    cutoff, nullptr, static_cast<cudaStream_t>(stream)));
}

}  // extern "C"

namespace {

int pool_impl(const void* q, const void* k, const void* v, int64_t B, int64_t Tq, int64_t Tk,
              int64_t H, int64_t D, int64_t q_sB, int64_t q_sT, int64_t q_sH, int64_t k_sB,
              int64_t k_sT, int64_t k_sH, int64_t v_sB, int64_t v_sT, int64_t v_sH,
              const int64_t* q_idx, const int64_t* kv_idx, int64_t idx_rows, int pool_q, float* qc,
              void* kc, void* vc, const int32_t* key_counts, int32_t* status, int32_t* k_arrive,
              float* mean, float* var, void* stream) {
  int rc = check_shapes(B, Tq, Tk, H, D);
  if (rc) return rc;
  if (!k || !v || !kc || !vc || (pool_q && (!q || !qc))) return SOLATTN_ERR_ARG;
  if ((q_idx || kv_idx) && idx_rows <= 0) return SOLATTN_ERR_ARG;
  if (!aligned16(k) || !aligned16(v) || (pool_q && !aligned16(q))) return SOLATTN_ERR_ARG;
  if (!strides_ok(k_sB, k_sT, k_sH) || !strides_ok(v_sB, v_sT, v_sH) ||
      (pool_q && !strides_ok(q_sB, q_sT, q_sH)))
    return SOLATTN_ERR_ARG;
  PoolParams p;
  p.x[0] = view(q, q_sB, q_sT, q_sH, q_idx, gather_rows(q_idx, idx_rows, Tq));
  p.x[1] = view(k, k_sB, k_sT, k_sH, kv_idx, gather_rows(kv_idx, idx_rows, Tk));
  p.x[2] = view(v, v_sB, v_sT, v_sH, kv_idx, gather_rows(kv_idx, idx_rows, Tk));
  p.T[0] = (int)Tq;
  p.T[1] = p.T[2] = (int)Tk;
  p.nb[0] = (int)cdiv(Tq, kBlock);
  p.nb[1] = p.nb[2] = (int)cdiv(Tk, kBlock);
  p.units[0] = pool_q ? B * p.nb[0] * H : 0;
  p.units[1] = p.units[2] = B * p.nb[1] * H;
  p.y[0] = qc;
  p.y[1] = kc;
  p.y[2] = vc;
  p.B = (int)B;
  p.H = (int)H;
  p.tk_b = key_counts;
  p.k_arrive = k_arrive;
  p.mean = mean;
  p.var = var;
  p.status = status;
  return from_cuda(launch_pool(p, (int)D, static_cast<cudaStream_t>(stream)));
}

// solattn_attention with an optional output row index (out_idx [B, Tq], out_rows rows of an NHD
// output); see solattn_sol_forward_scatter.
int attention_impl(const void* q, const void* k, const void* v, int64_t B, int64_t Tq,
                   int64_t Tk, int64_t H, int64_t D, int64_t q_sB, int64_t q_sT, int64_t q_sH,
                   int64_t k_sB, int64_t k_sT, int64_t k_sH, int64_t v_sB, int64_t v_sT,
                   int64_t v_sH, const int64_t* q_idx, const int64_t* kv_idx, int64_t idx_rows,
                   const void* kc, const void* vc, const float* qc, const float* cutoff,
                   const uint8_t* protect, float scale, int force, int local,
                   int kv_sink_blocks, int q_sink_blocks, void* out, const int64_t* out_idx,
                   int64_t out_rows, const int32_t* key_counts, int32_t* counts, int32_t* status,
                   uint32_t* masks, int32_t* arrive, const float* mean, const float* var,
                   float* cutoff_out, float beta, void* stream) {
  int rc = check_shapes(B, Tq, Tk, H, D);
  if (rc) return rc;
  if (!q || !k || !v || !kc || !vc || !out) return SOLATTN_ERR_ARG;
  if (force == SOLATTN_FORCE_THRESHOLD && !masks) return SOLATTN_ERR_ARG;
  if (masks && !aligned16(masks)) return SOLATTN_ERR_ARG;
  if (out_idx && out_rows <= 0) return SOLATTN_ERR_ARG;
  if (key_counts && !kv_idx) return SOLATTN_ERR_ARG;  // ragged key counts: indexed inputs only
  if ((q_idx || kv_idx) && idx_rows <= 0) return SOLATTN_ERR_ARG;
  if (force < 0 || force > 2 || (force == 0 && (!qc || (!cutoff && !(mean && var)))))
    return SOLATTN_ERR_ARG;
  if (!(scale > 0.f) || !isfinite(scale) || kv_sink_blocks < 0 || q_sink_blocks < 0)
    return SOLATTN_ERR_ARG;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out) || !aligned16(kc) ||
      !aligned16(vc))
    return SOLATTN_ERR_ARG;
  if (!strides_ok(q_sB, q_sT, q_sH) || !strides_ok(k_sB, k_sT, k_sH) ||
      !strides_ok(v_sB, v_sT, v_sH))
    return SOLATTN_ERR_ARG;
  AttnParams p;
  p.q = view(q, q_sB, q_sT, q_sH, q_idx, gather_rows(q_idx, idx_rows, Tq));
  p.k = view(k, k_sB, k_sT, k_sH, kv_idx, gather_rows(kv_idx, idx_rows, Tk));
  p.v = view(v, v_sB, v_sT, v_sH, kv_idx, gather_rows(kv_idx, idx_rows, Tk));
  p.kc = static_cast<const __nv_bfloat16*>(kc);
  p.vc = static_cast<const __nv_bfloat16*>(vc);
  p.qc = qc;
  p.cutoff = cutoff;
  p.mean = force == 0 ? mean : nullptr;
  p.var = force == 0 ? var : nullptr;
  p.cutoff_out = cutoff_out;
  p.beta = beta;
  p.protect = protect;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.out_idx = out_idx;
  p.out_rows = out_idx ? out_rows : 0;
  p.counts = counts;
  p.status = status;
  p.masks = masks;
  p.lists = lists_of(masks, B, Tq, Tk, H);
  set_item_order(p, masks, B, Tq, Tk, H);
  if (arrive && p.arrive) p.arrive = arrive;  // counters the caller zeroed for this call
  p.B = (int)B;
  p.Tq = (int)Tq;
  p.Tk = (int)Tk;
  p.H = (int)H;
  p.nqb = (int)cdiv(Tq, kBlock);
  p.nkb = (int)cdiv(Tk, kBlock);
  p.tk_b = key_counts;
  p.scale = scale;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.force = force;
  p.local = local;
  p.kv_sink_blocks = kv_sink_blocks;
  p.q_sink_blocks = q_sink_blocks;
  return from_cuda(launch_attention(p, (int)D, static_cast<cudaStream_t>(stream)));
}

int sol_forward_impl(const void* q, const void* k, const void* v, int64_t B, int64_t Tq,
                     int64_t Tk, int64_t H, int64_t D, int64_t q_sB, int64_t q_sT, int64_t q_sH,
                     int64_t k_sB, int64_t k_sT, int64_t k_sH, int64_t v_sB, int64_t v_sT,
                     int64_t v_sH, const int64_t* q_idx, const int64_t* kv_idx, int64_t idx_rows,
                     const uint8_t* protect, float scale, float beta, int local,
                     int kv_sink_blocks, int q_sink_blocks, void* workspace,
                     int64_t workspace_bytes, void* out, const int64_t* out_idx, int64_t out_rows,
                     const int32_t* key_counts, int32_t* counts, void* stream) {
  int rc = check_shapes(B, Tq, Tk, H, D);
  if (rc) return rc;
  if (isnan(beta) || !workspace) return SOLATTN_ERR_ARG;
  // Every argument is checked before the first CUDA call.
  if (!q || !k || !v || !out || !aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out))
    return SOLATTN_ERR_ARG;
  if (!strides_ok(q_sB, q_sT, q_sH) || !strides_ok(k_sB, k_sT, k_sH) ||
      !strides_ok(v_sB, v_sT, v_sH))
    return SOLATTN_ERR_ARG;
  if ((q_idx || kv_idx) && idx_rows <= 0) return SOLATTN_ERR_ARG;
  if (key_counts && !kv_idx) return SOLATTN_ERR_ARG;
  if (!(scale > 0.f) || !isfinite(scale) || kv_sink_blocks < 0 || q_sink_blocks < 0)
    return SOLATTN_ERR_ARG;
  const Layout L = layout(B, Tq, Tk, H, D);
  if (workspace_bytes < L.total || (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
    return SOLATTN_ERR_ARG;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const int force = isinf(beta) ? (beta < 0 ? SOLATTN_FORCE_ALL : SOLATTN_FORCE_NONE)
                                : SOLATTN_FORCE_THRESHOLD;
  const int64_t nqb = cdiv(Tq, kBlock), nkb = cdiv(Tk, kBlock);
  float* qc = reinterpret_cast<float*>(ws + L.qc);
  void* kc = ws + L.kc;
  void* vc = ws + L.vc;
  float* cutoff = reinterpret_cast<float*>(ws + L.cutoff);
  int32_t* status = reinterpret_cast<int32_t*>(ws + L.status);
  int32_t* route_arrive = status + 4;             // byte 16
  int32_t* k_arrive = route_arrive + B * H;       // the pooling kernel's finished K units
  float* mean = reinterpret_cast<float*>(ws + L.mean);
  float* var = reinterpret_cast<float*>(ws + L.var);
  // The status word and both counter arrays in one memset.
  if (cudaMemsetAsync(status, 0, (size_t)(16 + 8 * B * H), static_cast<cudaStream_t>(stream)) !=
      cudaSuccess)
    return SOLATTN_ERR_CUDA;
  const bool thr = force == SOLATTN_FORCE_THRESHOLD;
  // Threshold mode on the tcgen05 path (up to 4096 key blocks, where the routing pass runs):
  // the pooling kernel computes each head's key moments as its K units finish and the routing
  // pass forms the cutoffs, so no threshold launch sits between pooling and routing.  The
  // mma.sync kernel (more key blocks) routes in its own prologue from cutoffs computed first.
  const bool fused = thr && nkb <= 4096;
  rc = pool_impl(q, k, v, B, Tq, Tk, H, D, q_sB, q_sT, q_sH, k_sB, k_sT, k_sH, v_sB, v_sT, v_sH,
                 q_idx, kv_idx, idx_rows, thr, qc, kc, vc, key_counts, status,
                 fused ? k_arrive : nullptr, mean, var, stream);
  if (rc) return rc;
  if (thr && !fused) {
    rc = from_cuda(launch_threshold(static_cast<const __nv_bfloat16*>(kc), qc, (int)(B * H),
                                    (int)H, (int)nqb, (int)nkb, (int)D, scale, beta, mean, var,
                                    cutoff, key_counts, static_cast<cudaStream_t>(stream)));
    if (rc) return rc;
  }
  return attention_impl(q, k, v, B, Tq, Tk, H, D, q_sB, q_sT, q_sH, k_sB, k_sT, k_sH, v_sB,
                        v_sT, v_sH, q_idx, kv_idx, idx_rows, kc, vc, thr ? qc : nullptr,
                        thr && !fused ? cutoff : nullptr, protect, scale, force, local,
                        kv_sink_blocks, q_sink_blocks, out, out_idx, out_rows, key_counts, counts,
                        status, reinterpret_cast<uint32_t*>(ws + L.masks), route_arrive,
                        fused ? mean : nullptr, fused ? var : nullptr, fused ? cutoff : nullptr,
                        beta, stream);
}

}  // namespace

extern "C" {

int solattn_attention(const void* q, const void* k, const void* v, int64_t B, int64_t Tq,
                      int64_t Tk, int64_t H, int64_t D, int64_t q_sB, int64_t q_sT, int64_t q_sH,
                      int64_t k_sB, int64_t k_sT, int64_t k_sH, int64_t v_sB, int64_t v_sT,
                      int64_t v_sH, const int64_t* q_idx, const int64_t* kv_idx, int64_t idx_rows,
                      const void* kc, const void* vc, const float* qc, const float* cutoff,
                      const uint8_t* protect, float scale, int force, int local,
                      int kv_sink_blocks, int q_sink_blocks, void* out, int32_t* counts,
                      int32_t* status, uint32_t* masks, void* stream) {
  return attention_impl(q, k, v, B, Tq, Tk, H, D, q_sB, q_sT, q_sH, k_sB, k_sT, k_sH, v_sB, v_sT,
                        v_sH, q_idx, kv_idx, idx_rows, kc, vc, qc, cutoff, protect, scale, force,
                        local, kv_sink_blocks, q_sink_blocks, out, nullptr, 0, nullptr, counts,
                        status, masks, nullptr, nullptr, nullptr, nullptr, 0.f, stream);
}

int solattn_sol_forward(const void* q, const void* k, const void* v, int64_t B, int64_t Tq,
                        int64_t Tk, int64_t H, int64_t D, int64_t q_sB, int64_t q_sT,
                        int64_t q_sH, int64_t k_sB, int64_t k_sT, int64_t k_sH, int64_t v_sB,
                        int64_t v_sT, int64_t v_sH, const int64_t* q_idx, const int64_t* kv_idx,
                        int64_t idx_rows, const uint8_t* protect, float scale, float beta, int local,
                        int kv_sink_blocks, int q_sink_blocks, void* workspace,
                        int64_t workspace_bytes, void* out, int32_t* counts, void* stream) {
  return sol_forward_impl(q, k, v, B, Tq, Tk, H, D, q_sB, q_sT, q_sH, k_sB, k_sT, k_sH, v_sB,
                          v_sT, v_sH, q_idx, kv_idx, idx_rows, protect, scale, beta, local,
                          kv_sink_blocks, q_sink_blocks, workspace, workspace_bytes, out, nullptr,
                          0, nullptr, counts, stream);
}

int solattn_sol_forward_scatter(const void* q, const void* k, const void* v, int64_t B,
                                int64_t Tq, int64_t Tk, int64_t H, int64_t D, int64_t q_sB,
                                int64_t q_sT, int64_t q_sH, int64_t k_sB, int64_t k_sT,
                                int64_t k_sH, int64_t v_sB, int64_t v_sT, int64_t v_sH,
                                const int64_t* q_idx, const int64_t* kv_idx, int64_t idx_rows,
                                const uint8_t* protect, float scale, float beta, int local,
                                int kv_sink_blocks, int q_sink_blocks, void* workspace,
                                int64_t workspace_bytes, void* out, int64_t out_rows,
                                int32_t* counts, void* stream) {
  if (!q_idx || out_rows <= 0) return SOLATTN_ERR_ARG;
  return sol_forward_impl(q, k, v, B, Tq, Tk, H, D, q_sB, q_sT, q_sH, k_sB, k_sT, k_sH, v_sB,
                          v_sT, v_sH, q_idx, kv_idx, idx_rows, protect, scale, beta, local,
                          kv_sink_blocks, q_sink_blocks, workspace, workspace_bytes, out, q_idx,
                          out_rows, nullptr, counts, stream);
}

int solattn_sol_forward_ex(const void* q, const void* k, const void* v, int64_t B, int64_t Tq,
                           int64_t Tk, int64_t H, int64_t D, int64_t q_sB, int64_t q_sT,
                           int64_t q_sH, int64_t k_sB, int64_t k_sT, int64_t k_sH, int64_t v_sB,
                           int64_t v_sT, int64_t v_sH, const int64_t* q_idx, const int64_t* kv_idx,
                           int64_t idx_rows, const uint8_t* protect, float scale, float beta,
                           int local, int kv_sink_blocks, int q_sink_blocks, void* workspace,
                           int64_t workspace_bytes, const int32_t* key_counts, void* out,
                           int64_t out_rows, int32_t* counts, void* stream) {
  if (out_rows < 0 || (out_rows > 0 && !q_idx)) return SOLATTN_ERR_ARG;
  return sol_forward_impl(q, k, v, B, Tq, Tk, H, D, q_sB, q_sT, q_sH, k_sB, k_sT, k_sH, v_sB,
                          v_sT, v_sH, q_idx, kv_idx, idx_rows, protect, scale, beta, local,
                          kv_sink_blocks, q_sink_blocks, workspace, workspace_bytes, out,
                          out_rows > 0 ? q_idx : nullptr, out_rows, key_counts, counts, stream);
}

int solattn_dense_rows(const void* q, const void* k, const void* v, const int64_t* rows,
                       int64_t n_rows, int64_t N, int64_t H, int64_t D, int64_t q_sT,
                       int64_t q_sH, int64_t k_sT, int64_t k_sH, int64_t v_sT, int64_t v_sH,
                       float scale, void* out, int32_t* status, void* stream) {
  if (!rows || n_rows <= 0 || N <= 0) return SOLATTN_ERR_ARG;
  // One batch: the n_rows gathered query rows against all N keys (all-exact route, so the
  // K/V pointers stand in for the pooled statistics), written to out[rows].
  return attention_impl(q, k, v, 1, n_rows, N, H, D, 0, q_sT, q_sH, 0, k_sT, k_sH, 0, v_sT, v_sH,
                        rows, nullptr, N, k, v, nullptr, nullptr, nullptr, scale,
                        SOLATTN_FORCE_ALL, -1, 0, 0, out, rows, N, nullptr, nullptr, status,
                        nullptr, nullptr, nullptr, nullptr, nullptr, 0.f, stream);
}

int solattn_dense(const void* q, const void* k, const void* v, int64_t B, int64_t Tq, int64_t Tk,
                  int64_t H, int64_t D, int64_t q_sB, int64_t q_sT, int64_t q_sH, int64_t k_sB,
                  int64_t k_sT, int64_t k_sH, int64_t v_sB, int64_t v_sT, int64_t v_sH,
                  float scale, void* out, int32_t* status, void* stream) {
  // All-exact route: no pooled statistics are read (kc/vc are only dereferenced for
  // centroid tiles, and force = 1 produces none), so the K/V pointers stand in for them.
  return solattn_attention(q, k, v, B, Tq, Tk, H, D, q_sB, q_sT, q_sH, k_sB, k_sT, k_sH, v_sB,
                           v_sT, v_sH, nullptr, nullptr, 0, k, v, nullptr, nullptr, nullptr, scale,
                           SOLATTN_FORCE_ALL, -1, 0, 0, out, nullptr, status, nullptr, stream);
}

int solattn_copy_2d(void* dst, int64_t dst_pitch, const void* src, int64_t src_pitch,
                    int64_t width_bytes, int64_t rows, int direction, void* stream) {
  if (!dst || !src || width_bytes <= 0 || rows <= 0 || dst_pitch < width_bytes ||
      src_pitch < width_bytes || (direction != 0 && direction != 1))
    return SOLATTN_ERR_ARG;
  const cudaError_t e = cudaMemcpy2DAsync(
      dst, (size_t)dst_pitch, src, (size_t)src_pitch, (size_t)width_bytes, (size_t)rows,
      direction == 0 ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToHost,
      static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? SOLATTN_OK : SOLATTN_ERR_CUDA;
}

int solattn_status_to_host(const int32_t* status, int32_t* host_dst, void* stream) {
  if (!status || !host_dst) return SOLATTN_ERR_ARG;
  return cudaMemcpyAsync(host_dst, status, sizeof(int32_t), cudaMemcpyDeviceToHost,
                         static_cast<cudaStream_t>(stream)) == cudaSuccess
             ? SOLATTN_OK
             : SOLATTN_ERR_CUDA;
}

int solattn_read_status(int32_t* status, int32_t* value, void* stream) {
  if (!status || !value) return SOLATTN_ERR_ARG;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int32_t host = 0;
  if (cudaMemcpyAsync(&host, status, sizeof(int32_t), cudaMemcpyDeviceToHost, s) != cudaSuccess)
    return SOLATTN_ERR_CUDA;
  if (cudaStreamSynchronize(s) != cudaSuccess) return SOLATTN_ERR_CUDA;
  if (cudaMemsetAsync(status, 0, sizeof(int32_t), s) != cudaSuccess) return SOLATTN_ERR_CUDA;
  *value = host;
  return host ? SOLATTN_ERR_DEVICE : SOLATTN_OK;
}

}  // extern "C"
