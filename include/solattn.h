/*
 * solattn.h - C ABI of the B200 (sm_100a) SOL routed block-sparse attention library
 * (libsolattn.so).
 *
 * Every entry point takes raw device pointers, sizes, element strides, scalars and a
 * CUDA stream passed as `void*` (a cudaStream_t; NULL is the legacy default stream). No
 * entry point allocates or synchronises (solattn_read_status and solattn_noalloc_read_status
 * excepted): buffers are owned by
 * the caller (in the Python layer, torch), and only solattn_sol_forward_noalloc keeps state
 * between calls (its fixed scratch array). Work is enqueued on `stream` asynchronously.
 * Return value: SOLATTN_OK (0) or a negative SOLATTN_ERR_* code; solattn_strerror() gives
 * the message. Errors that a kernel detects on the device (a bounded wait that ran out, an
 * index outside its tensor) are written to the caller's status word (see
 * solattn_workspace_layout) and copied out with solattn_status_to_host() (asynchronous) or
 * solattn_read_status() (blocking).
 *
 * Tensor conventions (mirroring zihaomu/SolAttn-AMD):
 *   - BTHD activations q [B, Tq, H, D], k and v [B, Tk, H, D], BF16, any positive element
 *     strides (sB, sT, sH) with a contiguous head dimension (attention.py:37-38).
 *   - Indexed (NHD) activations [N, H, D] are passed with B = windows, sB = 0 and a gather
 *     index per tensor: token t of window w is row q_idx[w*Tq + t] (resp. kv_idx[w*Tk + t])
 *     of the NHD tensor (indexed.py:99); idx_rows = N.  An index outside [0, N) is reported
 *     in the status word (kernels read row 0 instead).
 *   - Blocks are 64 tokens; nqb = ceil(Tq/64), nkb = ceil(Tk/64).
 *   - Output is a fresh contiguous [B, Tq, H, D] BF16 tensor (kernels.py:179-180);
 *     counts is int32 [B, nqb, H] (kernels.py:181-182, attention.py:10-16).
 */
#ifndef SOLATTN_H_
#define SOLATTN_H_

#include <stdint.h>

#if defined(__GNUC__)
#define SOLATTN_API __attribute__((visibility("default")))
#else
#define SOLATTN_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define SOLATTN_OK 0
#define SOLATTN_ERR_ARG (-1)         /* invalid argument (shape, stride, alignment, pointer) */
#define SOLATTN_ERR_UNSUPPORTED (-2) /* valid but not implemented here (e.g. D not 64/128) */
#define SOLATTN_ERR_LAUNCH (-3)      /* CUDA reported an error at launch */
#define SOLATTN_ERR_DEVICE (-4)      /* a kernel reported a device-side error in the status word */
#define SOLATTN_ERR_CUDA (-5)        /* a CUDA runtime call failed */
#define SOLATTN_ERR_TOO_LARGE (-6)   /* the problem needs more scratch than the fixed no-allocation array */

/* Routing force modes (kernels.py:208): 0 threshold, 1 all blocks exact (beta=-inf),
 * 2 only protected blocks exact (beta=+inf). */
#define SOLATTN_FORCE_THRESHOLD 0
#define SOLATTN_FORCE_ALL 1
#define SOLATTN_FORCE_NONE 2

/* Library version string, e.g. "sol-attn-b200 0.1.0 sm_100a". */
SOLATTN_API const char* solattn_version(void);

/* Message for a SOLATTN_* code. */
SOLATTN_API const char* solattn_strerror(int code);

/*
 * Scratch layout of one forward call.  Replaces the torch.empty allocations of the
 * reference launcher (kernels.py:185-190, 203-217): kc/vc (BF16 K/V block means), qc (FP32
 * Q block means), mean/var (FP32 key moments), cutoff (FP32 Eq. 15 thresholds), the status
 * section (one device status word at its start, then at byte 16 two int32 [B * H] counter
 * arrays that solattn_sol_forward zeroes together with the status word), and masks
 * (solattn_masks_bytes(): the routing decisions, uint32 bitmask [B, H, nqb, ceil(nkb/32)],
 * then the fused kernel's work counter, per-item tile lists and item order).
 * Offsets are in bytes from the workspace base, each 256-byte aligned.  The pooled tensors
 * use the layout [B, H, blocks, D]; cutoff is [B, H, nqb].
 * Returns the total size in bytes, or 0 on an invalid shape.
 */
SOLATTN_API int64_t solattn_workspace_layout(int64_t B, int64_t Tq, int64_t Tk, int64_t H, int64_t D,
                                 int64_t* off_kc, int64_t* off_vc, int64_t* off_qc,
                                 int64_t* off_mean, int64_t* off_var, int64_t* off_cutoff,
                                 int64_t* off_status, int64_t* off_masks);

/*
 * Block pooling of Q, K and V in one launch.  Replaces `_pooled`/`_pool`
 * (kernels.py:16-27, 185-190): per 64-token block and head, the FP32 mean over the valid
 * rows min(64, T - 64*blk) (the ragged tail uses its own count).  K and V means are stored
 * as BF16 (round to nearest even), Q means as FP32.  With pool_q = 0 the Q pass is skipped
 * (beta = +-inf, kernels.py:209).  q_idx / kv_idx are NULL for BTHD or the indexed gather
 * indices described above.
 * Summation order (fixed, deterministic): 8 row groups; group g sums rows g, g+8, ..., g+56
 * in order; the 8 group sums are then added in order g = 0..7; mean = sum / count (IEEE).
 */
SOLATTN_API int solattn_pool_qkv(const void* q, const void* k, const void* v,
                     int64_t B, int64_t Tq, int64_t Tk, int64_t H, int64_t D,
                     int64_t q_sB, int64_t q_sT, int64_t q_sH,
                     int64_t k_sB, int64_t k_sT, int64_t k_sH,
                     int64_t v_sB, int64_t v_sT, int64_t v_sH,
                     const int64_t* q_idx, const int64_t* kv_idx, int64_t idx_rows, int pool_q,
                     float* qc, void* kc, void* vc, int32_t* status, void* stream);

/*
 * Key moments and Eq. 15 thresholds (the stage-by-stage form; solattn_sol_forward computes
 * the same bits inside its pooling and routing launches).  Replaces `_moments` + `_threshold`
 * (kernels.py:30-64, launches 211-215): per (b, h, d) mean = sum(kc)/nkb and
 * var = max(sum(kc^2)/nkb - mean^2, 0) over all key blocks, unweighted, each sum taken as
 * eight slice sums s_j over blocks j, j+8, j+16, ... (in order) combined as
 * ((s0+s1)+(s2+s3))+((s4+s5)+(s6+s7)); per (b, h, q-block)
 * cutoff = (sum_d qc*mean + beta * sqrt(sum_d (qc*qc)*var)) * scale, each sum over d taken
 * as eight partial sums over d = 8i + e combined in the same tree.  The cutoff is in
 * natural-log units: the attention kernel selects key block j iff dot * scale > cutoff,
 * where dot = sum_d qc[d]*kc_j[d] taken as eight partial sums p_j over d = 8i + j, each term
 * one fused multiply-add rounded once, combined as ((p0+p1)+(p2+p3))+((p4+p5)+(p6+p7)); every
 * other operation is rounded to nearest FP32 without contraction.  beta must be finite.
 */
SOLATTN_API int solattn_threshold(const void* kc, const float* qc, int64_t B, int64_t H, int64_t nqb,
                      int64_t nkb, int64_t D, float scale, float beta, float* mean, float* var,
                      float* cutoff, void* stream);

/* Bytes of the `masks` buffer of solattn_attention (0 on an invalid shape). */
SOLATTN_API int64_t solattn_masks_bytes(int64_t B, int64_t Tq, int64_t Tk, int64_t H);

/*
 * Fused routed attention.  Replaces `_sol` (kernels.py:101-182, launch 216-224): per
 * (b, h, 64-row q-block) it routes every key block (threshold / force mode, OR the local
 * rule |kb-qb| <= local (local < 0 disables it), kb < kv_sink_blocks, qb < q_sink_blocks
 * and protected[b, qb, kb] when `protect` is not NULL), computes the selected blocks exactly
 * (BF16 QK and PV, FP32 online softmax) and folds every unselected block in through its
 * centroid (logit q.kc*scale + log(len), value vc).  cutoff and qc may be NULL when
 * force != 0.  counts may be NULL.  status may be NULL.
 * masks receives the routing decisions as a bitmask [B, H, nqb, ceil(nkb/32)] of uint32
 * words (bit kb%32 of word kb/32 set = block kb exact); the call writes it in a routing pass
 * and the attention kernel reads it back.  The buffer (16-byte aligned) holds
 * solattn_masks_bytes(B, Tq, Tk, H) bytes: the bitmask, then the attention kernel's work
 * counter (zeroed by the routing pass, then incremented as the persistent CTAs take work
 * items), one tile list per q-block pair (built by the routing pass), and the item order:
 * per head a counter of routing CTAs, a stamp and the head's q-block pairs sorted by tile
 * count (the attention kernel hands items out longest first within each head).  The
 * counters must be zero before a buffer's first use (a zero-filled buffer); every call leaves
 * them zero.  It is required when force == SOLATTN_FORCE_THRESHOLD and may be NULL in the
 * force modes (the rules are then evaluated inside the kernel and the work is split round
 * robin).
 */
SOLATTN_API int solattn_attention(const void* q, const void* k, const void* v,
                      int64_t B, int64_t Tq, int64_t Tk, int64_t H, int64_t D,
                      int64_t q_sB, int64_t q_sT, int64_t q_sH,
                      int64_t k_sB, int64_t k_sT, int64_t k_sH,
                      int64_t v_sB, int64_t v_sT, int64_t v_sH,
                      const int64_t* q_idx, const int64_t* kv_idx, int64_t idx_rows,
                      const void* kc, const void* vc, const float* qc, const float* cutoff,
                      const uint8_t* protect, float scale, int force, int local,
                      int kv_sink_blocks, int q_sink_blocks, void* out, int32_t* counts,
                      int32_t* status, uint32_t* masks, void* stream);

/*
 * All-in SOL forward, the whole of `launch_sol` (kernels.py:203-225), using the caller's
 * workspace of solattn_workspace_layout() bytes: pooling (which, for force == 0, also
 * computes each head's key moments as its last K unit finishes), the routing pass (which
 * forms the cutoffs of its q-blocks from them), then the fused attention; the moments,
 * cutoffs and routing are bit-identical to solattn_threshold + solattn_attention.  With more
 * than 4096 key blocks the threshold kernel runs between pooling and attention instead.
 * beta may be +-inf (selects the force mode) but not NaN.
 */
SOLATTN_API int solattn_sol_forward(const void* q, const void* k, const void* v,
                        int64_t B, int64_t Tq, int64_t Tk, int64_t H, int64_t D,
                        int64_t q_sB, int64_t q_sT, int64_t q_sH,
                        int64_t k_sB, int64_t k_sT, int64_t k_sH,
                        int64_t v_sB, int64_t v_sT, int64_t v_sH,
                        const int64_t* q_idx, const int64_t* kv_idx, int64_t idx_rows,
                        const uint8_t* protect,
                        float scale, float beta, int local, int kv_sink_blocks,
                        int q_sink_blocks, void* workspace, int64_t workspace_bytes,
                        void* out, int32_t* counts, void* stream);

/*
 * solattn_sol_forward for indexed inputs that writes each query row's output straight to its
 * original row: `out` is an NHD [out_rows, H, D] BF16 tensor (rows of H*D elements) and query
 * row t of window b goes to out[q_idx[b*Tq + t]]; rows named by no window are left untouched.
 * Replaces the caller-side scatter `out[plan.rows] = result` of the reference's VDN adapter
 * (integrations/vdn.py:54-71), and with it the [B, Tq, H, D] intermediate.  Requires q_idx;
 * windows that name the same row race on it.  Row indices outside [0, out_rows) are reported
 * through the status word and skipped.
 */
SOLATTN_API int solattn_sol_forward_scatter(const void* q, const void* k, const void* v,
                        int64_t B, int64_t Tq, int64_t Tk, int64_t H, int64_t D,
                        int64_t q_sB, int64_t q_sT, int64_t q_sH,
                        int64_t k_sB, int64_t k_sT, int64_t k_sH,
                        int64_t v_sB, int64_t v_sT, int64_t v_sH,
                        const int64_t* q_idx, const int64_t* kv_idx, int64_t idx_rows,
                        const uint8_t* protect,
                        float scale, float beta, int local, int kv_sink_blocks,
                        int q_sink_blocks, void* workspace, int64_t workspace_bytes,
                        void* out, int64_t out_rows, int32_t* counts, void* stream);

/*
 * solattn_sol_forward with both indexed extensions.  key_counts (device int32 [B], or NULL)
 * gives window b its own number of keys, key_counts[b] in [1, Tk]: kv_idx rows are padded to
 * Tk and only the first key_counts[b] of row b are read - one launch for windows whose key
 * sets differ in size (a ragged IndexedPlan), with results identical to separate calls per
 * window.  A count outside [1, Tk] is clamped and reported through the status word.
 * key_counts requires kv_idx.  out_rows > 0 scatters into an NHD output exactly as
 * solattn_sol_forward_scatter (requires q_idx); out_rows == 0 writes [B, Tq, H, D].
 */
SOLATTN_API int solattn_sol_forward_ex(const void* q, const void* k, const void* v,
                        int64_t B, int64_t Tq, int64_t Tk, int64_t H, int64_t D,
                        int64_t q_sB, int64_t q_sT, int64_t q_sH,
                        int64_t k_sB, int64_t k_sT, int64_t k_sH,
                        int64_t v_sB, int64_t v_sT, int64_t v_sH,
                        const int64_t* q_idx, const int64_t* kv_idx, int64_t idx_rows,
                        const uint8_t* protect,
                        float scale, float beta, int local, int kv_sink_blocks,
                        int q_sink_blocks, void* workspace, int64_t workspace_bytes,
                        const int32_t* key_counts, void* out, int64_t out_rows,
                        int32_t* counts, void* stream);

/*
 * Dense attention of a subset of query rows against all keys, written in place: for each
 * i < n_rows, out[rows[i]] = softmax(q[rows[i]] . k^T * scale) . v over all N keys, with q, k,
 * v and out NHD [N, H, D] BF16 (element strides q_sT/q_sH etc.; the head dimension is
 * contiguous).  The VDN adapter's dense global-query step (`out[rows] = dense(q[rows], k, v)`,
 * integrations/vdn.py:58-63) without the gathered copy of Q or the scatter.  Needs no workspace.
 * A row index outside [0, N) is skipped and reported through `status` (a device int32 word the
 * caller clears, or NULL).
 */
SOLATTN_API int solattn_dense_rows(const void* q, const void* k, const void* v,
                  const int64_t* rows, int64_t n_rows, int64_t N, int64_t H, int64_t D,
                  int64_t q_sT, int64_t q_sH, int64_t k_sT, int64_t k_sH,
                  int64_t v_sT, int64_t v_sH, float scale, void* out, int32_t* status,
                  void* stream);

/*
 * Dense noncausal attention over all keys (BF16 QK/PV, FP32 softmax).  Replaces
 * `launch_dense`/`_dense` (kernels.py:67-98, 193-200); implemented as the all-exact route
 * of the fused kernel, so it needs no workspace.  `status`: a device int32 word that receives
 * device-side errors (a bounded wait that ran out), cleared by the caller, or NULL.
 */
SOLATTN_API int solattn_dense(const void* q, const void* k, const void* v,
                  int64_t B, int64_t Tq, int64_t Tk, int64_t H, int64_t D,
                  int64_t q_sB, int64_t q_sT, int64_t q_sH,
                  int64_t k_sB, int64_t k_sT, int64_t k_sH,
                  int64_t v_sB, int64_t v_sT, int64_t v_sH,
                  float scale, void* out, int32_t* status, void* stream);

/*
 * All-in SOL forward that allocates nothing (no counterpart in the reference).
 * For callers that cannot allocate device memory at call time - e.g. a plugin inside a host
 * program that owns all device memory through its own pool and forbids direct cudaMalloc, or a
 * latency-critical loop that cannot afford cudaMalloc's implicit synchronisation.  Same
 * arguments and results as solattn_sol_forward minus the workspace: the scratch is a fixed
 * file-scope device array of solattn_noalloc_scratch_bytes() bytes (32 MiB) that every GPU
 * loading this library holds until the process exits.  Problems whose
 * solattn_workspace_layout() size exceeds it return SOLATTN_ERR_TOO_LARGE before any GPU work.
 * All calls on a device share that array and it keeps the last call's contents (the status
 * word is cleared by each call; everything else a call reads, it writes first), so calls that
 * overlap on the GPU - different streams without ordering, or concurrent host threads - race.
 * The first call on each device looks up the array's device address (cudaGetSymbolAddress with
 * that device current) and caches it; make that first call before any stream capture begins.
 * Calls no cudaMalloc, cudaFree or other allocating routine.
 */
SOLATTN_API int solattn_sol_forward_noalloc(const void* q, const void* k, const void* v,
                        int64_t B, int64_t Tq, int64_t Tk, int64_t H, int64_t D,
                        int64_t q_sB, int64_t q_sT, int64_t q_sH,
                        int64_t k_sB, int64_t k_sT, int64_t k_sH,
                        int64_t v_sB, int64_t v_sT, int64_t v_sH,
                        const int64_t* q_idx, const int64_t* kv_idx, int64_t idx_rows,
                        const uint8_t* protect,
                        float scale, float beta, int local, int kv_sink_blocks,
                        int q_sink_blocks, void* out, int32_t* counts, void* stream);

/* Size in bytes of the fixed scratch array used by solattn_sol_forward_noalloc (no counterpart
 * in the reference). */
SOLATTN_API int64_t solattn_noalloc_scratch_bytes(void);

/* Device address of that scratch array on the current device (no counterpart in the reference).
 * Its first int32 is the status word of the last solattn_sol_forward_noalloc call on the device:
 * pass it to solattn_status_to_host for a check that does not block. */
SOLATTN_API int solattn_noalloc_scratch_address(void** address);

/* solattn_read_status on the no-allocation status word of the current device (no counterpart in
 * the reference): synchronises `stream`, returns the word through *value and clears it. */
SOLATTN_API int solattn_noalloc_read_status(int32_t* value, void* stream);

/*
 * Strided 2-D copy between host and device memory on `stream` (no counterpart in the reference,
 * whose API takes device tensors only): `rows` rows of `width_bytes` bytes, consecutive rows
 * `src_pitch` / `dst_pitch` bytes apart.  direction 0 = host -> device, 1 = device -> host.
 * A BTHD tensor's slice of heads [h0, h1) is B*T rows of (h1-h0)*D*2 bytes at pitch H*D*2, so
 * host-resident inputs can be moved head group by head group (sol_attn_b200.host streams the
 * groups through the GPU with the copies overlapping the compute).  Pinned host memory is needed
 * for the copy to be asynchronous.
 */
SOLATTN_API int solattn_copy_2d(void* dst, int64_t dst_pitch, const void* src, int64_t src_pitch,
                                int64_t width_bytes, int64_t rows, int direction, void* stream);

/*
 * Enqueues on `stream` an asynchronous copy of the device status word at `status` into
 * `host_dst` (pinned host memory for the copy to stay asynchronous) and returns at once.  The
 * word is final once the stream has passed the copy (an event recorded after it has
 * completed); nonzero = a kernel of the calls enqueued before reported a device-side error
 * (1 a bounded wait ran out, 2 an index outside its tensor, 3 TMEM, 4 a TMA coordinate).
 * The Python layer copies every call's status this way and raises on the next call (or on
 * SolStats.density()), so production calls never block on it.  No counterpart in the
 * reference, whose kernels report nothing.
 */
SOLATTN_API int solattn_status_to_host(const int32_t* status, int32_t* host_dst, void* stream);

/*
 * Synchronises `stream`, copies the device status word at `status` to the host, clears it
 * and returns it through *value (0 = no device-side error).  It blocks: the non-blocking form
 * is solattn_status_to_host.
 */
SOLATTN_API int solattn_read_status(int32_t* status, int32_t* value, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SOLATTN_H_ */
