/*
 * oscar_b200.h -- C ABI of the B200-native OSCAR INT2 rotated KV-cache hot path.
 *
 * Every entry point takes plain pointers and sizes (no framework types), runs
 * asynchronously on the CUDA stream passed as `stream` (a cudaStream_t; NULL =
 * legacy default stream) and returns a status code:
 *
 *   OSCAR_OK (0)            launched
 *   OSCAR_ERR_INVALID (1)   invalid layout, size or geometry (the Python layer raises ValueError)
 *   OSCAR_ERR_UNSUPPORTED(2) a valid layout this build has no kernel for
 *   OSCAR_ERR_CUDA (3)      the CUDA runtime reported an error (RuntimeError)
 *
 * oscar_last_error() returns the message of the last failure on the calling thread.
 *
 * Device pointers: every tensor argument is device memory unless it is marked
 * HOST.  Caches are byte views of the paged KV caches, shape
 * [num_blocks, block_size, num_kv_heads, slot_bytes] with strides in bytes.
 * Slot layout (oscar_ascend/format.py:19-38, kernels/store_kernel.py:4-9):
 *   K slot: [0:2] K scale fp16 LE | [2:4] K zero | [4:6] V scale | [6:8] V zero
 *           | [8:32] pad (never written) | [32:32+D/4] K codes (4 per byte, low index in low bits)
 *   V slot: [0:D/4] V codes
 *
 * Indices read from device memory (slot_mapping, block tables, owner tags)
 * are bounds-checked inside the kernels: an out-of-range index skips the
 * access and latches a device error flag that oscar_device_error() reads.
 */
#ifndef OSCAR_B200_H
#define OSCAR_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { OSCAR_OK = 0, OSCAR_ERR_INVALID = 1, OSCAR_ERR_UNSUPPORTED = 2, OSCAR_ERR_CUDA = 3 };
enum { OSCAR_DTYPE_F32 = 0, OSCAR_DTYPE_BF16 = 1, OSCAR_DTYPE_F16 = 2 };

/* ABI version of this header (bumped on any signature change). */
int oscar_abi_version(void);

/* Message of the last failed call on this thread ("" if none). */
const char* oscar_last_error(void);

/* Number of kernels this library has launched in this process (all devices). */
uint64_t oscar_launch_count(void);

/* Selects the attention kernel family for later oscar_slab_attention calls
 * in this process: 0 = automatic (the tcgen05 decode kernel where eligible —
 * D = 256, at most 32 query rows per GQA group, a history that fits its
 * plan — else the mma.sync decode kernel where eligible, else the tile
 * kernel), 1 = the tile kernel only, 2 = the mma.sync decode kernel where
 * eligible (else the tile kernel), 3 = the tcgen05 decode kernel where
 * eligible (else the tile kernel).  All families compute the same function;
 * the switch keeps each of them parity-tested.  Other values: status 1. */
int oscar_set_attention_path(int path);

/* Selects the rotation kernel for later oscar_rotate_rows* and layer-step
 * calls in this process, chosen per segment by the segment's own size: 0 =
 * automatic (fp32 segments of at least 2560 rows -- the attention output's
 * o @ R_v^T -- on the tcgen05 kind::tf32 kernel; 16-bit segments of at least
 * 6144 rows -- the k / v / q rotations, whose rounding the INT2 codes and
 * the attention scores are sensitive to -- on the register-tiled fp32 FMA
 * kernel (D 128 or 256; 64-row tiles below 16384 rows, 128-row tiles from
 * there); the rest on the fp32 FMA kernel of 16-row tiles), 1 = the 16-row
 * FMA kernel only, 2 = the tensor-core kernel, 3 = the register-tiled FMA
 * kernel (D 128 or 256, tiles by size as above).  The last two need 16-byte
 * aligned output rows, else the 16-row kernel runs.  The tensor-core kernel splits R (and fp32
 * x) into two tf32 terms, so both compute x @ R to within a few fp32 ulps;
 * the switch keeps both parity-tested.  Other values: status 1. */
int oscar_set_rotation_path(int path);

/* Synchronises `stream`, returns and clears the device-side bounds flag of the
 * current device: 0 = clean, otherwise a bitmask (1 = slot out of range,
 * 2 = block-table entry out of range, 8 = merge target row out of range,
 * 16 = a tensor-core decode wait timed out, 32 = more history splits per
 * request than the tensor-core merge holds).
 * Debug/test helper; the hot path never synchronises. */
int oscar_device_error(void* stream);

/* ------------------------------------------------------------------------
 * K1  INT2 store: clip -> per-vector asymmetric INT2 quantize -> pack -> scatter.
 *
 * Replaces kernels/store_kernel.py:54-102 (oscar_store_ref) and :247-279
 * (oscar_store_triton); the clamp of backend.py:140-146 (_rotate_clip) is
 * folded in (clip ratio 0 = no clamp, so with 0/0 this is oscar_store_ref).
 * Codes and scale/zero bytes are bit-exact with the reference for identical
 * rotated fp32 input.  slot_mapping < 0 skips the token.
 */
int oscar_store_int2(const float* k_rot, const float* v_rot, /* [n_tokens, num_kv_heads, head_dim] fp32 */
                     int64_t n_tokens, int32_t num_kv_heads, int32_t head_dim,
                     float k_clip_ratio, float v_clip_ratio,
                     uint8_t* k_cache, uint8_t* v_cache, int64_t num_blocks, int32_t block_size,
                     int64_t k_stride_block, int64_t k_stride_token, int64_t k_stride_head,
                     int64_t v_stride_block, int64_t v_stride_token, int64_t v_stride_head,
                     const int64_t* slot_mapping, /* [n_tokens] */
                     void* stream);

/* ------------------------------------------------------------------------
 * K5  FP32 sink/recent staging window.
 *
 * oscar_staging_invalidate replaces the owner invalidation of
 * backend.py:172-176 (do_kv_cache_update): owner[seat(slot)] = -1 for every
 * slot >= 0, seat = (slot / block_size % stage_rows, slot % block_size).
 *
 * oscar_staging_write replaces backend.py:513-555 (_staging_write): for every
 * seat written this call the LAST token (in token order) wins; its owner tag
 * becomes slot / block_size if the token is inside the sink or recent window
 * (pos < sink_eff || pos >= seq - recent) else -1, and kept tokens store
 * their rotated, UNCLIPPED fp32 K/V in the arena.  Token t belongs to request
 * r with qsl[r] <= t < qsl[r+1]; its position is seqs[r] - qsl[r+1] + t.
 * `seat_winner` is caller-owned scratch of stage_rows*block_size uint64,
 * zeroed once; `epoch` must increase by one per call on the same arena
 * (first call: 1).  The scratch is never cleared between calls.
 */
int oscar_staging_invalidate(const int64_t* slot_mapping, int64_t n_tokens,
                             int64_t* owner, int64_t stage_rows, int32_t block_size,
                             void* stream);

int oscar_staging_write(const float* k_rot, const float* v_rot, /* [n_tokens, num_kv_heads, head_dim] */
                        int64_t n_tokens, int32_t num_kv_heads, int32_t head_dim,
                        const int64_t* slot_mapping,           /* [n_tokens] */
                        const int32_t* qsl, const int32_t* seqs, int32_t num_requests, /* device [B+1], [B] */
                        int32_t sink_eff, int32_t recent_tokens,
                        float* stage_k, float* stage_v, int64_t* owner, /* [rows, bs, Hk, D], [rows, bs] */
                        int64_t stage_rows, int32_t block_size,
                        uint64_t* seat_winner, uint32_t epoch,
                        void* stream);

/* The write side of a decode-sized step in one launch: oscar_store_int2 and
 * oscar_staging_write of the same tokens (same arguments), for at most 256
 * tokens and 256 requests (OSCAR_ERR_UNSUPPORTED beyond).  No counterpart in
 * the reference, whose forward runs do_kv_cache_update (owner invalidation,
 * rotate/clip, store; backend.py:151-198) then _staging_write
 * (backend.py:513-555): the invalidation is left out because every seat it
 * clears is rewritten by that seat's last writer, and the last writer per seat
 * is found without scratch or epoch (the call can be replayed from a graph). */
int oscar_write_step(const float* k_rot, const float* v_rot, int64_t n_tokens, int32_t num_kv_heads, int32_t head_dim,
                     float k_clip_ratio, float v_clip_ratio, uint8_t* k_cache, uint8_t* v_cache, int64_t num_blocks,
                     int32_t block_size, int64_t k_stride_block, int64_t k_stride_token, int64_t k_stride_head,
                     int64_t v_stride_block, int64_t v_stride_token, int64_t v_stride_head,
                     const int64_t* slot_mapping, const int32_t* qsl, const int32_t* seqs, int32_t num_requests,
                     int32_t sink_eff, int32_t recent_tokens, float* stage_k, float* stage_v, int64_t* owner,
                     int64_t stage_rows, void* stream);

/* Staging-window write for callers that cannot allocate device memory.
 * No counterpart in the reference.  Same semantics and arguments as
 * oscar_staging_write, minus seat_winner/epoch: the scratch is a static
 * device array inside this library holding at most 65536 seats
 * (stage_rows * block_size; larger arenas return OSCAR_ERR_INVALID), so an
 * engine that has given all device memory to its KV cache, or a host that
 * forbids allocations outside start-up, can still run the write.  Each GPU
 * that loads the library keeps that 512 KiB for the life of the process.
 * The first call on a device looks up the array's device address (set-up);
 * make that first call before any stream capture.  All calls share the one
 * array (cleared at the start of every call), so calls that overlap on the
 * GPU -- on different streams, or from different threads -- race. */
int oscar_staging_write_noalloc(const float* k_rot, const float* v_rot, int64_t n_tokens, int32_t num_kv_heads,
                                int32_t head_dim, const int64_t* slot_mapping, const int32_t* qsl,
                                const int32_t* seqs, int32_t num_requests, int32_t sink_eff, int32_t recent_tokens,
                                float* stage_k, float* stage_v, int64_t* owner, int64_t stage_rows,
                                int32_t block_size, void* stream);

/* ------------------------------------------------------------------------
 * K2/K3/K4  streaming attention over paged INT2 history.
 *
 * Replaces kernels/slab_attention.py:376-476 (slab_attention) -- semantics of
 * kernels/streaming_attention.py:134-196 (streaming_attention_ref): exact
 * softmax attention of q over [history from the packed cache, with fp32
 * staged overrides where owner[seat] == block] followed by the current chunk
 * (k_new/v_new, causal, right-aligned).  History values are rounded to fp16
 * and then to the query dtype before use (streaming_attention.py:124).
 * Without k_new (cache-only), request r's keys are [0, seqs[r]) and query i
 * of the request sees keys [0, seqs[r] - q_len + i].
 *
 * q        [n_tokens, num_q_heads, head_dim] (dtype: BF16 or F16)
 * k_new/v_new [n_tokens, num_kv_heads, head_dim] same dtype, or both NULL
 * block_table [bt_rows, bt_stride] int32 (kernel-granular block ids)
 * qsl/seqs HOST int32 arrays [num_requests + 1] / [num_requests]
 * stage_k/stage_v/owner: staging arena or all NULL (stage_rows = 0)
 * out      [n_tokens, num_q_heads, head_dim] fp32 (rotated space)
 * lse      [n_tokens, num_q_heads] fp32, natural log, scale included
 * workspace: device scratch for split-KV partials and, at head dim 256
 *   with q-blocks of 128 rows, the keys' tiles written once by a pre-pass
 *   (ceil(seq / 64) * num_kv_heads * 64 KiB per request, after the partials,
 *   256-byte aligned workspace).  Any size (0 included) is valid -- a small
 *   workspace only lowers parallelism or makes each attention CTA dequantise
 *   its own tiles.  The planned size is oscar_slab_attention_workspace().
 */
int oscar_slab_attention(const void* q, const void* k_new, const void* v_new, int32_t dtype,
                         int64_t n_tokens, int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                         const uint8_t* k_cache, const uint8_t* v_cache, int64_t num_blocks, int32_t block_size,
                         int64_t k_stride_block, int64_t k_stride_token, int64_t k_stride_head,
                         int64_t v_stride_block, int64_t v_stride_token, int64_t v_stride_head,
                         const int32_t* block_table, int64_t bt_rows, int64_t bt_stride,
                         const int32_t* qsl, const int32_t* seqs, int32_t num_requests,
                         float scale,
                         const float* stage_k, const float* stage_v, const int64_t* owner, int64_t stage_rows,
                         float* out, float* lse,
                         void* workspace, int64_t workspace_bytes,
                         void* stream);

/* History-shard attention: the partial (O, LSE) of q over one shard of the
 * paged history, for split-KV across GPUs (each rank holds a page-aligned
 * range of every request's history; the ranks' partials are combined with
 * oscar_merge_slab).  No counterpart entry in the reference: it is the
 * slab loop of kernels/slab_attention.py:458-475 with the slabs of one
 * shard only.  Every key of [0, history_lens[r]) (through block_table row
 * r) is visible to every query row of request r -- the shard holds no keys
 * of the current chunk, which the owner adds in its own pass.  Arguments as
 * oscar_slab_attention without k_new / v_new; history_lens is a HOST int32
 * array.  Runs on the decode kernels only: head_dim 256 and at most 32
 * query rows (q_len x query heads per KV head) per request and KV head,
 * else ERR_UNSUPPORTED. */
int oscar_slab_attention_shard(const void* q, int32_t dtype,
                               int64_t n_tokens, int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                               const uint8_t* k_cache, const uint8_t* v_cache, int64_t num_blocks,
                               int32_t block_size,
                               int64_t k_stride_block, int64_t k_stride_token, int64_t k_stride_head,
                               int64_t v_stride_block, int64_t v_stride_token, int64_t v_stride_head,
                               const int32_t* block_table, int64_t bt_rows, int64_t bt_stride,
                               const int32_t* qsl, const int32_t* history_lens, int32_t num_requests,
                               float scale,
                               const float* stage_k, const float* stage_v, const int64_t* owner,
                               int64_t stage_rows,
                               float* out, float* lse,
                               void* workspace, int64_t workspace_bytes,
                               void* stream);

/* Workspace bytes the planner would use: full split-KV parallelism, plus
 * the continuation pre-pass tiles where that path applies. */
int64_t oscar_slab_attention_workspace(const int32_t* qsl, const int32_t* seqs, int32_t num_requests,
                                       int32_t has_new, int32_t num_q_heads, int32_t num_kv_heads,
                                       int32_t head_dim);

/* ------------------------------------------------------------------------
 * K4  LSE merge of a partial (O, LSE) into a running (O, LSE), in place.
 *
 * Replaces kernels/slab_attention.py:341-373 (merge_slab) / :156-194
 * (_merge_slab): m = max(l1, l2); a = e^(l1-m), b = e^(l2-m);
 * O = (a*O1 + b*O2) / (a+b); LSE = m + log(a+b).  -inf partials contribute
 * nothing (their O is never read), a zero denominator becomes 1, NaN
 * propagates.  Target rows: query_start + i, or query_ids[i] if non-NULL.
 * Also the combine step for split-KV sequence shards across GPUs.
 * out/lse hold out_rows query rows; ids outside [0, out_rows) are skipped
 * and latch device error bit 8.
 */
int oscar_merge_slab(float* out, float* lse, int64_t out_rows, /* [out_rows, num_q_heads, head_dim], [out_rows, num_q_heads] */
                     const void* part, int32_t part_dtype,  /* [n, num_q_heads, head_dim] */
                     const float* part_lse,                 /* [n, num_q_heads] */
                     int64_t n, int32_t num_q_heads, int32_t head_dim,
                     int64_t query_start, const int32_t* query_ids,
                     void* stream);

/* Per-layer rotation of head vectors: out = x @ R (transpose = 0) or
 * x @ R^T (transpose = 1), fp32 products and sums.  No counterpart in the
 * reference's kernel API: backend.py:238-246 (and the k/q/v/output rotations
 * of backend.py:151-198, 334-393) run it as fp32 library GEMMs.  x holds
 * `rows` vectors of head_dim (64, 128 or 256) elements of x_dtype, x_stride
 * elements apart (a multiple of 8; x 16-byte aligned); rot is
 * [head_dim, head_dim] fp32 row-major, 16-byte aligned.
 * Either output may be null: out (out_dtype, out_stride elements between rows)
 * and out_f32 (fp32, out_f32_stride).  Asynchronous on `stream`. */
int oscar_rotate_rows(const void* x, int32_t x_dtype, int64_t rows, int64_t x_stride, int32_t head_dim,
                      const float* rot, int32_t transpose,
                      void* out, int32_t out_dtype, int64_t out_stride,
                      float* out_f32, int64_t out_f32_stride,
                      void* stream);

/* One segment of oscar_rotate_rows_batch: the arguments of
 * oscar_rotate_rows for one tensor. */
typedef struct oscar_rotate_seg {
  const void* x;
  int64_t rows;
  int64_t x_stride;
  const float* rot;
  int32_t transpose;
  void* out;
  int64_t out_stride;
  float* out_f32;
  int64_t out_f32_stride;
} oscar_rotate_seg;

/* Up to 4 rotations in one launch (e.g. the step's queries with R_k and its
 * keys / values with R_k / R_v); every segment shares x_dtype, head_dim and
 * out_dtype, and follows the rules of oscar_rotate_rows.  No counterpart in
 * the reference's kernel API. */
int oscar_rotate_rows_batch(const oscar_rotate_seg* segs, int32_t n_segs, int32_t x_dtype, int32_t head_dim,
                            int32_t out_dtype, void* stream);

/* ------------------------------------------------------------------------
 * One FULL-attention layer step of a decode-sized batch in one call: the
 * backend forward of backend.py:249-282 (streaming mode, staging window on)
 * when every request has cached history, n_tokens <= 256 and
 * num_requests <= 256.  No counterpart entry in the reference, where the
 * forward is Python around its kernels; here the host cost of a decode step
 * is one call.  In order, on `stream`:
 *   1. k @ R_k and v @ R_v (fp32 rows for the store and the window, query
 *      dtype rows for the attention) and q @ R_k (query dtype), one launch;
 *   2. oscar_write_step of the step's tokens (clip + INT2 store + staging);
 *   3. oscar_slab_attention over the history and the causal chunk, rotated;
 *   4. o @ R_v^T into `out` in the query dtype.
 * q [n, Hq, D], k / v [n, Hk, D]: heads contiguous, token rows q_stride /
 * k_stride / v_stride elements apart (multiples of 8; e.g. views of a fused
 * QKV projection); out [n, Hq * D] rows out_stride elements apart.  R_k, R_v
 * and R_v^T are fp32 [D, D] row-major.  slot_mapping / qsl_dev / seqs_dev
 * are device arrays (oscar_write_step), qsl / seqs the same on the HOST.
 * scratch: device memory, 256-byte aligned, at least
 * oscar_decode_layer_step_scratch() bytes for the step's rotated rows and
 * attention output; bytes beyond that are the attention workspace
 * (oscar_slab_attention's `workspace`).  A request without cached history
 * returns ERR_UNSUPPORTED (its chunk attends in the model's domain). */
int oscar_decode_layer_step(const void* q, const void* k, const void* v, int32_t dtype, int64_t q_stride,
                            int64_t k_stride, int64_t v_stride, int64_t n_tokens, int32_t num_q_heads,
                            int32_t num_kv_heads, int32_t head_dim, const float* rot_k, const float* rot_v,
                            const float* rot_vt, float k_clip_ratio, float v_clip_ratio, uint8_t* k_cache,
                            uint8_t* v_cache, int64_t num_blocks, int32_t block_size, int64_t k_stride_block,
                            int64_t k_stride_token, int64_t k_stride_head, int64_t v_stride_block,
                            int64_t v_stride_token, int64_t v_stride_head, const int64_t* slot_mapping,
                            const int32_t* qsl_dev, const int32_t* seqs_dev, const int32_t* block_table,
                            int64_t bt_rows, int64_t bt_stride, const int32_t* qsl, const int32_t* seqs,
                            int32_t num_requests, int32_t sink_eff, int32_t recent_tokens, float scale,
                            float* stage_k, float* stage_v, int64_t* owner, int64_t stage_rows, void* out,
                            int64_t out_stride, void* scratch, int64_t scratch_bytes, void* stream);

/* Bytes of oscar_decode_layer_step's scratch before the attention workspace. */
int64_t oscar_decode_layer_step_scratch(int64_t n_tokens, int32_t num_q_heads, int32_t num_kv_heads,
                                        int32_t head_dim, int32_t dtype);

#ifdef __cplusplus
}
#endif

#endif /* OSCAR_B200_H */
