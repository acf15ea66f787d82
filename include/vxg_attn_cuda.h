/*
 * vxg_attn_cuda.h -- C ABI of the B200 (sm_100a) backend for the vxg-tensor attention hot path:
 * Q8_0 KV-cache append, split-KV GQA decode attention over that cache, and the gated-DeltaNet
 * recurrent state update.
 *
 * It extends the reference's native GPU ABI conventions (native/abi.h:1-10, native/cuda.cu:31-68):
 *   - create() returns an opaque handle or NULL and writes a message into (err, cap);
 *   - every other call returns int: 0 = ok, < 0 = error class (values of include/vxg.h:22-30),
 *     and writes a message into (err, cap) on failure;
 *   - a failed call synchronises its stream before returning, so no copy still targets caller
 *     memory (native/cuda.cu:62-65);
 *   - a device (CUDA) error poisons the context: every later call fails with
 *     VXG_ATTN_ERR_INTERNAL, like a failed GPU state in the reference (docs/GPU.md:5-8,
 *     crates/vxg-tensor/src/llm.rs:546-550).  There is no CPU fallback.
 * Plain C types only: pointers, sizes, ints, floats.
 *
 * KV layout (unchanged from the reference): a KV pool holds, for each of n_seq sequences, cap
 * tokens of KvQ8Block[n_head_kv][head_dim/32] for K and the same for V, i.e. the byte image of
 * the reference's per-layer Vec<KvQ8Block> (crates/vxg-tensor/src/llm_prefill.rs:17-24,
 * 311-324) at offset seq * cap * n_head_kv * (head_dim/32) * 34.
 *
 * Pointers marked "mem" are host or device memory according to the call's `memkind`.  With
 * VXG_ATTN_MEM_HOST the call copies in and out itself (pinned host memory is fastest; see
 * vxg_attn_cuda_host_alloc).  `stream` may be NULL: the call then runs on the context's stream
 * and returns when the results are in place.  A non-NULL stream (cudaStream_t) makes
 * device-memory calls asynchronous on that stream; call vxg_attn_cuda_sync to collect device
 * status.  One context per host thread; contexts are not thread-safe.
 * Float / bf16 arrays in device memory (and the KV pools passed to
 * vxg_attn_cuda_q8_decode_noalloc) must be 16-byte aligned; a misaligned one is rejected with
 * VXG_ATTN_ERR_INVALID_OPTION.  Host-memory calls accept any alignment.
 */
#ifndef VXG_ATTN_CUDA_H
#define VXG_ATTN_CUDA_H
#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define VXG_ATTN_API __attribute__((visibility("default")))
#else
#define VXG_ATTN_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes (values of the reference's include/vxg.h:22-30). */
#define VXG_ATTN_OK 0
#define VXG_ATTN_WARN_NONFINITE 1       /* success, but an output is NaN/Inf (as on the CPU)   */
#define VXG_ATTN_ERR_NULL_PTR (-1)
#define VXG_ATTN_ERR_INVALID_OPTION (-2)
#define VXG_ATTN_ERR_BUFFER_TOO_SMALL (-3)
#define VXG_ATTN_ERR_UNSUPPORTED (-6)
#define VXG_ATTN_ERR_INTERNAL (-7)      /* CUDA error; the context is poisoned                 */

#define VXG_ATTN_MEM_HOST 0
#define VXG_ATTN_MEM_DEVICE 1

/* Library version string (as vxg_version_string, include/vxg.h:40). */
VXG_ATTN_API const char* vxg_attn_cuda_version(void);

/* ---------------------------------------------------------------- context ------------------ */
/* Binds device $VXG_CUDA_DEVICE (default: the current device), creates a stream; on success
 * writes the device name into err.  Mirrors vxg_cuda_create (native/cuda.cu:31-41). */
VXG_ATTN_API void* vxg_attn_cuda_create(char* err, size_t cap);
/* Synchronises and frees the context (native/cuda.cu:68). */
VXG_ATTN_API void vxg_attn_cuda_destroy(void* ctx);
/* Waits for all work on `stream` (NULL: the context stream), then reports the device status
 * word (no counterpart: the reference's CUDA calls return only when done, native/cuda.cu:43-66): VXG_ATTN_WARN_NONFINITE, VXG_ATTN_ERR_INVALID_OPTION for skipped out-of-range entries,
 * VXG_ATTN_ERR_INTERNAL for a device error or a bounded wait that gave up. */
VXG_ATTN_API int vxg_attn_cuda_sync(void* ctx, void* stream, char* err, size_t cap);
/* Number of SMs of the bound device (the split-KV grid size).  No counterpart in the reference. */
VXG_ATTN_API int vxg_attn_cuda_sm_count(void* ctx);
/* Device time in ms of the last split-KV attention pass launched on the context (when timing
 * is enabled with vxg_attn_cuda_set_timing); -1 if unavailable.  Like the reference's
 * kernel_ms out-parameter (native/cuda.cu:52-60). */
VXG_ATTN_API int vxg_attn_cuda_set_timing(void* ctx, int enable);
VXG_ATTN_API double vxg_attn_cuda_last_split_ms(void* ctx);
/* Test hook: 1 forces the portable split kernel for every shape (cross-check of the fast one).
 * No counterpart in the reference. */
VXG_ATTN_API int vxg_attn_cuda_force_generic(void* ctx, int enable);

/* Device / pinned memory for callers without a CUDA toolchain (Rust, C).  No counterpart in the
 * reference, whose CUDA codec allocates inside each call (native/cuda.cu:43-66). */
VXG_ATTN_API void* vxg_attn_cuda_malloc(void* ctx, size_t bytes, char* err, size_t cap);
VXG_ATTN_API void vxg_attn_cuda_free(void* ctx, void* dptr);
VXG_ATTN_API void* vxg_attn_cuda_host_alloc(void* ctx, size_t bytes, char* err, size_t cap);
VXG_ATTN_API void vxg_attn_cuda_host_free(void* ctx, void* hptr);
/* kind: 0 host->device, 1 device->host, 2 device->device.  Synchronous. */
VXG_ATTN_API int vxg_attn_cuda_memcpy(void* ctx, void* dst, const void* src, size_t bytes, int kind, char* err,
                         size_t cap);

/* ---------------------------------------------------------------- Q8 KV pool --------------- */
/* Replaces the per-layer Vec<KvQ8Block> pair of LlmState (crates/vxg-tensor/src/llm.rs:36-41,
 * 290-338) and vxt_metal_cb4_fast_state_create (crates/vxg-tensor/src/metal_cb4_fast_ffi.rs:
 * 149-154): zero-filled device K and V pools of n_seq x cap_tokens tokens.  head_dim must be a
 * multiple of 32 (llm.rs:291) and at most 256. */
VXG_ATTN_API void* vxg_attn_cuda_kv_create(void* ctx, uint32_t n_seq, uint32_t n_head_kv, uint32_t head_dim,
                              uint32_t cap_tokens, char* err, size_t cap);
/* Frees the pools (vxt_metal_cb4_fast_state_destroy, metal_cb4_fast_ffi.rs:156). */
VXG_ATTN_API void vxg_attn_cuda_kv_destroy(void* kv);
/* Bytes held by the K and V pools (metal_cb4_fast_ffi.rs:157, llm.rs:340-346). */
VXG_ATTN_API size_t vxg_attn_cuda_kv_bytes(void* kv);
/* Tokens per sequence the pools hold now (grown by vxg_attn_cuda_kv_reserve).  No counterpart:
 * the reference's Vec<KvQ8Block> grows implicitly (llm_prefill.rs:311-324). */
VXG_ATTN_API uint32_t vxg_attn_cuda_kv_capacity(void* kv);
/* Grows every sequence to at least cap_tokens tokens, keeping contents (doubling policy of
 * native/metal_cb4_fast.h:174-191). */
VXG_ATTN_API int vxg_attn_cuda_kv_reserve(void* kv, uint32_t cap_tokens, char* err, size_t cap);
/* Device base pointers of the K and V pools and the byte stride between sequences (for
 * vxg_attn_cuda_q8_decode_noalloc and callers' own kernels).  No counterpart in the reference. */
VXG_ATTN_API int vxg_attn_cuda_kv_device_ptrs(void* kv, void** k_pool, void** v_pool, size_t* seq_stride);
/* Byte-identical import / export of tokens [tok_begin, tok_begin + n_tok) of sequence `seq`:
 * k_blocks / v_blocks are n_tok * n_head_kv * head_dim/32 KvQ8Blocks (34 B each), i.e. a slice
 * of the reference's Vec<KvQ8Block>. */
VXG_ATTN_API int vxg_attn_cuda_kv_import(void* ctx, void* kv, uint32_t seq, uint32_t tok_begin, uint32_t n_tok,
                            const void* k_blocks, const void* v_blocks, int memkind, char* err,
                            size_t cap);
VXG_ATTN_API int vxg_attn_cuda_kv_export(void* ctx, void* kv, uint32_t seq, uint32_t tok_begin, uint32_t n_tok,
                            void* k_blocks, void* v_blocks, int memkind, char* err, size_t cap);

/* Checkpoint / restore of recurrent state buffers (vxt_metal_cb4_fast_checkpoint,
 * native/metal_cb4_fast.mm:531-570): for i < n_buffers, copies bytes[i] device bytes from
 * states[i] to backups[i] (restore == 0) or back (restore != 0), e.g. the DeltaNet ssm and conv
 * states of every recurrent layer before a speculative step.  Device-to-device, on `stream`
 * (asynchronous) or synchronous when stream is NULL. */
VXG_ATTN_API int vxg_attn_cuda_state_checkpoint(void* ctx, uint32_t n_buffers, void* const* states,
                                                void* const* backups, const size_t* bytes,
                                                uint32_t restore, void* stream, char* err,
                                                size_t cap);

/* fp32 KV pools (KvCacheMode::Fp32, the reference's default, llm.rs:287): the per-layer
 * `k_caches` / `v_caches` vectors of LlmState (llm.rs:36-41) as device pools of
 * float[n_seq][cap_tokens][n_head_kv][head_dim] (token rows appended as in llm_ops.rs:256-257).
 * head_dim must be a multiple of 32 and at most 256.  kv_bytes, kv_capacity, kv_reserve,
 * kv_device_ptrs, kv_import and kv_export work on these pools too (import / export move raw
 * f32 rows: n_tok * n_head_kv * head_dim floats per cache). */
VXG_ATTN_API void* vxg_attn_cuda_kv_create_f32(void* ctx, uint32_t n_seq, uint32_t n_head_kv,
                                               uint32_t head_dim, uint32_t cap_tokens, char* err,
                                               size_t cap);

/* ---------------------------------------------------------------- ops ---------------------- */
/* Quantise-and-append (llm_prefill.rs:311-324 with KvQ8Block::quantize, :27-42), bit-exact:
 * for b < n_batch, t < n_tok: k_new/v_new[b][t][n_head_kv][head_dim] (f32, mem) go to sequence
 * seq_ids[b] at position pos[b] + t.  seq_ids, pos: int32 [n_batch] (mem). */
VXG_ATTN_API int vxg_attn_cuda_q8_append(void* ctx, void* kv, uint32_t n_batch, uint32_t n_tok,
                            const int32_t* seq_ids, const int32_t* pos, const float* k_new,
                            const float* v_new, int memkind, void* stream, char* err, size_t cap);

/* Batched decode step = append then attend, the order of step_full_gqa_q8
 * (llm_prefill.rs:311-369): for each b, if k_new != NULL the new token's K/V
 * ([n_batch][n_head_kv][head_dim] f32) is appended at pos[b] of seq_ids[b]; then the query
 * q[b] ([n_head][head_dim] f32, already normed / RoPE'd) attends to tokens [0, pos[b]] with
 * softmax scale `scale` (1/sqrt(head_dim) in the reference).  q_gate (nullable, same shape as q)
 * applies out *= sigmoid(gate) (llm_prefill.rs:363-368).  out: [n_batch][n_head][head_dim].
 * max_ctx: an upper bound of pos[b] + 1 (0 = the pool capacity).
 * The KV ranges are split across the SMs in proportion to the rates the previous call of the
 * context measured (batches of two or more entries), so two identical calls can sum a query's
 * partials in a different order and differ in the last bits (within the accuracy bound). */
VXG_ATTN_API int vxg_attn_cuda_q8_decode(void* ctx, void* kv, uint32_t n_batch, uint32_t n_head,
                            const int32_t* seq_ids, const int32_t* pos, const float* q,
                            const float* k_new, const float* v_new, const float* q_gate,
                            float scale, uint32_t max_ctx, float* out, int memkind, void* stream,
                            char* err, size_t cap);

/* The decode step of vxg_attn_cuda_q8_decode on host memory, overlapped with its neighbours.
 * No counterpart in the reference, whose step is synchronous (llm_prefill.rs:311-369 called once
 * per token).  The call validates like the host-memory form of vxg_attn_cuda_q8_decode, queues
 * the upload of its inputs on a copy stream, the step's kernels on the context stream and the
 * download of `out` on a second copy stream, and returns at once with *ticket naming the step.
 * Consecutive steps alternate between two device staging slots, so the upload of step t+1 and
 * the download of step t-1 run while the kernels of step t do; queueing step t+2 first waits for
 * step t to be back on the host.  Inputs are read, and `out` written, asynchronously: keep the
 * input buffers unchanged and do not read `out` until vxg_attn_cuda_ticket_wait has returned for
 * the ticket.  Pinned host memory (vxg_attn_cuda_host_alloc) is required for the copies to
 * overlap.  (The Metal runner's asynchronous pair vxt_metal_cb4_fast_enqueue_async / _wait_cmd,
 * metal_cb4_fast_ffi.rs:194-204, is the nearest shape.) */
VXG_ATTN_API int vxg_attn_cuda_q8_decode_host_async(void* ctx, void* kv, uint32_t n_batch,
                            uint32_t n_head, const int32_t* seq_ids, const int32_t* pos,
                            const float* q, const float* k_new, const float* v_new,
                            const float* q_gate, float scale, uint32_t max_ctx, float* out,
                            uint64_t* ticket, char* err, size_t cap);
/* Waits until the step `ticket` is back on the host and returns its outcome with the codes of
 * vxg_attn_cuda_sync (VXG_ATTN_OK, VXG_ATTN_WARN_NONFINITE, VXG_ATTN_ERR_INVALID_OPTION for
 * skipped out-of-range entries, VXG_ATTN_ERR_INTERNAL).  Ticket 0 and tickets already waited for
 * return VXG_ATTN_OK. */
VXG_ATTN_API int vxg_attn_cuda_ticket_wait(void* ctx, uint64_t ticket, char* err, size_t cap);

/* The same decode step as vxg_attn_cuda_q8_decode for callers that cannot allocate device
 * memory.  This entry point has no counterpart in the reference.  It is for engines whose device
 * memory belongs to a budgeted pool or to another framework's allocator, and for decode loops
 * that must not stall on cudaMalloc, which can synchronise the device.  It allocates nothing:
 * every argument is caller-owned device memory, the KV pools included (layout as above, e.g.
 * from vxg_attn_cuda_kv_device_ptrs or the caller's own buffers), and its split-KV scratch is a
 * built-in 32 MiB device array that each GPU using the library keeps until the process exits.
 * A batch whose scratch does not fit is rejected with VXG_ATTN_ERR_BUFFER_TOO_SMALL (at 16 q /
 * 2 kv heads, head_dim 256 on a 148-SM B200: up to 190 entries per call; fewer on GPUs with more
 * SMs).  Other shapes run the generic split kernel, whose scratch grows with cap_tokens, so there
 * the batch limit falls as the pools' capacity grows (63 entries at 16 q heads, head_dim 128
 * and a 32768-token pool).  All calls on a device share that array, so calls that overlap on
 * the GPU race; serialise them.  The first call on a device sets up the array's address for that
 * device; make it before any stream capture.  That address is kept per device index for the
 * device's primary context (the CUDA runtime's default); do not call this from a second,
 * driver-API context on the same device.  With
 * stream == NULL the call runs on the default stream and reports the device status like
 * vxg_attn_cuda_q8_decode; with a stream it is asynchronous and reports launch errors only. */
VXG_ATTN_API int vxg_attn_cuda_q8_decode_noalloc(
    void* k_pool, void* v_pool, uint32_t n_seq, uint32_t cap_tokens, uint32_t n_head_kv,
    uint32_t head_dim, uint32_t n_batch, uint32_t n_head, const int32_t* seq_ids,
    const int32_t* pos, const float* q, const float* k_new, const float* v_new,
    const float* q_gate, float scale, float* out, void* stream, char* err, size_t cap);

/* fp32-KV counterparts of vxg_attn_cuda_q8_append / _q8_decode on pools from
 * vxg_attn_cuda_kv_create_f32: the append copies k_new/v_new rows (llm_ops.rs:256-257) and the
 * attention is step_full_gqa's (llm_ops.rs:258-299): scores q.k * scale, softmax, sum p v,
 * optional sigmoid gate.  Same arguments and layouts as the Q8 calls. */
VXG_ATTN_API int vxg_attn_cuda_f32_append(void* ctx, void* kv, uint32_t n_batch, uint32_t n_tok,
                                          const int32_t* seq_ids, const int32_t* pos,
                                          const float* k_new, const float* v_new, int memkind,
                                          void* stream, char* err, size_t cap);
VXG_ATTN_API int vxg_attn_cuda_f32_decode(void* ctx, void* kv, uint32_t n_batch, uint32_t n_head,
                                          const int32_t* seq_ids, const int32_t* pos,
                                          const float* q, const float* k_new, const float* v_new,
                                          const float* q_gate, float scale, uint32_t max_ctx,
                                          float* out, int memkind, void* stream, char* err,
                                          size_t cap);

/* Chunked prefill of n_tok prompt tokens per sequence, the batched form of what the reference
 * runs token by token (prefill_cpu_tiled, llm_prefill.rs:497-527, calling step_full_gqa_q8,
 * :311-369) and of the Metal prefill pair vxt_cb4_gqa_prep_batch + vxt_cb4_gqa_attn_batch
 * (native/metal_cb4_fast_run.mm:283-308): for b < n_batch, t < n_tok, the K/V of prompt token t
 * (k_new/v_new [n_batch][n_tok][n_head_kv][head_dim]) is appended at position pos[b] + t of
 * sequence seq_ids[b], and query token t (q [n_batch][n_tok][n_head][head_dim], prepared)
 * attends causally to the Q8 cache [0, pos[b] + t].  q_gate (nullable, q's shape) applies
 * out *= sigmoid(gate).  out: [n_batch][n_tok][n_head][head_dim] f32.
 * dtype: VXG_ATTN_DTYPE_F32 or VXG_ATTN_DTYPE_BF16 for q, k_new, v_new and q_gate.
 * Supported shapes: head_dim 64, 128 or 256, and n_head / n_head_kv dividing 128.
 * max_ctx: an upper bound of pos[b] + n_tok (0 = the pool capacity); device scratch of
 * 8 * n_batch * max_ctx * n_head_kv * head_dim bytes holds the dequantised cache (f16 hi and
 * lo planes of K and V). */
#define VXG_ATTN_DTYPE_F32 0
#define VXG_ATTN_DTYPE_BF16 1
VXG_ATTN_API int vxg_attn_cuda_q8_prefill(void* ctx, void* kv, uint32_t n_batch, uint32_t n_tok,
                                          uint32_t n_head, const int32_t* seq_ids,
                                          const int32_t* pos, const void* q, const void* k_new,
                                          const void* v_new, const void* q_gate, int dtype,
                                          float scale, uint32_t max_ctx, float* out, int memkind,
                                          void* stream, char* err, size_t cap);

/* Split-KV partial over tokens [kv_begin[b], kv_end[b]) of each sequence (no append): per
 * (b, head) the running max m (log2 units: max_t score_t * log2(e)), the sum
 * l = sum_t 2^(score_t*log2(e) - m) and the unnormalised o = sum_t 2^(...) * v_t.  Shapes:
 * m, l [n_batch][n_head]; o [n_batch][n_head][head_dim].  Empty ranges give m = -inf, l = 0,
 * o = 0.  This is the per-GPU half of the multi-GPU KV-range split; no counterpart in the
 * reference (one device), its softmax (llm_prefill.rs:347-362) re-associated over token ranges. */
VXG_ATTN_API int vxg_attn_cuda_q8_decode_partial(void* ctx, void* kv, uint32_t n_batch, uint32_t n_head,
                                    const int32_t* seq_ids, const int32_t* kv_begin,
                                    const int32_t* kv_end, const float* q, float scale,
                                    uint32_t max_ctx, float* m, float* l, float* o, int memkind,
                                    void* stream, char* err, size_t cap);

/* Log-sum-exp merge of n_parts partials (layout [n_parts][n_rows] for m and l,
 * [n_parts][n_rows][head_dim] for o) into out [n_rows][head_dim]; optional sigmoid gate
 * (llm_prefill.rs:363-368).  The other half of the KV-range split; no counterpart in the
 * reference. */
VXG_ATTN_API int vxg_attn_cuda_lse_combine(void* ctx, uint32_t n_parts, uint32_t n_rows, uint32_t head_dim,
                              const float* m, const float* l, const float* o, const float* gate,
                              float* out, int memkind, void* stream, char* err, size_t cap);
/* The same merge over packed parts, the layout an all-gather of per-rank partials produces:
 * packed[k] = [m (n_rows) | l (n_rows) | o (n_rows * head_dim)] for k < n_parts. */
VXG_ATTN_API int vxg_attn_cuda_lse_combine_packed(void* ctx, uint32_t n_parts, uint32_t n_rows,
                                                  uint32_t head_dim, const float* packed,
                                                  const float* gate, float* out, int memkind,
                                                  void* stream, char* err, size_t cap);

/* ---------------------------------------------------------------- NVLink peer exchange ----- */
/* The all-gather + combine of the long-context KV-range split (vxg_attn_cuda_q8_decode_partial
 * on every rank, then vxg_attn_cuda_lse_combine_packed over the gathered parts) done through
 * NVLink peer memory instead of a collective; no counterpart in the reference (its step runs on
 * one device).  One process per GPU, world <= 8.  Each rank allocates an exchange buffer
 * (vxg_attn_cuda_peer_alloc, which also returns its 64-byte CUDA IPC handle), hands the handle
 * to the other ranks by any host channel, and maps theirs with vxg_attn_cuda_peer_open.
 * vxg_attn_cuda_peer_step then stores this rank's packed partials `send` ([m | l | o], n_rows *
 * (head_dim + 2) floats) into every rank's buffer and, once every rank's partials of the same
 * step have arrived (a wait bounded in time; VXG_ATTN_ERR_INTERNAL from vxg_attn_cuda_sync if it
 * gives up), writes the merged rows to `out` ([n_rows][head_dim], optional sigmoid `gate`).
 * bufs[r] is rank r's buffer as mapped here (bufs[rank] = the own buffer).  Every rank must
 * issue the same sequence of steps; the step counter is kept in device memory, so captured CUDA
 * graphs of steps replay correctly.  Device memory only; asynchronous on `stream` (NULL: the
 * context stream, synchronous).  Buffers are zero-initialised: allocate all of them before the
 * first step and free them only after every rank's last step. */
VXG_ATTN_API size_t vxg_attn_cuda_peer_buffer_bytes(uint32_t world, uint32_t n_rows,
                                                    uint32_t head_dim);
VXG_ATTN_API void* vxg_attn_cuda_peer_alloc(void* ctx, uint32_t world, uint32_t n_rows,
                                            uint32_t head_dim, void* ipc_handle, char* err,
                                            size_t cap);
VXG_ATTN_API void* vxg_attn_cuda_peer_open(void* ctx, const void* ipc_handle, char* err,
                                           size_t cap);
VXG_ATTN_API void vxg_attn_cuda_peer_close(void* ctx, void* mapped);
VXG_ATTN_API void vxg_attn_cuda_peer_free(void* ctx, void* buf);
VXG_ATTN_API int vxg_attn_cuda_peer_step(void* ctx, void* const* bufs, uint32_t world,
                                         uint32_t rank, uint32_t n_rows, uint32_t head_dim,
                                         const float* send, const float* gate, float* out,
                                         void* stream, char* err, size_t cap);

/* Drop-in for step_full_gqa_q8 (llm_prefill.rs:259-278) on host buffers for one sequence `seq`
 * of `kv`: q_raw [n_head][hd] (or [n_head][2*hd] with gated_q), k_cur (updated in place with
 * the normed / RoPE'd K, as in the reference), v_cur [n_head_kv][hd], optional q_norm/k_norm
 * [hd] RMSNorm weights, RoPE parameters, appends at `pos` and writes attn_out [n_head][hd]. */
VXG_ATTN_API int vxg_attn_cuda_step_full_gqa_q8(void* ctx, void* kv, uint32_t seq, const float* q_raw,
                                   float* k_cur, const float* v_cur, const float* q_norm,
                                   const float* k_norm, int gated_q, uint32_t n_head,
                                   uint32_t n_head_kv, uint32_t head_dim, uint32_t pos,
                                   uint32_t rope_pos, uint32_t rope_dim, float rope_freq_base,
                                   int rope_neox, float eps, float* attn_out, char* err,
                                   size_t cap);

/* Drop-in for step_full_gqa (crates/vxg-tensor/src/llm_ops.rs:196-300), the fp32-KV operator:
 * the same argument list (q_raw, k_cur updated in place, v_cur, norms, gated_q, shapes, pos,
 * RoPE at pos, eps, att_cat out) with the layer's fp32 pool + sequence id in place of
 * `&mut Vec<f32>` caches.  Host buffers; synchronous. */
VXG_ATTN_API int vxg_attn_cuda_step_full_gqa(void* ctx, void* kv, uint32_t seq, const float* q_raw,
                                             float* k_cur, const float* v_cur,
                                             const float* q_norm, const float* k_norm,
                                             int gated_q, uint32_t n_head, uint32_t n_head_kv,
                                             uint32_t head_dim, uint32_t pos, uint32_t rope_dim,
                                             float rope_freq_base, int rope_neox, float eps,
                                             float* att_cat, char* err, size_t cap);

/* Gated-DeltaNet core step (llm_ops.rs:139-184) for n_batch sequences:
 * q, k [n_batch][n_kh][dk] (raw, L2-normalised inside, q also scaled by q_scale, 1/sqrt(dk) in
 * the reference), v [n_batch][n_vh][dv], beta_raw / alpha_raw [n_batch][n_vh], ssm_a / dt_bias
 * [n_vh]; state [n_batch][n_vh][dv][dk] updated in place; o [n_batch][n_vh][dv] = S_new q.
 * dk in {64, 128, 256}; dv a multiple of 32. */
VXG_ATTN_API int vxg_attn_cuda_deltanet_step(void* ctx, uint32_t n_batch, uint32_t n_kh, uint32_t n_vh,
                                uint32_t dk, uint32_t dv, const float* q, const float* k,
                                const float* v, const float* beta_raw, const float* alpha_raw,
                                const float* ssm_a, const float* dt_bias, float q_scale, float eps,
                                float* state, float* o, int memkind, void* stream, char* err,
                                size_t cap);

/* Gated-DeltaNet core over n_tok consecutive tokens of each sequence (prefill).  The reference
 * prefill applies the recurrent step token by token (llm_prefill.rs:470-480 calling
 * llm_ops.rs:103-193); this runs the same recurrence with the state kept on chip.  q, k
 * [n_batch][n_tok][n_kh][dk], v [n_batch][n_tok][n_vh][dv], beta_raw / alpha_raw
 * [n_batch][n_tok][n_vh]; state [n_batch][n_vh][dv][dk] updated in place; o
 * [n_batch][n_tok][n_vh][dv] = S_t q_t for every token. */
VXG_ATTN_API int vxg_attn_cuda_deltanet_prefill(
    void* ctx, uint32_t n_batch, uint32_t n_tok, uint32_t n_kh, uint32_t n_vh, uint32_t dk,
    uint32_t dv, const float* q, const float* k, const float* v, const float* beta_raw,
    const float* alpha_raw, const float* ssm_a, const float* dt_bias, float q_scale, float eps,
    float* state, float* o, int memkind, void* stream, char* err, size_t cap);

/* Drop-in for step_deltanet_recurrent (llm_ops.rs:103-121), batched over n_batch sequences:
 * qkv_mixed [n_batch][conv_ch] (conv_ch = 2*n_kh*dk + n_vh*dv), z [n_batch][n_vh*dv],
 * alpha_raw / beta_raw [n_batch][n_vh], ssm_conv1d [conv_ch][k_sz], ssm_a / ssm_dt_bias [n_vh],
 * ssm_norm [dv]; conv_state [n_batch][k_sz-1][conv_ch] and ssm_state [n_batch][n_vh][dv][dk]
 * are updated in place as in the reference; y_concat [n_batch][n_vh*dv] receives
 * RMSNorm(S q) * ssm_norm * SiLU(z).  dk in {64,128,256}, dv a multiple of 32 up to 256. */
VXG_ATTN_API int vxg_attn_cuda_step_deltanet_recurrent(
    void* ctx, uint32_t n_batch, const float* qkv_mixed, uint32_t conv_ch, const float* z,
    const float* alpha_raw, const float* beta_raw, const float* ssm_conv1d, const float* ssm_a,
    const float* ssm_dt_bias, const float* ssm_norm, float* conv_state, float* ssm_state,
    uint32_t n_kh, uint32_t n_vh, uint32_t dk, uint32_t dv, uint32_t k_sz, float eps,
    float* y_concat, int memkind, void* stream, char* err, size_t cap);

#ifdef __cplusplus
}
#endif
#endif /* VXG_ATTN_CUDA_H */
