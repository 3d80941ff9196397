/*
 * turboquant_c.h -- C ABI of the B200 int4 KV-cache attention library
 * (libturboquant_b200.so). Plain C types only: device pointers, sizes, dtype
 * enums and a cudaStream_t passed as void*.
 *
 * Conventions shared by every entry point:
 *   - Return 0 on success, a TQ_ERR_* code otherwise; tq_last_error() gives a
 *     message for the calling thread. Arguments are validated on the host
 *     before anything is launched (the reference throws std::runtime_error
 *     instead: lib/turboquant.cpp:363-365).
 *   - Nothing here allocates device memory. The caller owns inputs, outputs
 *     and any workspace (the reference allocates outputs inside eval_gpu:
 *     lib/turboquant.cpp:372).
 *   - Work is enqueued asynchronously on `stream` (NULL = legacy default
 *     stream); no call synchronises, so calls can be captured in CUDA graphs
 *     once workspaces are allocated.
 *   - Device pointers must be 16-byte aligned (TMA bulk copies).
 *
 * int4 cache layout (the reference's, lib/turboquant.h:197-200, with an
 * explicit token capacity so the cache can be preallocated):
 *   codes   uint32 (B, Hkv, capacity, D/8): element 8w+j of a token row at
 *           bits 4j..4j+3 of word w (lib/turboquant.metal:796-799);
 *   scales  (B, Hkv, capacity, D/64) in sb_dtype (fp16 by default);
 *   biases  same shape/dtype; value = scale * code + bias.
 *   capacity must be a multiple of 4.
 */
#ifndef TURBOQUANT_C_H
#define TURBOQUANT_C_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define TQ_API __attribute__((visibility("default")))
#else
#define TQ_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum tq_dtype { TQ_F32 = 0, TQ_F16 = 1, TQ_BF16 = 2 } tq_dtype;

enum {
  TQ_OK = 0,
  TQ_ERR_INVALID = 1,     /* bad argument (shape, alignment, null pointer) */
  TQ_ERR_UNSUPPORTED = 2, /* valid but not implemented (e.g. head_dim 96) */
  TQ_ERR_CUDA = 3,        /* a CUDA runtime call or launch failed */
  TQ_ERR_WORKSPACE = 4,   /* workspace too small (see *_workspace_size) */
  TQ_ERR_DEVICE = 5       /* a kernel reported an error through the device error word */
};

/* Message for the last failing call on this thread ("" if none). */
TQ_API const char* tq_last_error(void);

/* Library version string. */
TQ_API const char* tq_version(void);

/* No-op kept for source compatibility with the reference
 * (lib/turboquant.h:209, set_metallib_path): there is no shader library to
 * locate; kernels are linked into this shared object. */
TQ_API void tq_set_metallib_path(const char* path);

/* Affine group-64 4-bit quantization of `rows` contiguous rows of head_dim
 * values (MLX quantize(x, 64, 4): engine/gemma4_multilayer.cpp:228-229,
 * tests/test_sdpa_int4.cpp:25-26). scale = (max-min)/15 and bias = min,
 * rounded to sb_dtype; codes = clamp(rint((x-bias)/scale), 0, 15) computed
 * with the rounded scale/bias; a constant group gets scale 0 and codes 0.
 * x: (rows, D) in x_dtype; codes (rows, D/8); scales/biases (rows, D/64). */
TQ_API int tq_quantize(const void* x, tq_dtype x_dtype, int64_t rows, int head_dim, uint32_t* codes,
                void* scales, void* biases, tq_dtype sb_dtype, void* stream);

/* value = scale * code + bias (MLX dequantize(w, s, b, 64, 4):
 * engine/gemma4_multilayer.cpp:307-308, tests/test_sdpa_int4.cpp:31-32).
 * out: (rows, D) in out_dtype. */
TQ_API int tq_dequantize(const uint32_t* codes, const void* scales, const void* biases,
                  tq_dtype sb_dtype, int64_t rows, int head_dim, void* out, tq_dtype out_dtype,
                  void* stream);

/* Quantize-on-append: quantize n_new new tokens per (sequence, KV head) of K
 * and V and write them in place at token slots pos .. pos+n_new-1 of a
 * preallocated cache. Replaces the reference's quantize + concatenate of the
 * whole cache per token (engine/gemma4_multilayer.cpp:228-240).
 * k_new, v_new: (B, Hkv, n_new, D) contiguous in in_dtype.
 * positions: NULL (every sequence appends at `pos`) or a device int32[B]
 * of per-sequence positions. Slots must satisfy slot + n_new <= capacity. */
TQ_API int tq_quantize_append(const void* k_new, const void* v_new, tq_dtype in_dtype, int batch,
                       int num_kv_heads, int head_dim, int n_new, uint32_t* k_quant,
                       void* k_scales, void* k_biases, uint32_t* v_quant, void* v_scales,
                       void* v_biases, tq_dtype sb_dtype, int capacity, int pos,
                       const int32_t* positions, void* stream);

/* Workspace bytes that tq_sdpa_int4 / tq_sdpa_int4_partial need for these
 * sizes (split-KV partials + merge counters). n_tokens is the largest
 * sequence length the call will see. The workspace must be zero-filled once
 * before first use (tq_workspace_init); kernels leave it reusable, and one
 * workspace may serve calls of any size that fits (its first 64 KiB hold
 * merge counters that every call leaves at zero). Calls that share a
 * workspace must not run concurrently. */
TQ_API size_t tq_sdpa_int4_workspace_size(int batch, int num_heads, int num_kv_heads, int head_dim,
                                   int n_tokens, int sliding_window);

/* Zero a workspace (cudaMemsetAsync on `stream`). */
TQ_API int tq_workspace_init(void* workspace, size_t workspace_bytes, void* stream);

/* Fused single-query decode attention straight from the int4 cache
 * (replaces turboquant::sdpa_int4, lib/turboquant.h:202-207 /
 * lib/turboquant.cpp:405-417; same argument order, then sizes).
 *   queries: (B, H, D) in q_dtype, H = num_kv_heads * gqa_factor,
 *            query head h reads KV head h / gqa_factor;
 *   out:     (B, H, D) in out_dtype;
 *   n_tokens: tokens in every sequence, or the maximum when seq_lens (device
 *            int32[B]) is given;
 *   scale multiplies q.k (reference default 1.0);
 *   sliding_window > 0 masks tokens t with (N-1-t) >= sliding_window
 *   (lib/turboquant.metal:779); 0 = global attention.
 * Long contexts are split across CTAs and merged in-kernel; the workspace
 * must hold tq_sdpa_int4_workspace_size(...) bytes (may be NULL when that is
 * 0). head_dim in {128, 256, 512}; gqa_factor in {1, 2, 4, 8}. */
TQ_API int tq_sdpa_int4(const void* queries, tq_dtype q_dtype, const uint32_t* k_quant,
                 const void* k_scales, const void* k_biases, const uint32_t* v_quant,
                 const void* v_scales, const void* v_biases, tq_dtype sb_dtype, int gqa_factor,
                 float scale, int sliding_window, int batch, int num_kv_heads, int head_dim,
                 int n_tokens, int capacity, const int32_t* seq_lens, void* out,
                 tq_dtype out_dtype, void* workspace, size_t workspace_bytes, void* stream);

/* One decode step of one layer: quantize-on-append of the step's new K/V
 * row of every sequence into slot n - 1 of the cache (n = seq_lens[b], or
 * n_tokens), then decode attention over the n tokens. The result, cache
 * bytes included, equals tq_quantize_append(k_new, v_new, ..., pos = n - 1)
 * followed by tq_sdpa_int4; the engine runs those as MLX quantize +
 * concatenate (engine/gemma4_multilayer.cpp:228-236) then
 * turboquant::sdpa_int4 (lib/turboquant.h:202-207). With the tensor-core
 * decode kernel (head_dim 128/256) both happen in ONE launch: the CTA that
 * owns slot n - 1 quantizes the row while its first tiles stream in.
 *   k_new, v_new: (B, num_kv_heads, head_dim) in new_dtype, 16-byte aligned;
 *   other arguments as tq_sdpa_int4. */
TQ_API int tq_sdpa_int4_append(const void* queries, tq_dtype q_dtype, const void* k_new,
                        const void* v_new, tq_dtype new_dtype, uint32_t* k_quant, void* k_scales,
                        void* k_biases, uint32_t* v_quant, void* v_scales, void* v_biases,
                        tq_dtype sb_dtype, int gqa_factor, float scale, int sliding_window,
                        int batch, int num_kv_heads, int head_dim, int n_tokens, int capacity,
                        const int32_t* seq_lens, void* out, tq_dtype out_dtype, void* workspace,
                        size_t workspace_bytes, void* stream);

/* The same step for a ring cache (a sliding-window layer whose capacity is
 * its window): the new row goes to `slot` (its position modulo the capacity)
 * and attention runs over slots [0, n_tokens) unmasked -- a ring of the last
 * W tokens holds exactly the tokens the window rule (N-1-t) < W keeps
 * (lib/turboquant.metal:779), and attention does not depend on their order.
 * Replaces the engine's quantize + concatenate + front trim of sliding
 * layers (engine/gemma4_multilayer.cpp:228-249). batch 1 or a slot shared by
 * every sequence; slot < n_tokens <= capacity. */
TQ_API int tq_sdpa_int4_append_at(const void* queries, tq_dtype q_dtype, const void* k_new,
                           const void* v_new, tq_dtype new_dtype, uint32_t* k_quant,
                           void* k_scales, void* k_biases, uint32_t* v_quant, void* v_scales,
                           void* v_biases, tq_dtype sb_dtype, int gqa_factor, float scale,
                           int batch, int num_kv_heads, int head_dim, int n_tokens, int capacity,
                           int slot, void* out, tq_dtype out_dtype, void* workspace,
                           size_t workspace_bytes, void* stream);

/* The same step with one slot per sequence, read from device memory: slots[b]
 * (int32, device) is where sequence b's new row goes, and attention runs
 * over its seq_lens[b] tokens (seq_lens may be NULL: n_tokens for every
 * sequence) with the sliding window as in tq_sdpa_int4_append (0 for a ring
 * cache). A batch of ring-cache sequences at different positions, or a step
 * whose slots are only known on the device (a captured graph replayed every
 * token). Each slot must lie in [0, its sequence's token count); a slot
 * outside it writes nothing. */
TQ_API int tq_sdpa_int4_append_slots(const void* queries, tq_dtype q_dtype, const void* k_new,
                                     const void* v_new, tq_dtype new_dtype, uint32_t* k_quant,
                                     void* k_scales, void* k_biases, uint32_t* v_quant,
                                     void* v_scales, void* v_biases, tq_dtype sb_dtype,
                                     int gqa_factor, float scale, int sliding_window, int batch,
                                     int num_kv_heads, int head_dim, int n_tokens, int capacity,
                                     const int32_t* seq_lens, const int32_t* slots, void* out,
                                     tq_dtype out_dtype, void* workspace, size_t workspace_bytes,
                                     void* stream);

/* Sequence-split shard of decode attention: this cache holds global token
 * positions [token_offset, token_offset + n_local) of a sequence whose total
 * length is n_total (all sequences of the batch share both). Writes the
 * shard's partial softmax state per query head in the merge layout of
 * tq_lse_merge, fp32: part_out[b] = { o (H, D) unnormalised, ml (H, 2) with
 * m = max score (natural-log units) and l = sum exp(score - m) }.
 * A shard with no visible token writes m = -inf, l = 0, o = 0.
 * No counterpart in the reference (it has no multi-GPU code); it is the
 * per-GPU half of the NCCL all-gather + merge path. */
TQ_API int tq_sdpa_int4_partial(const void* queries, tq_dtype q_dtype, const uint32_t* k_quant,
                         const void* k_scales, const void* k_biases, const uint32_t* v_quant,
                         const void* v_scales, const void* v_biases, tq_dtype sb_dtype,
                         int gqa_factor, float scale, int sliding_window, int batch,
                         int num_kv_heads, int head_dim, int n_local, int capacity,
                         int token_offset, int n_total, float* part_out, void* workspace,
                         size_t workspace_bytes, void* stream);

/* ---- sequence split over peer memory (CUDA IPC + NVLink P2P stores) ------
 * In place of an all-gather + tq_lse_merge: every rank of a sequence split
 * allocates one exchange buffer (tq_peer_buffer_bytes / _alloc, zeroed),
 * shares it with tq_ipc_handle (TQ_IPC_HANDLE_BYTES opaque bytes, exchanged
 * by the caller, e.g. an all-gather of objects) and opens the others' with
 * tq_ipc_open. tq_peer_merge then, in one launch, stores this rank's partial
 * state (the layout of tq_sdpa_int4_partial's part_out) into every rank's
 * buffer, raises a per-rank step flag there, waits for all ranks' flags of the
 * step and writes the merged (B, H, D) output. peer_bufs is a DEVICE array of
 * the world's buffer pointers (this rank's own at [rank]). Every rank calls it
 * once per step, in the same order; a rank that does not arrive within
 * timeout_us makes the others record TQ_DEVICE_ERR_PEER_TIMEOUT in the device
 * error word (tq_device_error) and return with NaN in the outputs they could
 * not merge. Such an exchange is marked failed in its own buffer and stays
 * failed (later merges return NaN and record the timeout again, its step
 * counter no longer moves): close it and allocate a new one. No counterpart
 * in the reference (it is single-device). */
#define TQ_IPC_HANDLE_BYTES 64
#define TQ_DEVICE_ERR_BARRIER_TIMEOUT 1u
#define TQ_DEVICE_ERR_PEER_TIMEOUT 2u
TQ_API size_t tq_peer_buffer_bytes(int world, int batch, int num_heads, int head_dim);
TQ_API int tq_peer_buffer_alloc(size_t bytes, void** buf);
TQ_API int tq_peer_buffer_free(void* buf);
TQ_API int tq_ipc_handle(void* buf, void* handle);
TQ_API int tq_ipc_open(const void* handle, void** peer_buf);
TQ_API int tq_ipc_close(void* peer_buf);
TQ_API int tq_peer_merge(const float* part, void* const* peer_bufs, int world, int rank,
                         int batch, int num_heads, int head_dim, void* out, tq_dtype out_dtype,
                         int timeout_us, void* stream);

/* The same exchange with the push moved into the decode kernel: the CTA that
 * finishes a (sequence, KV head) slice of the partial state stores it straight
 * into slot [step parity][rank] of every rank's exchange buffer as
 * {fp32 value, step} pairs, one store per pair (step = this rank's step
 * counter + 1), so the state crosses NVLink while the rest is still being
 * computed and no fence or flag is needed: the merge takes a value once its
 * pair carries the step. tq_sdpa_int4_partial_publish takes the arguments of
 * tq_sdpa_int4_partial with (peer_bufs, world, rank) in place of part_out, and
 * optionally the new token's K/V rows (k_new, v_new: (B, Hkv, D) in new_dtype,
 * NULL for none), quantized into slot n_local - 1 of this shard in the same
 * launch, as tq_sdpa_int4_append does (the rank holding the sequence's end); the
 * buffers must come from tq_peer_buffer_bytes with the same world, batch,
 * num_heads and head_dim. It runs on the tensor-core decode kernel only
 * (head_dim 128 or 256; else TQ_ERR_UNSUPPORTED). tq_peer_merge_published,
 * called next on the same stream, may start before the decode kernel ends,
 * waits for the pairs of the step from every rank, merges and advances the
 * step counter; its timeout, NaN and failed-exchange rules are tq_peer_merge's.
 * Use one exchange either with tq_peer_merge or with this pair, not both. No
 * counterpart in the reference (it is single-device). */
TQ_API int tq_sdpa_int4_partial_publish(const void* queries, tq_dtype q_dtype,
                                        const uint32_t* k_quant, const void* k_scales,
                                        const void* k_biases, const uint32_t* v_quant,
                                        const void* v_scales, const void* v_biases,
                                        tq_dtype sb_dtype, int gqa_factor, float scale,
                                        int sliding_window, int batch, int num_kv_heads,
                                        int head_dim, int n_local, int capacity, int token_offset,
                                        int n_total, const void* k_new, const void* v_new,
                                        tq_dtype new_dtype, void* const* peer_bufs, int world,
                                        int rank, void* workspace, size_t workspace_bytes,
                                        void* stream);
TQ_API int tq_peer_merge_published(void* const* peer_bufs, int world, int rank, int batch,
                                   int num_heads, int head_dim, void* out, tq_dtype out_dtype,
                                   int timeout_us, void* stream);
/* Head split over the same exchange: every rank decodes its own num_heads
 * query heads over the whole sequence and publishes their state with
 * tq_sdpa_int4_partial_publish (token_offset 0, n_total = n_local);
 * tq_peer_gather_published then writes each rank's heads, normalised, into
 * the full output (batch, world * num_heads, head_dim): rank k's heads at
 * k * num_heads.. -- a gather, not a merge. Same waits, timeout, NaN and
 * failed-exchange rules as tq_peer_merge; use one exchange for one of the
 * three forms. No counterpart in the reference (it is single-device). */
TQ_API int tq_peer_gather_published(void* const* peer_bufs, int world, int rank, int batch,
                                    int num_heads, int head_dim, void* out, tq_dtype out_dtype,
                                    int timeout_us, void* stream);

/* Log-sum-exp merge of n_parts partial states (e.g. one per GPU after an
 * all-gather). parts: n_parts blocks of (H*(D+2)) floats per batch entry,
 * laid out [part][batch][H*(D+2)]; out: (B, H, D) in out_dtype.
 * out = sum_p e^(m_p - M) o_p / sum_p e^(m_p - M) l_p, M = max_p m_p; a head
 * whose total l is 0 gets 0 (lib/turboquant.metal:838-888 merges the same
 * state across simdgroups). */
TQ_API int tq_lse_merge(const float* parts, int n_parts, int batch, int num_heads, int head_dim,
                 void* out, tq_dtype out_dtype, void* stream);

/* Same as tq_sdpa_int4, but with no workspace argument and no allocation of
 * any kind: for callers that cannot call cudaMalloc (for example code running
 * inside a host callback or a custom allocator, or a process whose device
 * memory is fully reserved up front), the split-KV scratch comes from a
 * 2 MiB array built into the library, which every GPU that loads the library
 * keeps until the process exits. Sizes whose scratch does not fit are
 * rejected with TQ_ERR_WORKSPACE.
 * The first call on each device looks up the array's device address
 * (cudaGetSymbolAddress); make that first call outside any stream capture.
 * With lazy module loading (the CUDA 12 default) that lookup is also when
 * the driver places the 2 MiB array on the device, so a caller that reserves
 * all remaining device memory up front should make one call whose sizes
 * need scratch (any context longer than one split) before reserving; later
 * calls allocate nothing. Shapes are checked before the scratch is sized: an unsupported
 * head_dim or gqa_factor returns TQ_ERR_UNSUPPORTED.
 * All calls on a device share the array: calls that overlap on the GPU
 * (different streams, or concurrent graphs) race and must be serialised.
 * No counterpart in the reference (its outputs and temporaries come from
 * MLX's allocator). */
TQ_API int tq_sdpa_int4_noalloc(const void* queries, tq_dtype q_dtype, const uint32_t* k_quant,
                                const void* k_scales, const void* k_biases,
                                const uint32_t* v_quant, const void* v_scales,
                                const void* v_biases, tq_dtype sb_dtype, int gqa_factor,
                                float scale, int sliding_window, int batch, int num_kv_heads,
                                int head_dim, int n_tokens, int capacity,
                                const int32_t* seq_lens, void* out, tq_dtype out_dtype,
                                void* stream);

/* ---- many query rows per KV head on the tensor cores (tcgen05 + TMEM) -------
 * n_q queries (n_q, H, D) against one int4 cache (Hkv, capacity, D/8) holding
 * n_tokens tokens: the batched decode of many sequences against a shared cache
 * (causal = 0: every query sees all n_tokens, the sliding window counts back
 * from the last token) and the prefill chunk (causal = 1: query i sits at
 * position pos0 + i and sees tokens t <= pos0 + i, and pos0 + i - t < window
 * when sliding_window > 0). The reference runs both through MLX dequantize +
 * fast::sdpa with a CPU-built mask (engine/gemma4_multilayer.cpp:307-308,
 * 347-367,441-464). head_dim 128; queries are used in fp16 (bf16 and fp16
 * inputs exactly); out (n_q, H, D) in out_dtype. The workspace
 * (tq_sdpa_int4_multi_workspace_size, zero-filled once) may be NULL when
 * that size is 0. */
TQ_API size_t tq_sdpa_int4_multi_workspace_size(int n_q, int num_heads, int num_kv_heads,
                                                int head_dim, int n_tokens);
TQ_API int tq_sdpa_int4_multi(const void* queries, tq_dtype q_dtype, const uint32_t* k_quant,
                              const void* k_scales, const void* k_biases, const uint32_t* v_quant,
                              const void* v_scales, const void* v_biases, tq_dtype sb_dtype,
                              int gqa_factor, float scale, int sliding_window, int num_kv_heads,
                              int head_dim, int n_q, int n_tokens, int capacity, int causal,
                              int pos0, void* out, tq_dtype out_dtype, void* workspace,
                              size_t workspace_bytes, void* stream);

/* Config 2's two cases by name (same kernel as tq_sdpa_int4_multi):
 *   tq_sdpa_int4_batched: n_seq sequences x 1 query each over one shared
 *     cache of n_tokens tokens (every query at the last position);
 *   tq_sdpa_int4_prefill: causal chunk of n_q queries at positions
 *     pos0 .. pos0 + n_q - 1 whose K/V are already in the cache (slots up to
 *     pos0 + n_q - 1); query i sees tokens t <= pos0 + i (and the window).
 * Workspace: tq_sdpa_int4_multi_workspace_size(n, ..., n_tokens). */
TQ_API int tq_sdpa_int4_batched(const void* queries, tq_dtype q_dtype, const uint32_t* k_quant,
                                const void* k_scales, const void* k_biases,
                                const uint32_t* v_quant, const void* v_scales,
                                const void* v_biases, tq_dtype sb_dtype, int gqa_factor,
                                float scale, int sliding_window, int num_kv_heads, int head_dim,
                                int n_seq, int n_tokens, int capacity, void* out,
                                tq_dtype out_dtype, void* workspace, size_t workspace_bytes,
                                void* stream);
TQ_API int tq_sdpa_int4_prefill(const void* queries, tq_dtype q_dtype, const uint32_t* k_quant,
                                const void* k_scales, const void* k_biases,
                                const uint32_t* v_quant, const void* v_scales,
                                const void* v_biases, tq_dtype sb_dtype, int gqa_factor,
                                float scale, int sliding_window, int num_kv_heads, int head_dim,
                                int n_q, int pos0, int capacity, void* out, tq_dtype out_dtype,
                                void* workspace, size_t workspace_bytes, void* stream);

/* ---- PolarQuant + QJL compressed keys ----------------------------------------
 * Blocks of `block` values (16, 32, 64 or 128; head_dim a multiple of 128) are
 * encoded as in lib/turboquant.metal:8-98 (polar_fused_quantize), generalised
 * from 4 levels to log2(block) levels: per level, each pair (a, b) of the
 * previous level's values gives angle atan2(b, a) (level 1 wrapped to
 * [0, 2pi)) and radius sqrt(a*a + b*b); the angle is replaced by the index of
 * the nearest codebook entry (linear scan, first minimum); the last radius is
 * stored as fp16. Angles are level-major inside a block (level 1's block/2
 * angles first). codebooks: levels x 16 fp32 (level 1 first); cb_sizes: the
 * entries used per level (NULL = 16 each). */

/* y: (rows, head_dim) fp32, already multiplied by the preconditioner if one is
 * used (the reference does y = x P^T before encoding, lib/turboquant.cpp:102).
 * Outputs (angles or packed may be NULL, not both):
 *   angles uint8 (rows, head_dim/block, block-1), one byte per angle index;
 *   packed uint8 (rows, head_dim/block, block/2): 4-bit indices, low nibble
 *          first (the last nibble of a block is 0);
 *   radii  fp16 (rows, head_dim/block).
 * Replaces polar_quantize / polar_quantize_packed (lib/turboquant.h:52-59,80-86). */
TQ_API int tq_polar_encode(const float* y, int64_t rows, int head_dim, int block,
                           const float* codebooks, const int* cb_sizes, uint8_t* angles,
                           uint8_t* packed, void* radii, void* stream);

/* Inverse (lib/turboquant.metal:100-164): y (rows, head_dim) fp32 from exactly
 * one of angles / packed plus radii. Replaces polar_dequantize_fast and
 * polar_dequantize_packed_fast (lib/turboquant.h:96-106,144-151); multiply by
 * the preconditioner afterwards for polar_dequantize (lib/turboquant.cpp:122). */
TQ_API int tq_polar_decode(const uint8_t* angles, const uint8_t* packed, const void* radii,
                           int64_t rows, int head_dim, int block, const float* codebooks,
                           float* y, void* stream);

/* QJL residual sketch (arXiv 2406.03482; the reference has no implementation):
 * r = y - y_hat; signs uint32 (rows, m/32), bit i = ((S r)_i >= 0); rnorm fp16
 * (rows) = |r|. S: (m, head_dim) fp32, m a multiple of 32 in [32, 256]. */
TQ_API int tq_qjl_encode(const float* y, const float* y_hat, int64_t rows, int head_dim,
                         const float* S, int m, uint32_t* signs, void* rnorm, void* stream);

/* Scores of single queries against compressed keys (replaces compressed_score,
 * lib/turboquant.h:154-162, lib/turboquant.metal:424-499, with GQA):
 *   scores[h][n] = scale * ( <q_h, decode(key n of KV head h/G)>
 *                            + sqrt(pi/2)/m * rnorm * <S q_h, sign bits> )
 * queries (H, head_dim) in q_dtype (already preconditioned); packed/radii as
 * from tq_polar_encode for (Hkv, n_keys) key rows; signs/rnorm/S may be NULL
 * (no QJL term). scores: (H, n_keys) fp32. */
TQ_API int tq_compressed_score(const void* queries, tq_dtype q_dtype, const uint8_t* packed,
                               const void* radii, const uint32_t* signs, const void* rnorm,
                               const float* S, int m, int num_heads, int num_kv_heads,
                               int head_dim, int n_keys, int block, const float* codebooks,
                               float scale, float* scores, void* stream);

/* Workspace bytes for tq_compressed_sdpa (zero-filled once before first use,
 * tq_workspace_init; kernels leave it reusable). */
TQ_API size_t tq_compressed_sdpa_workspace_size(int num_heads, int num_kv_heads, int head_dim,
                                                int n_keys);

/* Compressed-key attention (replaces compressed_sdpa, lib/turboquant.h:129-142,
 * lib/turboquant.metal:166-224): softmax over the scores above, then . V with V
 * in the int4 cache layout (v_quant (Hkv, n_keys, D/8), scales/biases
 * (Hkv, n_keys, D/64) in sb_dtype). out (H, head_dim) in out_dtype; an empty
 * context gives 0. */
TQ_API int tq_compressed_sdpa(const void* queries, tq_dtype q_dtype, const uint8_t* packed,
                              const void* radii, const uint32_t* signs, const void* rnorm,
                              const float* S, int m, int num_heads, int num_kv_heads,
                              int head_dim, int n_keys, int block, const float* codebooks,
                              float scale, const uint32_t* v_quant, const void* v_scales,
                              const void* v_biases, tq_dtype sb_dtype, void* out,
                              tq_dtype out_dtype, void* workspace, size_t workspace_bytes,
                              void* stream);

/* tq_compressed_sdpa with dense values (Hkv, n_keys, head_dim) in v_dtype, as
 * the reference's compressed_sdpa takes fp32 values (lib/turboquant.h:129-142,
 * lib/turboquant.metal:166-224; the reference normalises by sum + 1e-8, this
 * by the exact sum). */
TQ_API int tq_compressed_sdpa_dense_v(const void* queries, tq_dtype q_dtype, const uint8_t* packed,
                                      const void* radii, const uint32_t* signs, const void* rnorm,
                                      const float* S, int m, int num_heads, int num_kv_heads,
                                      int head_dim, int n_keys, int block, const float* codebooks,
                                      float scale, const void* values, tq_dtype v_dtype, void* out,
                                      tq_dtype out_dtype, void* workspace, size_t workspace_bytes,
                                      void* stream);

/* The reference's packed format for 16-value blocks (polar_quantize_packed,
 * lib/turboquant.h:75-92, lib/turboquant.metal:501-600): from/to the
 * level-major angle bytes of tq_polar_encode (15 per block). packed_l1 holds
 * level 1's 8 4-bit indices per block (low nibble first); packed_l2..l4 hold
 * levels 2..4 as 2-bit fields (4, 2, 1 per byte), so their indices must be < 4. */
TQ_API int tq_polar_pack_ref(const uint8_t* angles, int64_t n_blocks, uint32_t* packed_l1,
                             uint8_t* packed_l2, uint8_t* packed_l3, uint8_t* packed_l4,
                             void* stream);
TQ_API int tq_polar_unpack_ref(const uint32_t* packed_l1, const uint8_t* packed_l2,
                               const uint8_t* packed_l3, const uint8_t* packed_l4, int64_t n_blocks,
                               uint8_t* angles, void* stream);

/* Level-major angle bytes (n_blocks, block-1) -> 4-bit packed (n_blocks, block/2),
 * the format the compressed-key attention reads. */
TQ_API int tq_polar_pack4(const uint8_t* angles, int64_t n_blocks, int block, uint8_t* packed,
                          void* stream);

/* Preconditioner (lib/turboquant.cpp:102,122): y = x P^T (transpose_p = 0, the
 * encode side) or y = x P (transpose_p = 1, the decode side); x (rows, head_dim)
 * in x_dtype, P (head_dim, head_dim) fp32, y fp32. */
TQ_API int tq_precondition(const void* x, tq_dtype x_dtype, int64_t rows, int head_dim,
                           const float* P, int transpose_p, float* y, void* stream);

/* ---- one decode step from host memory -------------------------------------
 * The per-token call of a decoding loop with host buffers on both sides, as
 * the reference's engine makes it against unified memory
 * (engine/gemma4_multilayer.cpp:222-236: quantize the new K/V row, append it,
 * sdpa_int4 over the cache, read the output). A step object binds one layer's
 * cache (B, Hkv, capacity, ...) and owns mapped pinned staging, a device copy
 * of the inputs, a workspace, a stream and a CUDA graph of two kernels:
 *   gather [queries | k_new | v_new | n_tokens | slots] from the mapped staging
 *   -> tq_sdpa_int4_append (programmatic dependent launch) writing the output
 *      into the mapped output staging,
 * captured on the first run and again whenever the decode plan for the
 * longest sequence changes (about every splits x 64 tokens). Unlike the rest
 * of this ABI it allocates (at create, and the workspace on a re-plan).
 *
 * tq_decode_step_run: n_tokens[b] (host, batch entries) counts sequence b's
 * tokens including the new one (1 <= n <= capacity); the new row goes to slot
 * n - 1. queries (B, H, D) in q_dtype, k_new/v_new (B, Hkv, D) in new_dtype and
 * out (B, H, D) in out_dtype are HOST pointers; each may be the staging buffer
 * tq_decode_step_buffers returns (no host copy then) and out may be NULL (the
 * result stays in the staging buffer). The call returns once the output is on
 * the host. Not thread-safe per object; objects on one device may run from
 * different threads. tq_decode_step_destroy releases everything (NULL: no-op).
 * tq_decode_step_run_at takes the slot of each new row (host, batch entries,
 * 0 <= slots[b] < n_tokens[b]): a ring cache of a sliding layer (create with
 * sliding_window 0 and capacity = the window) passes n = min(t + 1, W) and
 * slot = t mod W for its t-th token. */
typedef struct tq_decode_step tq_decode_step;
TQ_API int tq_decode_step_create(tq_dtype q_dtype, tq_dtype new_dtype, uint32_t* k_quant,
                                 void* k_scales, void* k_biases, uint32_t* v_quant, void* v_scales,
                                 void* v_biases, tq_dtype sb_dtype, int gqa_factor, float scale,
                                 int sliding_window, int batch, int num_kv_heads, int head_dim,
                                 int capacity, tq_dtype out_dtype, tq_decode_step** step);
TQ_API int tq_decode_step_buffers(tq_decode_step* step, void** queries, void** k_new,
                                  void** v_new, void** out);
TQ_API int tq_decode_step_run(tq_decode_step* step, const void* queries, const void* k_new,
                              const void* v_new, const int32_t* n_tokens, void* out);
TQ_API int tq_decode_step_run_at(tq_decode_step* step, const void* queries, const void* k_new,
                                 const void* v_new, const int32_t* n_tokens,
                                 const int32_t* slots, void* out);
TQ_API int tq_decode_step_destroy(tq_decode_step* step);

/* ---- measurement ------------------------------------------------------------
 * Read-only HBM stream over [src, src + bytes) by `ctas` CTAs, each taking one
 * contiguous range: mode 0 with 1-D bulk copies into a shared-memory ring (the
 * decode kernels' load path), mode 1 with 16-byte non-caching loads. The XOR of
 * the data is XOR-accumulated into sink[cta] (ctas words). The practical
 * ceiling the decode kernels' GB/s are compared with (a copy's figure counts a
 * write per read). No counterpart in the reference. */
TQ_API int tq_read_probe(const void* src, size_t bytes, int ctas, int mode, uint32_t* sink,
                         void* stream);

/* Failure-path self-test: one warp waits on a shared-memory barrier that
 * never completes, with the bounded wait every pipeline here uses, given up
 * after timeout_us (1 .. 10^7). Expected outcome: TQ_DEVICE_ERR_BARRIER_TIMEOUT
 * in the device error word, *gave_up (device uint32, caller-zeroed)
 * incremented by each of the 32 threads, and a usable context afterwards.
 * (The pipelines' own bound is about 2 s of SM clock.) No counterpart in the
 * reference. */
TQ_API int tq_wait_selftest(int timeout_us, uint32_t* gave_up, void* stream);

/* Read and clear the device error word that kernels set when a bounded wait
 * gives up (0 = no error). Synchronises `stream`. */
TQ_API int tq_device_error(void* stream, uint32_t* code);

#ifdef __cplusplus
}
#endif

#endif /* TURBOQUANT_C_H */
