/*
 * turboquant.hpp -- C++ host API of libturboquant_b200.so, the B200 backend of
 * gemma4metal's int4 KV-cache attention path.
 *
 * It keeps the names, argument order, defaults and shape conventions of the
 * reference's lib/turboquant.h (namespace turboquant, lib/turboquant.h:52-209)
 * and of the MLX calls the engine makes around it (quantize / dequantize,
 * engine/gemma4_multilayer.cpp:228-229,307-308), so engine code and
 * tests/test_sdpa_int4.cpp switch backends by swapping the include:
 *
 *   mlx::core::array     -> turboquant::array   (device tensor, ref-counted)
 *   StreamOrDevice s = {} -> cudaStream_t s = nullptr
 *
 * Differences from the reference, on purpose:
 *   - Work is enqueued on `s` immediately (CUDA streams), not built as a lazy
 *     graph; array::to_host() synchronises the stream.
 *   - Errors throw std::runtime_error, as the reference's primitives do
 *     (lib/turboquant.cpp:363-365), with the library's message.
 *   - Outputs are allocated stream-ordered (cudaMallocAsync) on `s`, as the
 *     reference allocates outputs inside eval_gpu (lib/turboquant.cpp:372).
 *     The allocation-free path is the C ABI (turboquant_c.h) and KVCache.
 *   - Attention accepts fp32, fp16 or bf16 queries and fp16 or fp32
 *     scales/biases (the reference hard-codes fp32, lib/turboquant.metal:725-732)
 *     and head_dim 128/256/512 (the reference: 256/512, lib/turboquant.cpp:378).
 */
#ifndef TURBOQUANT_HPP
#define TURBOQUANT_HPP

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <map>
#include <memory>
#include <string>
#include <vector>

#if defined(__GNUC__)
#define TQ_CXX_API __attribute__((visibility("default")))
#else
#define TQ_CXX_API
#endif

struct tq_decode_step;  // turboquant_c.h

namespace turboquant {

enum class Dtype : int { float32 = 0, float16 = 1, bfloat16 = 2, uint32 = 3, int32 = 4, uint8 = 5 };

TQ_CXX_API size_t itemsize(Dtype d);

// Dense, row-major device tensor (the subset of mlx::core::array the path
// needs). Copies share storage; reshape() returns a view.
class TQ_CXX_API array {
 public:
  array() = default;
  // Uninitialised device memory on the current device, allocated on stream s.
  array(std::vector<int> shape, Dtype dtype, cudaStream_t s = nullptr);

  static array zeros(std::vector<int> shape, Dtype dtype, cudaStream_t s = nullptr);
  // Copy `size() * itemsize` bytes from host memory (synchronous for the host buffer).
  static array from_host(const void* src, std::vector<int> shape, Dtype dtype,
                         cudaStream_t s = nullptr);
  // Copy to host memory; synchronises s.
  void to_host(void* dst, cudaStream_t s = nullptr) const;
  template <typename T>
  std::vector<T> to_vector(cudaStream_t s = nullptr) const {
    std::vector<T> v(nbytes() / sizeof(T));
    to_host(v.data(), s);
    return v;
  }

  const std::vector<int>& shape() const { return shape_; }
  int shape(int dim) const { return shape_.at(dim < 0 ? dim + ndim() : dim); }
  int ndim() const { return static_cast<int>(shape_.size()); }
  size_t size() const;
  size_t nbytes() const { return size() * itemsize(dtype_); }
  Dtype dtype() const { return dtype_; }
  void* data() { return ptr_; }
  const void* data() const { return ptr_; }
  int device() const { return device_; }
  bool valid() const { return ptr_ != nullptr || size() == 0; }

  // Same storage, new shape (element count must match).
  array reshape(std::vector<int> shape) const;

 private:
  std::shared_ptr<void> buf_;
  void* ptr_ = nullptr;
  std::vector<int> shape_;
  Dtype dtype_ = Dtype::float32;
  int device_ = 0;
};

// ---- MLX-compatible quantizer (engine/gemma4_multilayer.cpp:228-229) -------
// Affine group-64 4-bit: returns {codes uint32 (..., D/8), scales (..., D/64),
// biases (..., D/64)}; scales/biases fp16 unless scales_dtype says otherwise.
TQ_CXX_API std::vector<array> quantize(const array& w, int group_size = 64, int bits = 4,
                            cudaStream_t s = nullptr, Dtype scales_dtype = Dtype::float16);
// value = scale * code + bias (engine/gemma4_multilayer.cpp:307-308); float32 out.
TQ_CXX_API array dequantize(const array& w, const array& scales, const array& biases, int group_size = 64,
                 int bits = 4, cudaStream_t s = nullptr, Dtype out_dtype = Dtype::float32);

// ---- fused int4 decode attention (lib/turboquant.h:196-207) ----------------
// queries (H, D); k_quant/v_quant (Hkv, N, D/8) uint32; scales/biases
// (Hkv, N, D/64). Returns (H, D) in the query dtype. Query head h reads KV
// head h / gqa_factor; sliding_window > 0 masks tokens t with
// (N-1-t) >= sliding_window. The kernels need every KV head's rows 16-byte
// aligned, i.e. a token axis that is a multiple of 4; a reference-shaped
// cache with any other N (the reference's test uses N = 10) is served through
// a copy into a capacity rounded up to 4 -- O(N) per call, as the engine's
// concatenate is. Engine code avoids it with KVCache, RingKVCache (any
// window) or sdpa_int4_tokens.
TQ_CXX_API array sdpa_int4(const array& queries, const array& k_quant, const array& k_scales,
                const array& k_biases, const array& v_quant, const array& v_scales,
                const array& v_biases, int gqa_factor, float scale = 1.0f,
                int sliding_window = 0, cudaStream_t s = nullptr);
// The same over the first n_tokens rows of cache arrays whose token axis is a
// capacity (a multiple of 4, >= n_tokens): any n_tokens, no copy.
TQ_CXX_API array sdpa_int4_tokens(const array& queries, const array& k_quant,
                                  const array& k_scales, const array& k_biases,
                                  const array& v_quant, const array& v_scales,
                                  const array& v_biases, int n_tokens, int gqa_factor,
                                  float scale = 1.0f, int sliding_window = 0,
                                  cudaStream_t s = nullptr);

// No-op (lib/turboquant.h:209): kernels are linked into the library.
TQ_CXX_API void set_metallib_path(const std::string& path);

// ---- preallocated cache: quantize-on-append + decode without copies ---------
// Replaces the engine's per-token quantize + concatenate + trim of the whole
// cache (engine/gemma4_multilayer.cpp:228-249) with in-place appends.
class TQ_CXX_API KVCache {
 public:
  KVCache(int batch, int num_kv_heads, int head_dim, int capacity,
          Dtype scales_dtype = Dtype::float16, cudaStream_t s = nullptr);
  // k_new, v_new: (B, Hkv, n_new, D) (or (Hkv, n_new, D) when B = 1), fp32/fp16/bf16,
  // written at token slots [length, length + n_new).
  void append(const array& k_new, const array& v_new, cudaStream_t s = nullptr);
  // Decode attention over the cached tokens: queries (B, H, D) or (H, D).
  array sdpa(const array& queries, int gqa_factor, float scale = 1.0f, int sliding_window = 0,
             cudaStream_t s = nullptr);
  // One decode step: append the step's K/V row (B, Hkv, D) or (B, Hkv, 1, D)
  // and attend over the cache including it -- one launch with the tensor-core
  // decode kernel; same result as append() followed by sdpa().
  array decode_step(const array& queries, const array& k_new, const array& v_new, int gqa_factor,
                    float scale = 1.0f, int sliding_window = 0, cudaStream_t s = nullptr);
  // Prefill chunk (batch 1): append n new tokens' K/V (Hkv, n, D), then causal
  // attention of their queries (n, H, D) -- query i at position length + i --
  // on the tensor cores (tcgen05). Returns (n, H, D) in out_dtype.
  array prefill_chunk(const array& queries, const array& k_chunk, const array& v_chunk,
                      int gqa_factor, float scale = 1.0f, int sliding_window = 0,
                      Dtype out_dtype = Dtype::bfloat16, cudaStream_t s = nullptr);
  // Batched decode over this (batch 1) cache shared by n sequences: queries
  // (n, H, D), each at the last position; tensor cores. Returns (n, H, D).
  array sdpa_multi(const array& queries, int gqa_factor, float scale = 1.0f,
                   int sliding_window = 0, Dtype out_dtype = Dtype::bfloat16,
                   cudaStream_t s = nullptr);
  int length() const { return length_; }
  int capacity() const { return capacity_; }
  void reset() { length_ = 0; }
  // Valid token count after the arrays were filled directly (e.g. by
  // load_kv_cache); 0 <= n <= capacity.
  void set_length(int n);
  array k_quant, k_scales, k_biases, v_quant, v_scales, v_biases;

 private:
  friend class HostDecodeStep;
  int batch_, num_kv_heads_, head_dim_, capacity_, length_ = 0;
};

class RingKVCache;

// ---- one decode step from host memory (tq_decode_step_*) ---------------------
// The engine's per-token call (engine/gemma4_multilayer.cpp:222-236) with the
// query, the new K/V row and the output in host memory: one CUDA graph launch
// (gather kernel + fused append/decode kernel writing the output into mapped
// host memory) and one synchronisation per run(). Binds `cache` (which must
// outlive the step) and advances its length.
class TQ_CXX_API HostDecodeStep {
 public:
  HostDecodeStep(KVCache& cache, int num_heads, float scale = 1.0f, int sliding_window = 0,
                 Dtype q_dtype = Dtype::float16, Dtype new_dtype = Dtype::float16,
                 Dtype out_dtype = Dtype::float16);
  // A sliding layer's ring: run() writes the next token at slot total % window
  // and attends over the window, advancing the ring's position.
  HostDecodeStep(RingKVCache& ring, int num_heads, float scale = 1.0f,
                 Dtype q_dtype = Dtype::float16, Dtype new_dtype = Dtype::float16,
                 Dtype out_dtype = Dtype::float16);
  ~HostDecodeStep();
  HostDecodeStep(const HostDecodeStep&) = delete;
  HostDecodeStep& operator=(const HostDecodeStep&) = delete;
  // queries (B, H, D), k_new/v_new (B, Hkv, D), out (B, H, D): host pointers
  // (or the staging buffers below; out may be nullptr). n_tokens: per-sequence
  // token counts including the new token (nullptr: cache length + 1 for all).
  void run(const void* queries, const void* k_new, const void* v_new, void* out,
           const int32_t* n_tokens = nullptr);
  // Explicit slot of each sequence's new row (0 <= slots[b] < n_tokens[b]).
  void run_at(const void* queries, const void* k_new, const void* v_new, void* out,
              const int32_t* n_tokens, const int32_t* slots);
  // Pinned staging buffers: inputs written here need no host copy in run().
  void* queries() const;
  void* k_new() const;
  void* v_new() const;
  void* out() const;

 private:
  KVCache* cache_;
  RingKVCache* ring_ = nullptr;
  tq_decode_step* step_ = nullptr;
  std::vector<int32_t> n_;
};

// ---- sliding-window layer as a ring of `window` slots (batch 1) ---------------
// Any window (the engine's 950-token cap included): the arrays' token axis is
// the window rounded up to 4, slots past the window stay unused.
// Token t lives in slot t % window, so the cache holds exactly the last
// `window` tokens -- the set the window rule keeps -- with no copy (the
// engine concatenates and trims the front, engine/gemma4_multilayer.cpp:228-249).
// Attention is order-independent: decode runs over the filled slots unmasked.
class TQ_CXX_API RingKVCache {
 public:
  RingKVCache(int num_kv_heads, int head_dim, int window, Dtype scales_dtype = Dtype::float16,
              cudaStream_t s = nullptr);
  // k_new, v_new: (1, Hkv, n, D) or (Hkv, n, D); wraps; only the last `window` survive.
  void append(const array& k_new, const array& v_new, cudaStream_t s = nullptr);
  array decode(const array& queries, int gqa_factor, float scale = 1.0f, cudaStream_t s = nullptr);
  // One launch: the step's K/V (1, Hkv, D) go to slot total % window, then attention.
  array decode_step(const array& queries, const array& k_new, const array& v_new, int gqa_factor,
                    float scale = 1.0f, cudaStream_t s = nullptr);
  int n_valid() const { return total_ < window_ ? static_cast<int>(total_) : window_; }
  long long total() const { return total_; }
  int window() const { return window_; }
  // Tokens seen so far after the slots were filled directly (slot t % window
  // holds token t); sets the cache's length to n_valid().
  void set_total(long long total);
  KVCache cache;

 private:
  friend class HostDecodeStep;
  int window_;
  long long total_ = 0;
};

// ---- sequence split across GPUs ----------------------------------------------
// Partial softmax state of a contiguous token shard [token_offset, +n_local) of a
// sequence of n_total tokens: (B, H*(D+2)) fp32 = o (H, D) unnormalised, then
// (m, l) per head (natural-log max, sum of exponentials).
TQ_CXX_API array sdpa_int4_partial(const array& queries, const KVCache& shard, int n_local, int token_offset,
                        int n_total, int gqa_factor, float scale = 1.0f, int sliding_window = 0,
                        cudaStream_t s = nullptr);
// Log-sum-exp merge of P stacked partial states (P, B, H*(D+2)) -> (B, H, D).
TQ_CXX_API array lse_merge(const array& parts, int num_heads, int head_dim, Dtype out_dtype = Dtype::float32,
                cudaStream_t s = nullptr);

// ---- PolarQuant compressed keys (lib/turboquant.h:52-165) --------------------
// Same names, arguments and shapes as the reference: 16-value blocks and four
// level codebooks cb_l1..cb_l4 (fp32 device arrays of <= 16 entries; the packed
// format's levels 2-4 hold 2-bit indices, so those codebooks need <= 4
// entries). Indices come back as the reference's per-level uint8 arrays
// i1 (N*nb*8), i2 (N*nb*4), i3 (N*nb*2), i4 (N*nb); radii fp16 (N*nb).
// Codebooks are read on the host (the stream is synchronised for it).
TQ_CXX_API std::vector<array> polar_quantize(const array& vectors, const array& precondition,
                                             const array& cb_l1, const array& cb_l2,
                                             const array& cb_l3, const array& cb_l4,
                                             int block_size = 16, cudaStream_t s = nullptr);
// (N, D) fp32 = decode(...) . precondition, D = precondition.shape(0).
TQ_CXX_API array polar_dequantize(const array& indices_l1, const array& indices_l2,
                                  const array& indices_l3, const array& indices_l4,
                                  const array& radii, const array& precondition,
                                  const array& cb_l1, const array& cb_l2, const array& cb_l3,
                                  const array& cb_l4, int block_size = 16, cudaStream_t s = nullptr);
// {packed_l1 uint32 (N_blocks), packed_l2/l3/l4 uint8 (N_blocks), radii fp16 (N_blocks)}
TQ_CXX_API std::vector<array> polar_quantize_packed(const array& vectors, const array& precondition,
                                                    const array& cb_l1, const array& cb_l2,
                                                    const array& cb_l3, const array& cb_l4,
                                                    int block_size = 16, cudaStream_t s = nullptr);
TQ_CXX_API array polar_dequantize_packed(const array& packed_l1, const array& packed_l2,
                                         const array& packed_l3, const array& packed_l4,
                                         const array& radii, const array& cb_l1, const array& cb_l2,
                                         const array& cb_l3, const array& cb_l4, int D,
                                         int block_size = 16, cudaStream_t s = nullptr);
// cs_l*: (entries, 2) fp32 {cos, sin} tables; decoded with the angles
// atan2(sin, cos) of the table entries.
TQ_CXX_API array polar_dequantize_packed_fast(const array& packed_l1, const array& packed_l2,
                                              const array& packed_l3, const array& packed_l4,
                                              const array& radii, const array& cs_l1,
                                              const array& cs_l2, const array& cs_l3,
                                              const array& cs_l4, int D, int block_size = 16,
                                              cudaStream_t s = nullptr);
// queries (Nq, D) preconditioned; query i attends to keys [i*N, (i+1)*N) and
// values (Nq*N, D) fp32 (N = values.shape(0) / Nq). Returns (Nq, D) fp32.
TQ_CXX_API array compressed_sdpa(const array& queries, const array& indices_l1,
                                 const array& indices_l2, const array& indices_l3,
                                 const array& indices_l4, const array& radii, const array& cb_l1,
                                 const array& cb_l2, const array& cb_l3, const array& cb_l4,
                                 const array& values, int block_size = 16, float scale = 0.0884f,
                                 cudaStream_t s = nullptr);
// Inverse polar only (no preconditioner): (N_blocks * block / D, D) fp32.
TQ_CXX_API array polar_dequantize_fast(const array& indices_l1, const array& indices_l2,
                                       const array& indices_l3, const array& indices_l4,
                                       const array& radii, const array& cb_l1, const array& cb_l2,
                                       const array& cb_l3, const array& cb_l4, int D,
                                       int block_size = 16, cudaStream_t s = nullptr);
// (Nq, N) fp32 scores of query i against keys [i*N, (i+1)*N).
TQ_CXX_API array compressed_score(const array& queries, const array& indices_l1,
                                  const array& indices_l2, const array& indices_l3,
                                  const array& indices_l4, const array& radii, const array& cb_l1,
                                  const array& cb_l2, const array& cb_l3, const array& cb_l4, int N,
                                  int block_size = 16, float scale = 0.0884f,
                                  cudaStream_t s = nullptr);

// ---- the engine's on-disk int4 KV cache (kv_cache.safetensors) ---------------
// Same file as the engine's save_kv_cache / load_kv_cache
// (engine/gemma4_multilayer.cpp:113-144): one safetensors file holding
// cache_offset (int32 [1]) and, per layer L with a cache, l{L}.kq/ks/kb/vq/vs/vb
// = codes (1, Hkv, T, D/8) uint32 and scales/biases (1, Hkv, T, D/64), T
// tokens oldest first (a sliding layer holds its last `window` tokens).
struct TQ_CXX_API LoadedKVCache {
  int cache_offset = 0;
  std::map<int, std::unique_ptr<KVCache>> caches;     // layers not in `windows`
  std::map<int, std::unique_ptr<RingKVCache>> rings;  // layers in `windows`
};
// Writes the valid tokens of every cache (batch 1), oldest first.
TQ_CXX_API void save_kv_cache(const std::string& path, int cache_offset,
                              const std::map<int, const KVCache*>& caches,
                              const std::map<int, const RingKVCache*>& rings = {},
                              cudaStream_t s = nullptr);
// Layers listed in `windows` (layer -> window) load into a RingKVCache, the
// others into a KVCache with room for max(capacity, T rounded up to 4)
// tokens. fp16 and fp32 scales/biases load as stored; bf16 ones (an engine
// running in bf16) are widened to fp32 exactly. Throws on a malformed file.
TQ_CXX_API LoadedKVCache load_kv_cache(const std::string& path, int capacity = 0,
                                       const std::map<int, int>& windows = {},
                                       cudaStream_t s = nullptr);

}  // namespace turboquant

#endif  // TURBOQUANT_HPP
