// extern "C" ABI of libturboquant_b200.so (declared in include/turboquant_c.h):
// host-side validation, planning and dispatch onto the caller's CUDA stream.
#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <string>
#include <unordered_map>

#include "../../include/turboquant_c.h"
#include "tq_common.cuh"
#include "tq_internal.h"
#include "peer_layout.cuh"

namespace {

thread_local std::string t_err;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_err = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(TQ_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

bool valid_dtype(int d) { return d == TQ_F32 || d == TQ_F16 || d == TQ_BF16; }

// Device error word: one per device, set by kernels whose bounded waits expire.
__device__ uint32_t g_device_error;

std::mutex g_err_mu;
std::unordered_map<int, uint32_t*> g_err_ptr;

uint32_t* device_error_ptr() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
  std::lock_guard<std::mutex> lock(g_err_mu);
  auto it = g_err_ptr.find(dev);
  if (it != g_err_ptr.end()) return it->second;
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) return nullptr;
  g_err_ptr[dev] = static_cast<uint32_t*>(p);
  return static_cast<uint32_t*>(p);
}

int check_head_dim(int D) {
  if (D != 128 && D != 256 && D != 512)
    return fail(TQ_ERR_UNSUPPORTED, "head_dim %d not supported (128, 256, 512)", D);
  return TQ_OK;
}

struct DecodeCommon {
  const void* q;
  int q_dtype;
  const uint32_t *kq, *vq;
  const void *ks, *kb, *vs, *vb;
  int sb_dtype, gqa, window, B, Hkv, D, n_tokens, capacity;
  float scale;
  // decode step with quantize-on-append of the new token (nullable)
  const void* k_new = nullptr;
  const void* v_new = nullptr;
  int new_dtype = 0;
  int new_slot = -1;
  const int32_t* new_slots = nullptr;  // device, one slot per sequence (overrides new_slot)
  // partial state published into every rank's exchange buffer (nullable)
  void* const* peer_bufs = nullptr;
  int peer_world = 0, peer_rank = 0;
};

int validate_decode(const DecodeCommon& c, const char* fn) {
  if (!c.q || !c.kq || !c.ks || !c.kb || !c.vq || !c.vs || !c.vb)
    return fail(TQ_ERR_INVALID, "%s: null pointer argument", fn);
  if (!valid_dtype(c.q_dtype)) return fail(TQ_ERR_INVALID, "%s: bad q_dtype %d", fn, c.q_dtype);
  if (c.sb_dtype != TQ_F16 && c.sb_dtype != TQ_F32)
    return fail(TQ_ERR_UNSUPPORTED, "%s: scale/bias dtype must be f16 or f32", fn);
  if (int rc = check_head_dim(c.D)) return rc;
  if (c.gqa != 1 && c.gqa != 2 && c.gqa != 4 && c.gqa != 8)
    return fail(TQ_ERR_UNSUPPORTED, "%s: gqa_factor %d not in {1,2,4,8}", fn, c.gqa);
  if (c.B < 1 || c.Hkv < 1) return fail(TQ_ERR_INVALID, "%s: batch/num_kv_heads must be >= 1", fn);
  if (c.n_tokens < 0 || c.capacity < 0 || c.n_tokens > c.capacity)
    return fail(TQ_ERR_INVALID, "%s: need 0 <= n_tokens (%d) <= capacity (%d)", fn, c.n_tokens,
                c.capacity);
  if (c.capacity % 4 != 0) return fail(TQ_ERR_INVALID, "%s: capacity %d not a multiple of 4", fn, c.capacity);
  if (c.window < 0) return fail(TQ_ERR_INVALID, "%s: sliding_window must be >= 0", fn);
  const void* ptrs[] = {c.kq, c.ks, c.kb, c.vq, c.vs, c.vb};
  for (const void* p : ptrs)
    if (!aligned16(p)) return fail(TQ_ERR_INVALID, "%s: cache pointers must be 16-byte aligned", fn);
  if (!aligned16(c.q)) return fail(TQ_ERR_INVALID, "%s: queries must be 16-byte aligned", fn);
  return TQ_OK;
}

int visible_max(int n_tokens, int window) {
  return window > 0 ? (n_tokens < window ? n_tokens : window) : n_tokens;
}

}  // namespace

namespace tq {

bool& pdl_launches() {
  static thread_local bool on = true;
  return on;
}

uint32_t* device_error_word() { return device_error_ptr(); }

void set_last_error(const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_err = buf;
}
}  // namespace tq

extern "C" {

const char* tq_last_error(void) { return t_err.c_str(); }

const char* tq_version(void) { return "turboquant_b200 0.1.0 (sm_100a)"; }

void tq_set_metallib_path(const char* path) { (void)path; }

int tq_quantize(const void* x, tq_dtype x_dtype, int64_t rows, int head_dim, uint32_t* codes,
                void* scales, void* biases, tq_dtype sb_dtype, void* stream) {
  t_err.clear();
  if (rows < 0) return fail(TQ_ERR_INVALID, "tq_quantize: rows < 0");
  if (head_dim <= 0 || head_dim % 64 != 0)
    return fail(TQ_ERR_INVALID, "tq_quantize: head_dim %d must be a positive multiple of 64", head_dim);
  if (!valid_dtype(x_dtype) || !valid_dtype(sb_dtype)) return fail(TQ_ERR_INVALID, "tq_quantize: bad dtype");
  if (rows == 0) return TQ_OK;
  if (!x || !codes || !scales || !biases) return fail(TQ_ERR_INVALID, "tq_quantize: null pointer");
  if (!aligned16(x)) return fail(TQ_ERR_INVALID, "tq_quantize: x must be 16-byte aligned");
  // destination token index == row index: one "sequence" of `rows` tokens
  cudaError_t e = tq::launch_quantize_rows(x, x_dtype, rows, head_dim, rows, 1, 0, 0, 0, nullptr,
                                           codes, scales, biases, sb_dtype,
                                           static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "tq_quantize launch");
  return TQ_OK;
}

int tq_dequantize(const uint32_t* codes, const void* scales, const void* biases,
                  tq_dtype sb_dtype, int64_t rows, int head_dim, void* out, tq_dtype out_dtype,
                  void* stream) {
  t_err.clear();
  if (rows < 0) return fail(TQ_ERR_INVALID, "tq_dequantize: rows < 0");
  if (head_dim <= 0 || head_dim % 64 != 0)
    return fail(TQ_ERR_INVALID, "tq_dequantize: head_dim %d must be a positive multiple of 64", head_dim);
  if (!valid_dtype(out_dtype) || !valid_dtype(sb_dtype)) return fail(TQ_ERR_INVALID, "tq_dequantize: bad dtype");
  if (rows == 0) return TQ_OK;
  if (!codes || !scales || !biases || !out) return fail(TQ_ERR_INVALID, "tq_dequantize: null pointer");
  cudaError_t e = tq::launch_dequantize(codes, scales, biases, sb_dtype, rows, head_dim, out,
                                        out_dtype, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "tq_dequantize launch");
  return TQ_OK;
}

int tq_quantize_append(const void* k_new, const void* v_new, tq_dtype in_dtype, int batch,
                       int num_kv_heads, int head_dim, int n_new, uint32_t* k_quant,
                       void* k_scales, void* k_biases, uint32_t* v_quant, void* v_scales,
                       void* v_biases, tq_dtype sb_dtype, int capacity, int pos,
                       const int32_t* positions, void* stream) {
  t_err.clear();
  if (head_dim <= 0 || head_dim % 64 != 0)
    return fail(TQ_ERR_INVALID, "tq_quantize_append: head_dim %d must be a positive multiple of 64", head_dim);
  if (!valid_dtype(in_dtype) || !valid_dtype(sb_dtype))
    return fail(TQ_ERR_INVALID, "tq_quantize_append: bad dtype");
  if (batch < 1 || num_kv_heads < 1 || n_new < 0)
    return fail(TQ_ERR_INVALID, "tq_quantize_append: bad sizes");
  if (n_new == 0) return TQ_OK;
  if (!k_new || !v_new || !k_quant || !k_scales || !k_biases || !v_quant || !v_scales || !v_biases)
    return fail(TQ_ERR_INVALID, "tq_quantize_append: null pointer");
  if (!aligned16(k_new) || !aligned16(v_new))
    return fail(TQ_ERR_INVALID, "tq_quantize_append: inputs must be 16-byte aligned");
  if (!positions && (pos < 0 || static_cast<long long>(pos) + n_new > capacity))
    return fail(TQ_ERR_INVALID, "tq_quantize_append: slots [%d, %d) exceed capacity %d", pos,
                pos + n_new, capacity);
  const long long rows = static_cast<long long>(batch) * num_kv_heads * n_new;
  const long long bstride = static_cast<long long>(num_kv_heads) * capacity;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = tq::launch_quantize_rows(k_new, in_dtype, rows, head_dim, n_new, num_kv_heads,
                                           capacity, bstride, pos, positions, k_quant, k_scales,
                                           k_biases, sb_dtype, s, v_new, v_quant, v_scales,
                                           v_biases);
  if (e != cudaSuccess) return cuda_fail(e, "tq_quantize_append launch");
  return TQ_OK;
}

size_t tq_sdpa_int4_workspace_size(int batch, int num_heads, int num_kv_heads, int head_dim,
                                   int n_tokens, int sliding_window) {
  if (batch < 1 || num_kv_heads < 1 || num_heads < num_kv_heads || n_tokens < 0) return 0;
  // the planner divides by head_dim: sizes no decode call accepts get 0
  if (head_dim != 128 && head_dim != 256 && head_dim != 512) return 0;
  int dev = 0;
  cudaGetDevice(&dev);
  tq::DecodePlan pl = tq::plan_decode(dev, batch, num_heads, num_kv_heads, head_dim,
                                      visible_max(n_tokens, sliding_window), sliding_window > 0);
  return pl.ws_bytes;
}

int tq_workspace_init(void* workspace, size_t workspace_bytes, void* stream) {
  t_err.clear();
  if (!workspace || workspace_bytes == 0) return TQ_OK;
  cudaError_t e = cudaMemsetAsync(workspace, 0, workspace_bytes, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "tq_workspace_init");
  return TQ_OK;
}

static int decode_common(const DecodeCommon& c, const char* fn, const int32_t* seq_lens,
                         int token_offset, int n_total, int partial, void* out, int out_dtype,
                         float* part_out, void* workspace, size_t workspace_bytes, void* stream) {
  if (int rc = validate_decode(c, fn)) return rc;
  const int H = c.Hkv * c.gqa;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, fn);
  // visible tokens of the largest sequence; a sequence shard sees the part of
  // its tokens that lies inside the window of the whole sequence
  const int vis = !partial       ? visible_max(c.n_tokens, c.window)
                  : c.window > 0 ? std::max(0, c.n_tokens - std::max(0, n_total - c.window -
                                                                          token_offset))
                                 : c.n_tokens;
  tq::DecodePlan pl = tq::plan_decode(dev, c.B, H, c.Hkv, c.D, vis, c.window > 0,
                                      c.q_dtype != TQ_F16);
  if (pl.splits < 0)
    return fail(TQ_ERR_UNSUPPORTED, "%s: batch * kv_heads too large for one launch", fn);
  if (pl.ws_bytes > 0 && (!workspace || workspace_bytes < pl.ws_bytes))
    return fail(TQ_ERR_WORKSPACE, "%s: workspace of %zu bytes needed, %zu given", fn, pl.ws_bytes,
                workspace ? workspace_bytes : static_cast<size_t>(0));
  if (pl.ws_bytes > 0 && !aligned16(workspace))
    return fail(TQ_ERR_INVALID, "%s: workspace must be 16-byte aligned", fn);
  tq::DecodeArgs a{};
  a.q = c.q;
  a.q_dtype = c.q_dtype;
  a.kq = c.kq;
  a.ks = c.ks;
  a.kb = c.kb;
  a.vq = c.vq;
  a.vs = c.vs;
  a.vb = c.vb;
  a.sb_dtype = c.sb_dtype;
  a.seq_lens = seq_lens;
  a.n_tokens = c.n_tokens;
  a.B = c.B;
  a.H = H;
  a.Hkv = c.Hkv;
  a.D = c.D;
  a.G = c.gqa;
  a.capacity = c.capacity;
  a.bstride_tok = static_cast<long long>(c.Hkv) * c.capacity;
  a.scale = c.scale;
  a.window = c.window;
  a.token_offset = token_offset;
  a.n_total = n_total;
  a.partial = partial;
  a.out = out;
  a.out_dtype = out_dtype;
  a.part_out = part_out;
  a.workspace = workspace;
  a.workspace_bytes = workspace_bytes;
  a.err = device_error_ptr();
  if (c.peer_bufs) {
    if (pl.variant != tq::kDecodeMma)
      return fail(TQ_ERR_UNSUPPORTED, "%s: publishing needs the tensor-core decode kernel", fn);
    a.peer_bufs = c.peer_bufs;
    a.peer_world = c.peer_world;
    a.peer_rank = c.peer_rank;
  }
  if (c.k_new) {
    // the mma kernel quantizes the new token in the same launch; the CUDA-core
    // kernel gets it from a quantize-on-append launch just before
    if (pl.variant == tq::kDecodeMma) {
      a.k_new = c.k_new;
      a.v_new = c.v_new;
      a.new_dtype = c.new_dtype;
      a.new_slot = c.new_slot;
      a.new_slots = c.new_slots;
    } else {
      // slot: per-sequence device slots, else the given slot, else n - 1
      // (seq_lens[b] - 1 per sequence)
      const bool at_slot = c.new_slot >= 0;
      const int32_t* positions = c.new_slots ? c.new_slots : at_slot ? nullptr : seq_lens;
      e = tq::launch_quantize_rows(
          c.k_new, c.new_dtype, static_cast<long long>(c.B) * c.Hkv, c.D, 1, c.Hkv, c.capacity,
          a.bstride_tok, at_slot ? c.new_slot : c.n_tokens - 1, positions,
          const_cast<uint32_t*>(c.kq), const_cast<void*>(c.ks), const_cast<void*>(c.kb), c.sb_dtype,
          static_cast<cudaStream_t>(stream), c.v_new, const_cast<uint32_t*>(c.vq),
          const_cast<void*>(c.vs), const_cast<void*>(c.vb), c.new_slots ? 0 : -1);
      if (e != cudaSuccess) return cuda_fail(e, fn);
    }
  }
  tq::launch_detail().clear();
  e = tq::launch_decode(a, pl, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    if (!tq::launch_detail().empty())
      return fail(TQ_ERR_CUDA, "%s: %s (%s)", fn, cudaGetErrorString(e), tq::launch_detail().c_str());
    return cuda_fail(e, fn);
  }
  return TQ_OK;
}

int tq_sdpa_int4(const void* queries, tq_dtype q_dtype, const uint32_t* k_quant,
                 const void* k_scales, const void* k_biases, const uint32_t* v_quant,
                 const void* v_scales, const void* v_biases, tq_dtype sb_dtype, int gqa_factor,
                 float scale, int sliding_window, int batch, int num_kv_heads, int head_dim,
                 int n_tokens, int capacity, const int32_t* seq_lens, void* out,
                 tq_dtype out_dtype, void* workspace, size_t workspace_bytes, void* stream) {
  t_err.clear();
  if (!out) return fail(TQ_ERR_INVALID, "tq_sdpa_int4: null out");
  if (!valid_dtype(out_dtype)) return fail(TQ_ERR_INVALID, "tq_sdpa_int4: bad out_dtype");
  DecodeCommon c{queries, q_dtype, k_quant, v_quant, k_scales, k_biases, v_scales, v_biases,
                 sb_dtype, gqa_factor, sliding_window, batch, num_kv_heads, head_dim, n_tokens,
                 capacity, scale};
  return decode_common(c, "tq_sdpa_int4", seq_lens, 0, 0, 0, out, out_dtype, nullptr, workspace,
                       workspace_bytes, stream);
}

static int append_common(const void* queries, tq_dtype q_dtype, const void* k_new,
                         const void* v_new, tq_dtype new_dtype, uint32_t* k_quant, void* k_scales,
                         void* k_biases, uint32_t* v_quant, void* v_scales, void* v_biases,
                         tq_dtype sb_dtype, int gqa_factor, float scale, int sliding_window,
                         int batch, int num_kv_heads, int head_dim, int n_tokens, int capacity,
                         const int32_t* seq_lens, int slot, const int32_t* slots, void* out,
                         tq_dtype out_dtype, void* workspace, size_t workspace_bytes,
                         void* stream) {
  t_err.clear();
  if (!out) return fail(TQ_ERR_INVALID, "tq_sdpa_int4_append: null out");
  if (!valid_dtype(out_dtype)) return fail(TQ_ERR_INVALID, "tq_sdpa_int4_append: bad out_dtype");
  if (!k_new || !v_new) return fail(TQ_ERR_INVALID, "tq_sdpa_int4_append: null k_new/v_new");
  if (!valid_dtype(new_dtype)) return fail(TQ_ERR_INVALID, "tq_sdpa_int4_append: bad new_dtype");
  if (!aligned16(k_new) || !aligned16(v_new))
    return fail(TQ_ERR_INVALID, "tq_sdpa_int4_append: k_new/v_new must be 16-byte aligned");
  if (!seq_lens && n_tokens < 1)
    return fail(TQ_ERR_INVALID, "tq_sdpa_int4_append: n_tokens must include the new token (>= 1)");
  if (slot >= 0 && (seq_lens || slot >= n_tokens))
    return fail(TQ_ERR_INVALID, "tq_sdpa_int4_append_at: slot must be < n_tokens (and no seq_lens)");
  DecodeCommon c{queries, q_dtype, k_quant, v_quant, k_scales, k_biases, v_scales, v_biases,
                 sb_dtype, gqa_factor, sliding_window, batch, num_kv_heads, head_dim, n_tokens,
                 capacity, scale, k_new, v_new, new_dtype, slot, slots};
  return decode_common(c, "tq_sdpa_int4_append", seq_lens, 0, 0, 0, out, out_dtype, nullptr,
                       workspace, workspace_bytes, stream);
}

int tq_sdpa_int4_append(const void* queries, tq_dtype q_dtype, const void* k_new,
                        const void* v_new, tq_dtype new_dtype, uint32_t* k_quant, void* k_scales,
                        void* k_biases, uint32_t* v_quant, void* v_scales, void* v_biases,
                        tq_dtype sb_dtype, int gqa_factor, float scale, int sliding_window,
                        int batch, int num_kv_heads, int head_dim, int n_tokens, int capacity,
                        const int32_t* seq_lens, void* out, tq_dtype out_dtype, void* workspace,
                        size_t workspace_bytes, void* stream) {
  return append_common(queries, q_dtype, k_new, v_new, new_dtype, k_quant, k_scales, k_biases,
                       v_quant, v_scales, v_biases, sb_dtype, gqa_factor, scale, sliding_window,
                       batch, num_kv_heads, head_dim, n_tokens, capacity, seq_lens, -1, nullptr,
                       out, out_dtype, workspace, workspace_bytes, stream);
}

int tq_sdpa_int4_append_slots(const void* queries, tq_dtype q_dtype, const void* k_new,
                              const void* v_new, tq_dtype new_dtype, uint32_t* k_quant,
                              void* k_scales, void* k_biases, uint32_t* v_quant, void* v_scales,
                              void* v_biases, tq_dtype sb_dtype, int gqa_factor, float scale,
                              int sliding_window, int batch, int num_kv_heads, int head_dim,
                              int n_tokens, int capacity, const int32_t* seq_lens,
                              const int32_t* slots, void* out, tq_dtype out_dtype,
                              void* workspace, size_t workspace_bytes, void* stream) {
  if (!slots) return fail(TQ_ERR_INVALID, "tq_sdpa_int4_append_slots: null slots");
  return append_common(queries, q_dtype, k_new, v_new, new_dtype, k_quant, k_scales, k_biases,
                       v_quant, v_scales, v_biases, sb_dtype, gqa_factor, scale, sliding_window,
                       batch, num_kv_heads, head_dim, n_tokens, capacity, seq_lens, -1, slots,
                       out, out_dtype, workspace, workspace_bytes, stream);
}

int tq_sdpa_int4_append_at(const void* queries, tq_dtype q_dtype, const void* k_new,
                           const void* v_new, tq_dtype new_dtype, uint32_t* k_quant,
                           void* k_scales, void* k_biases, uint32_t* v_quant, void* v_scales,
                           void* v_biases, tq_dtype sb_dtype, int gqa_factor, float scale,
                           int batch, int num_kv_heads, int head_dim, int n_tokens, int capacity,
                           int slot, void* out, tq_dtype out_dtype, void* workspace,
                           size_t workspace_bytes, void* stream) {
  if (slot < 0) return fail(TQ_ERR_INVALID, "tq_sdpa_int4_append_at: slot must be >= 0");
  return append_common(queries, q_dtype, k_new, v_new, new_dtype, k_quant, k_scales, k_biases,
                       v_quant, v_scales, v_biases, sb_dtype, gqa_factor, scale, 0, batch,
                       num_kv_heads, head_dim, n_tokens, capacity, nullptr, slot, nullptr, out,
                       out_dtype, workspace, workspace_bytes, stream);
}

int tq_sdpa_int4_partial(const void* queries, tq_dtype q_dtype, const uint32_t* k_quant,
                         const void* k_scales, const void* k_biases, const uint32_t* v_quant,
                         const void* v_scales, const void* v_biases, tq_dtype sb_dtype,
                         int gqa_factor, float scale, int sliding_window, int batch,
                         int num_kv_heads, int head_dim, int n_local, int capacity,
                         int token_offset, int n_total, float* part_out, void* workspace,
                         size_t workspace_bytes, void* stream) {
  t_err.clear();
  if (!part_out) return fail(TQ_ERR_INVALID, "tq_sdpa_int4_partial: null part_out");
  if (token_offset < 0 || n_total < token_offset + n_local)
    return fail(TQ_ERR_INVALID, "tq_sdpa_int4_partial: need 0 <= token_offset and "
                "token_offset + n_local <= n_total");
  DecodeCommon c{queries, q_dtype, k_quant, v_quant, k_scales, k_biases, v_scales, v_biases,
                 sb_dtype, gqa_factor, sliding_window, batch, num_kv_heads, head_dim, n_local,
                 capacity, scale};
  return decode_common(c, "tq_sdpa_int4_partial", nullptr, token_offset, n_total, 1, nullptr,
                       TQ_F32, part_out, workspace, workspace_bytes, stream);
}

int tq_sdpa_int4_partial_publish(const void* queries, tq_dtype q_dtype, const uint32_t* k_quant,
                                 const void* k_scales, const void* k_biases,
                                 const uint32_t* v_quant, const void* v_scales,
                                 const void* v_biases, tq_dtype sb_dtype, int gqa_factor,
                                 float scale, int sliding_window, int batch, int num_kv_heads,
                                 int head_dim, int n_local, int capacity, int token_offset,
                                 int n_total, const void* k_new, const void* v_new,
                                 tq_dtype new_dtype, void* const* peer_bufs, int world, int rank,
                                 void* workspace, size_t workspace_bytes, void* stream) {
  t_err.clear();
  if (!peer_bufs) return fail(TQ_ERR_INVALID, "tq_sdpa_int4_partial_publish: null peer_bufs");
  if (!k_new != !v_new)
    return fail(TQ_ERR_INVALID, "tq_sdpa_int4_partial_publish: give both k_new and v_new or neither");
  if (k_new && (!valid_dtype(new_dtype) || !aligned16(k_new) || !aligned16(v_new) || n_local < 1))
    return fail(TQ_ERR_INVALID, "tq_sdpa_int4_partial_publish: k_new/v_new need a valid dtype, "
                "16-byte alignment and n_local >= 1 (the new token's slot is n_local - 1)");
  if (world < 1 || world > tq::kPeerMaxWorld || rank < 0 || rank >= world)
    return fail(TQ_ERR_INVALID, "tq_sdpa_int4_partial_publish: bad world/rank");
  if (token_offset < 0 || n_total < token_offset + n_local)
    return fail(TQ_ERR_INVALID, "tq_sdpa_int4_partial_publish: need 0 <= token_offset and "
                "token_offset + n_local <= n_total");
  DecodeCommon c{queries, q_dtype, k_quant, v_quant, k_scales, k_biases, v_scales, v_biases,
                 sb_dtype, gqa_factor, sliding_window, batch, num_kv_heads, head_dim, n_local,
                 capacity, scale};
  c.peer_bufs = peer_bufs;
  c.peer_world = world;
  c.peer_rank = rank;
  c.k_new = k_new;  // quantize-on-append of the new token in the same launch (nullable)
  c.v_new = v_new;
  c.new_dtype = new_dtype;
  return decode_common(c, "tq_sdpa_int4_partial_publish", nullptr, token_offset, n_total, 1,
                       nullptr, TQ_F32, nullptr, workspace, workspace_bytes, stream);
}

int tq_lse_merge(const float* parts, int n_parts, int batch, int num_heads, int head_dim,
                 void* out, tq_dtype out_dtype, void* stream) {
  t_err.clear();
  if (!parts || !out) return fail(TQ_ERR_INVALID, "tq_lse_merge: null pointer");
  if (n_parts < 1 || n_parts > 64) return fail(TQ_ERR_INVALID, "tq_lse_merge: n_parts %d not in 1..64", n_parts);
  if (batch < 1 || num_heads < 1 || head_dim < 1) return fail(TQ_ERR_INVALID, "tq_lse_merge: bad sizes");
  if (!valid_dtype(out_dtype)) return fail(TQ_ERR_INVALID, "tq_lse_merge: bad out_dtype");
  cudaError_t e = tq::launch_lse_merge(parts, n_parts, batch, num_heads, head_dim, out, out_dtype,
                                       static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "tq_lse_merge launch");
  return TQ_OK;
}

int tq_device_error(void* stream, uint32_t* code) {
  t_err.clear();
  uint32_t* p = device_error_ptr();
  if (!p) return fail(TQ_ERR_CUDA, "tq_device_error: no device error word");
  uint32_t v = 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(&v, p, sizeof(v), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaMemsetAsync(p, 0, sizeof(uint32_t), s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_fail(e, "tq_device_error");
  if (code) *code = v;
  return TQ_OK;
}

}  // extern "C"
