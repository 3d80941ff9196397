// One decode step of one layer from host memory in one call: the host-side
// equivalent of the reference's per-token call sequence, where the query and
// the new K/V row live in host-visible (unified) memory and the output is read
// back on the host (engine/gemma4_multilayer.cpp:222-236 quantizes, appends
// and calls sdpa_int4 per layer; lib/turboquant.cpp:368-401 encodes the
// kernel). Here the step is a CUDA graph of two kernels captured once per
// decode plan:
//
//   gather: one thread per 16 bytes reads [queries | k_new | v_new |
//           seq_lens | slots] from mapped pinned host memory into a device
//           buffer
//   -> tq_sdpa_int4_append (quantize-on-append fused into the decode kernel),
//      a programmatic dependent launch: its prologue (barrier init, L2
//      prefetch of its first tiles) overlaps the gather; it writes the output
//      straight into mapped pinned host memory
//
// so the host pays one graph launch and one stream synchronisation per step,
// and no copy-engine node sits on the path. The per-sequence lengths and the
// slots the new rows go to travel with the inputs (n - 1 for a growing cache,
// position mod window for a ring), so one graph serves every length whose
// decode plan (splits x tiles per split) is the same; a new plan re-captures
// and updates the executable graph in place.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <new>

#include "../../include/turboquant_c.h"
#include "tq_common.cuh"
#include "tq_internal.h"

struct tq_decode_step {
  int device = 0;
  cudaStream_t stream = nullptr;
  // cache and step description
  tq_dtype q_dtype, new_dtype, sb_dtype, out_dtype;
  uint32_t* kq;
  void *ks, *kb;
  uint32_t* vq;
  void *vs, *vb;
  int gqa, window, B, Hkv, D, capacity;
  float scale;
  // staging: [q | k_new | v_new | seq_lens | slots] in mapped pinned host
  // memory and its device copy; the output in mapped pinned host memory
  size_t q_bytes, kv_bytes, len_bytes, in_bytes, out_bytes;
  unsigned char* h_in = nullptr;
  const uint4* h_in_dev = nullptr;  // h_in as the device sees it
  unsigned char* d_in = nullptr;
  void* h_out = nullptr;
  void* h_out_dev = nullptr;
  void* ws = nullptr;
  size_t ws_bytes = 0;
  // the captured step and the plan it was captured for
  cudaGraphExec_t exec = nullptr;
  int plan_splits = -1, plan_tps = -1, plan_variant = -1;
  // the last decode plan and the visible-tile count it was made for: the plan
  // depends on the lengths only through that count
  tq::DecodePlan last_plan{};
  int last_tiles = -1;
};

namespace {

constexpr int kGatherThreads = 256;

// Copy n16 16-byte words of the step's inputs from mapped host memory into
// device memory, one word per thread over as many CTAs as that takes, so all
// the reads cross PCIe at once (one round trip). The dependent decode kernel
// may start at once: it reads the copy only after its griddepcontrol.wait,
// which returns once this grid has completed and its writes are visible.
// Loads bypass the caches (.cv): the host rewrites the staging buffer between
// steps.
__global__ void __launch_bounds__(kGatherThreads) step_gather_kernel(const uint4* __restrict__ src,
                                                                     uint4* __restrict__ dst, int n16) {
  tq::pdl_trigger();
  const int i = blockIdx.x * kGatherThreads + threadIdx.x;
  if (i < n16) dst[i] = __ldcv(src + i);
}

size_t dtype_bytes(tq_dtype d) { return d == TQ_F32 ? 4 : 2; }

int fail_step(int code, const char* what) {
  tq::set_last_error("%s", what);
  return code;
}

int cuda_step_fail(cudaError_t e, const char* what) {
  tq::set_last_error("%s: %s", what, cudaGetErrorString(e));
  return TQ_ERR_CUDA;
}

void release(tq_decode_step* s) {
  if (s->exec) cudaGraphExecDestroy(s->exec);
  if (s->ws) cudaFree(s->ws);
  if (s->d_in) cudaFree(s->d_in);
  if (s->h_out) cudaFreeHost(s->h_out);
  if (s->h_in) cudaFreeHost(s->h_in);
  if (s->stream) cudaStreamDestroy(s->stream);
  delete s;
}

// Capture the step's two kernels (gather, fused append + decode) for a step
// whose longest sequence has n tokens and install them as the executable
// graph (update in place when one exists).
int capture(tq_decode_step* s, int n, const tq::DecodePlan& pl) {
  if (pl.ws_bytes > s->ws_bytes) {
    if (s->ws) cudaFree(s->ws);
    s->ws = nullptr;
    s->ws_bytes = 0;
    cudaError_t e = cudaMalloc(&s->ws, pl.ws_bytes);
    if (e == cudaSuccess) e = cudaMemset(s->ws, 0, pl.ws_bytes);
    if (e != cudaSuccess) return cuda_step_fail(e, "tq_decode_step_run: workspace");
    s->ws_bytes = pl.ws_bytes;
  }
  cudaGraph_t graph = nullptr;
  cudaError_t e = cudaStreamBeginCapture(s->stream, cudaStreamCaptureModeThreadLocal);
  if (e != cudaSuccess) return cuda_step_fail(e, "tq_decode_step_run: begin capture");
  const bool pdl = tq::pdl_launches();
  tq::pdl_launches() = true;  // the decode kernel follows the gather kernel
  const int32_t* seq = reinterpret_cast<const int32_t*>(s->d_in + s->q_bytes + 2 * s->kv_bytes);
  const int32_t* slots = reinterpret_cast<const int32_t*>(s->d_in + s->q_bytes + 2 * s->kv_bytes +
                                                          s->len_bytes);
  const int n16 = static_cast<int>(s->in_bytes / 16);
  step_gather_kernel<<<(n16 + kGatherThreads - 1) / kGatherThreads, kGatherThreads, 0, s->stream>>>(
      s->h_in_dev, reinterpret_cast<uint4*>(s->d_in), n16);
  e = cudaGetLastError();
  int rc = TQ_OK;
  if (e == cudaSuccess)
    rc = tq_sdpa_int4_append_slots(s->d_in, s->q_dtype, s->d_in + s->q_bytes,
                                   s->d_in + s->q_bytes + s->kv_bytes, s->new_dtype, s->kq, s->ks,
                                   s->kb, s->vq, s->vs, s->vb, s->sb_dtype, s->gqa, s->scale,
                                   s->window, s->B, s->Hkv, s->D, n, s->capacity, seq, slots,
                                   s->h_out_dev, s->out_dtype, s->ws, s->ws_bytes, s->stream);
  tq::pdl_launches() = pdl;
  const cudaError_t e3 = cudaStreamEndCapture(s->stream, &graph);
  if (e != cudaSuccess || e3 != cudaSuccess || rc != TQ_OK) {
    if (graph) cudaGraphDestroy(graph);
    if (rc != TQ_OK) return rc;  // tq_last_error() holds the entry point's message
    return cuda_step_fail(e != cudaSuccess ? e : e3, "tq_decode_step_run: capture");
  }
  if (s->exec) {
    cudaGraphExecUpdateResultInfo info;
    if (cudaGraphExecUpdate(s->exec, graph, &info) != cudaSuccess) {
      cudaGetLastError();  // a failed update leaves the old graph; instantiate anew
      cudaGraphExecDestroy(s->exec);
      s->exec = nullptr;
    }
  }
  if (!s->exec) e = cudaGraphInstantiate(&s->exec, graph, 0);
  cudaGraphDestroy(graph);
  if (e != cudaSuccess) {
    s->exec = nullptr;
    return cuda_step_fail(e, "tq_decode_step_run: instantiate");
  }
  s->plan_splits = pl.splits;
  s->plan_tps = pl.tiles_per_split;
  s->plan_variant = pl.variant;
  return TQ_OK;
}

}  // namespace

extern "C" {

TQ_API int tq_decode_step_create(tq_dtype q_dtype, tq_dtype new_dtype, uint32_t* k_quant,
                                 void* k_scales, void* k_biases, uint32_t* v_quant, void* v_scales,
                                 void* v_biases, tq_dtype sb_dtype, int gqa_factor, float scale,
                                 int sliding_window, int batch, int num_kv_heads, int head_dim,
                                 int capacity, tq_dtype out_dtype, tq_decode_step** step) {
  tq::set_last_error("%s", "");
  if (!step) return fail_step(TQ_ERR_INVALID, "tq_decode_step_create: null step");
  *step = nullptr;
  auto ok_dt = [](int d) { return d == TQ_F32 || d == TQ_F16 || d == TQ_BF16; };
  if (!ok_dt(q_dtype) || !ok_dt(new_dtype) || !ok_dt(out_dtype) ||
      (sb_dtype != TQ_F16 && sb_dtype != TQ_F32))
    return fail_step(TQ_ERR_INVALID, "tq_decode_step_create: bad dtype");
  if (!k_quant || !k_scales || !k_biases || !v_quant || !v_scales || !v_biases)
    return fail_step(TQ_ERR_INVALID, "tq_decode_step_create: null cache pointer");
  if (gqa_factor < 1 || batch < 1 || num_kv_heads < 1 || capacity < 4 || (capacity & 3) ||
      sliding_window < 0)
    return fail_step(TQ_ERR_INVALID, "tq_decode_step_create: bad sizes");
  if (head_dim != 128 && head_dim != 256 && head_dim != 512)
    return fail_step(TQ_ERR_UNSUPPORTED, "tq_decode_step_create: head_dim not supported (128, 256, 512)");
  tq_decode_step* s = new (std::nothrow) tq_decode_step();
  if (!s) return fail_step(TQ_ERR_INVALID, "tq_decode_step_create: out of host memory");
  s->q_dtype = q_dtype;
  s->new_dtype = new_dtype;
  s->sb_dtype = sb_dtype;
  s->out_dtype = out_dtype;
  s->kq = k_quant;
  s->ks = k_scales;
  s->kb = k_biases;
  s->vq = v_quant;
  s->vs = v_scales;
  s->vb = v_biases;
  s->gqa = gqa_factor;
  s->scale = scale;
  s->window = sliding_window;
  s->B = batch;
  s->Hkv = num_kv_heads;
  s->D = head_dim;
  s->capacity = capacity;
  const size_t H = static_cast<size_t>(num_kv_heads) * gqa_factor;
  // each section rounded up to 16 bytes: the kernels read them by bulk copy
  auto r16 = [](size_t x) { return (x + 15) & ~static_cast<size_t>(15); };
  s->q_bytes = r16(batch * H * head_dim * dtype_bytes(q_dtype));
  s->kv_bytes = r16(static_cast<size_t>(batch) * num_kv_heads * head_dim * dtype_bytes(new_dtype));
  s->len_bytes = r16(batch * sizeof(int32_t));
  s->in_bytes = s->q_bytes + 2 * s->kv_bytes + 2 * s->len_bytes;
  s->out_bytes = batch * H * head_dim * dtype_bytes(out_dtype);
  cudaError_t e = cudaGetDevice(&s->device);
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaHostAlloc(reinterpret_cast<void**>(&s->h_in), s->in_bytes, cudaHostAllocMapped);
  if (e == cudaSuccess) e = cudaHostAlloc(&s->h_out, s->out_bytes, cudaHostAllocMapped);
  void* hin_dev = nullptr;
  if (e == cudaSuccess) e = cudaHostGetDevicePointer(&hin_dev, s->h_in, 0);
  if (e == cudaSuccess) e = cudaHostGetDevicePointer(&s->h_out_dev, s->h_out, 0);
  if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void**>(&s->d_in), s->in_bytes);
  s->h_in_dev = static_cast<const uint4*>(hin_dev);
  if (e != cudaSuccess) {
    release(s);
    return cuda_step_fail(e, "tq_decode_step_create");
  }
  memset(s->h_in, 0, s->in_bytes);
  *step = s;
  return TQ_OK;
}

TQ_API int tq_decode_step_buffers(tq_decode_step* step, void** queries, void** k_new,
                                  void** v_new, void** out) {
  if (!step) return fail_step(TQ_ERR_INVALID, "tq_decode_step_buffers: null step");
  if (queries) *queries = step->h_in;
  if (k_new) *k_new = step->h_in + step->q_bytes;
  if (v_new) *v_new = step->h_in + step->q_bytes + step->kv_bytes;
  if (out) *out = step->h_out;
  return TQ_OK;
}

}  // extern "C"

namespace {

// One step: slots == nullptr writes each new row at slot n_tokens[b] - 1.
int run_step(tq_decode_step* s, const void* queries, const void* k_new, const void* v_new,
             const int32_t* n_tokens, const int32_t* slots, void* out) {
  if (!s) return fail_step(TQ_ERR_INVALID, "tq_decode_step_run: null step");
  if (!n_tokens) return fail_step(TQ_ERR_INVALID, "tq_decode_step_run: null n_tokens");
  int n_max = 0;
  for (int b = 0; b < s->B; ++b) {
    if (n_tokens[b] < 1 || n_tokens[b] > s->capacity) {
      tq::set_last_error("tq_decode_step_run: n_tokens[%d] = %d outside [1, capacity %d]", b,
                         n_tokens[b], s->capacity);
      return TQ_ERR_INVALID;
    }
    if (slots && (slots[b] < 0 || slots[b] >= n_tokens[b])) {
      tq::set_last_error("tq_decode_step_run_at: slots[%d] = %d outside [0, n_tokens %d)", b,
                         slots[b], n_tokens[b]);
      return TQ_ERR_INVALID;
    }
    n_max = std::max(n_max, n_tokens[b]);
  }
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev != s->device) {
    cudaError_t e = cudaSetDevice(s->device);
    if (e != cudaSuccess) return cuda_step_fail(e, "tq_decode_step_run: set device");
  }
  // inputs into staging (the caller may have written them there already)
  unsigned char* hq = s->h_in;
  const size_t qn = s->B * static_cast<size_t>(s->Hkv) * s->gqa * s->D * dtype_bytes(s->q_dtype);
  const size_t kn = s->B * static_cast<size_t>(s->Hkv) * s->D * dtype_bytes(s->new_dtype);
  if (queries && queries != hq) memcpy(hq, queries, qn);
  if (k_new && k_new != hq + s->q_bytes) memcpy(hq + s->q_bytes, k_new, kn);
  if (v_new && v_new != hq + s->q_bytes + s->kv_bytes)
    memcpy(hq + s->q_bytes + s->kv_bytes, v_new, kn);
  int32_t* h_len = reinterpret_cast<int32_t*>(hq + s->q_bytes + 2 * s->kv_bytes);
  int32_t* h_slot = reinterpret_cast<int32_t*>(hq + s->q_bytes + 2 * s->kv_bytes + s->len_bytes);
  for (int b = 0; b < s->B; ++b) {
    h_len[b] = n_tokens[b];
    h_slot[b] = slots ? slots[b] : n_tokens[b] - 1;
  }

  const int vis = s->window > 0 ? std::min(n_max, s->window) : n_max;
  const int tiles = s->last_tiles >= 0
                        ? (vis + s->last_plan.tokens_per_tile - 1) / s->last_plan.tokens_per_tile
                        : -1;
  if (tiles < 0 || tiles != s->last_tiles) {
    s->last_plan = tq::plan_decode(s->device, s->B, s->Hkv * s->gqa, s->Hkv, s->D, vis,
                                   s->window > 0, s->q_dtype != TQ_F16);
    s->last_tiles = (vis + s->last_plan.tokens_per_tile - 1) / s->last_plan.tokens_per_tile;
  }
  const tq::DecodePlan& pl = s->last_plan;
  if (pl.splits < 0) {
    if (dev != s->device) cudaSetDevice(dev);
    return fail_step(TQ_ERR_UNSUPPORTED, "tq_decode_step_run: batch * kv_heads too large");
  }
  int rc = TQ_OK;
  if (!s->exec || pl.splits != s->plan_splits || pl.tiles_per_split != s->plan_tps ||
      pl.variant != s->plan_variant)
    rc = capture(s, n_max, pl);
  cudaError_t e = cudaSuccess;
  if (rc == TQ_OK) {
    e = cudaGraphLaunch(s->exec, s->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s->stream);
    if (e != cudaSuccess) rc = cuda_step_fail(e, "tq_decode_step_run");
  }
  if (dev != s->device) cudaSetDevice(dev);
  if (rc != TQ_OK) return rc;
  if (out && out != s->h_out) memcpy(out, s->h_out, s->out_bytes);
  return TQ_OK;
}

}  // namespace

extern "C" {

TQ_API int tq_decode_step_run(tq_decode_step* step, const void* queries, const void* k_new,
                              const void* v_new, const int32_t* n_tokens, void* out) {
  return run_step(step, queries, k_new, v_new, n_tokens, nullptr, out);
}

TQ_API int tq_decode_step_run_at(tq_decode_step* step, const void* queries, const void* k_new,
                                 const void* v_new, const int32_t* n_tokens,
                                 const int32_t* slots, void* out) {
  if (!slots) return fail_step(TQ_ERR_INVALID, "tq_decode_step_run_at: null slots");
  return run_step(step, queries, k_new, v_new, n_tokens, slots, out);
}

TQ_API int tq_decode_step_destroy(tq_decode_step* step) {
  if (!step) return TQ_OK;
  int dev = 0;
  cudaGetDevice(&dev);
  const int own = step->device;
  if (dev != own) cudaSetDevice(own);
  cudaStreamSynchronize(step->stream);
  release(step);
  if (dev != own) cudaSetDevice(dev);
  return TQ_OK;
}

}  // extern "C"
