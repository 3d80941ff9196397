// tq_sdpa_int4_noalloc: decode attention for callers that cannot allocate
// device memory.
//
// tq_sdpa_int4 needs a caller-provided workspace for its split-KV partial
// results and merge counters. Some callers have no way to provide one: code
// that runs where cudaMalloc is off limits (inside a host callback, a custom
// allocator's own hot path, a process whose memory pool is fully reserved up
// front, or a foreign runtime that only hands out input/output buffers).
// This entry point serves them with a scratch area that lives in the library
// itself: a fixed-size __device__ array that every GPU which loads the
// library holds until the process exits. Nothing here calls cudaMalloc,
// cudaFree or any allocating routine. With lazy module loading the driver
// places the array on a device when its address is first looked up, which is
// the first call on that device; callers that reserve all device memory up
// front make that first call before reserving.
#include <cstdio>
#include <mutex>
#include <unordered_map>

#include "../../include/turboquant_c.h"
#include "tq_internal.h"

namespace {

// Largest split-KV workspace this entry point can serve (2 MiB per device).
// Enough for every head_dim 128/256 decode the planner produces (e.g. config 1
// at 32K needs ~0.5 MiB); head_dim 512 at long contexts needs more and is
// rejected.
constexpr size_t kNoAllocScratchBytes = 2u << 20;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_mu;
std::unordered_map<int, void*> g_scratch_ptr;  // device -> device address of the array

// Host code must not use &g_noalloc_scratch directly: on the host that name is
// a stand-in, not a device address. Resolve the real address once per device,
// with that device current.
int scratch_for_current_device(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    tq::set_last_error("tq_sdpa_int4_noalloc: cudaGetDevice failed: %s", cudaGetErrorString(e));
    return TQ_ERR_CUDA;
  }
  std::lock_guard<std::mutex> lock(g_mu);
  auto it = g_scratch_ptr.find(dev);
  if (it != g_scratch_ptr.end()) {
    *out = it->second;
    return TQ_OK;
  }
  void* ptr = nullptr;
  e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
  if (e != cudaSuccess || ptr == nullptr) {
    tq::set_last_error("tq_sdpa_int4_noalloc: cudaGetSymbolAddress failed on device %d: %s", dev,
                       cudaGetErrorString(e));
    return TQ_ERR_CUDA;
  }
  g_scratch_ptr[dev] = ptr;
  *out = ptr;
  return TQ_OK;
}

}  // namespace

extern "C" TQ_API int tq_sdpa_int4_noalloc(const void* queries, tq_dtype q_dtype,
                                           const uint32_t* k_quant, const void* k_scales,
                                           const void* k_biases, const uint32_t* v_quant,
                                           const void* v_scales, const void* v_biases,
                                           tq_dtype sb_dtype, int gqa_factor, float scale,
                                           int sliding_window, int batch, int num_kv_heads,
                                           int head_dim, int n_tokens, int capacity,
                                           const int32_t* seq_lens, void* out,
                                           tq_dtype out_dtype, void* stream) {
  // The shape checks come before the scratch is sized: sizing plans the
  // split, and the plan is only defined for shapes the decode accepts.
  if (head_dim != 128 && head_dim != 256 && head_dim != 512) {
    tq::set_last_error("tq_sdpa_int4_noalloc: head_dim %d not supported (128, 256, 512)", head_dim);
    return TQ_ERR_UNSUPPORTED;
  }
  if (gqa_factor != 1 && gqa_factor != 2 && gqa_factor != 4 && gqa_factor != 8) {
    tq::set_last_error("tq_sdpa_int4_noalloc: gqa_factor %d not in {1,2,4,8}", gqa_factor);
    return TQ_ERR_UNSUPPORTED;
  }
  if (batch < 1 || num_kv_heads < 1 || n_tokens < 0 || sliding_window < 0) {
    tq::set_last_error("tq_sdpa_int4_noalloc: need batch >= 1, num_kv_heads >= 1, n_tokens >= 0 "
                       "and sliding_window >= 0");
    return TQ_ERR_INVALID;
  }
  const size_t need = tq_sdpa_int4_workspace_size(batch, num_kv_heads * gqa_factor, num_kv_heads,
                                                  head_dim, n_tokens, sliding_window);
  if (need > kNoAllocScratchBytes) {
    tq::set_last_error(
        "tq_sdpa_int4_noalloc: these sizes need %zu bytes of split-KV scratch, more than the "
        "%zu-byte built-in area; use tq_sdpa_int4 with a caller workspace",
        need, kNoAllocScratchBytes);
    return TQ_ERR_WORKSPACE;
  }
  void* scratch = nullptr;
  if (need > 0) {
    if (int rc = scratch_for_current_device(&scratch)) return rc;
    // The array keeps whatever the previous call left. Only the merge
    // counters (the first kCounterRegionBytes) must start at zero; the split
    // partials are always written before they are read.
    const size_t clear = need < tq::kCounterRegionBytes ? need : tq::kCounterRegionBytes;
    cudaError_t e = cudaMemsetAsync(scratch, 0, clear, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) {
      tq::set_last_error("tq_sdpa_int4_noalloc: clearing the scratch counters failed: %s",
                         cudaGetErrorString(e));
      return TQ_ERR_CUDA;
    }
  }
  return tq_sdpa_int4(queries, q_dtype, k_quant, k_scales, k_biases, v_quant, v_scales, v_biases,
                      sb_dtype, gqa_factor, scale, sliding_window, batch, num_kv_heads, head_dim,
                      n_tokens, capacity, seq_lens, out, out_dtype, scratch,
                      need > 0 ? kNoAllocScratchBytes : 0, stream);
}
