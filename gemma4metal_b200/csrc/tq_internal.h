// Host-side launch interface between the C ABI (capi.cu) and the kernels.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <string>

namespace tq {

cudaError_t launch_quantize_rows(const void* x, int x_dtype, long long rows, int D, long long n_new,
                                 int Hkv, int capacity, long long bstride_tok, int pos,
                                 const int32_t* positions, uint32_t* codes, void* scales,
                                 void* biases, int sb_dtype, cudaStream_t stream,
                                 const void* x2 = nullptr, uint32_t* codes2 = nullptr,
                                 void* scales2 = nullptr, void* biases2 = nullptr,
                                 int pos_bias = 0);  // added to positions[b]

cudaError_t launch_dequantize(const uint32_t* codes, const void* scales, const void* biases,
                              int sb_dtype, long long rows, int D, void* out, int out_dtype,
                              cudaStream_t stream);

// Split-KV decode attention over an int4 cache.
struct DecodeArgs {
  const void* q;  // (B, H, D)
  int q_dtype;
  const uint32_t* kq;
  const void* ks;
  const void* kb;
  const uint32_t* vq;
  const void* vs;
  const void* vb;
  int sb_dtype;
  const int32_t* seq_lens;  // nullable: per-sequence local token count
  int n_tokens;             // uniform local count (or max when seq_lens given)
  int B, H, Hkv, D, G;      // G = query heads per KV head
  int capacity;
  long long bstride_tok;  // tokens between sequences in the cache arrays
  float scale;
  int window;
  int token_offset;  // global position of local slot 0 (sequence shards)
  int n_total;       // global sequence length (for the window); <=0: same as local
  int partial;       // 0: normalised output; 1: (o, m, l) partial state
  void* out;         // partial == 0: (B, H, D) in out_dtype
  int out_dtype;
  float* part_out;   // partial == 1: (B, H*(D+2))
  void* workspace;
  size_t workspace_bytes;
  uint32_t* err;
  // fused quantize-on-append (mma kernel only; nullable): (B, Hkv, D) rows
  // written to slot n_local - 1 of each sequence before the attention reads it
  const void* k_new = nullptr;
  const void* v_new = nullptr;
  int new_dtype = 0;
  int new_slot = -1;  // < 0: n_local - 1
  const int32_t* new_slots = nullptr;  // device, one slot per sequence (overrides new_slot)
  // partial == 1, tensor-core kernel: publish the state into every rank's
  // exchange buffer (peer_layout.cuh) instead of part_out
  void* const* peer_bufs = nullptr;
  int peer_world = 0;
  int peer_rank = 0;
};

// Decode kernel variants: the CUDA-core kernel (sdpa_decode.cu) and the
// warp-level tensor-core kernel (sdpa_decode_mma.cu).
enum DecodeVariant : int { kDecodeSimt = 0, kDecodeMma = 1 };

// Variant used for (D, heads per CTA); TQ_DECODE_KERNEL=simt|mma overrides.
int choose_decode_variant(int D, int G);

bool mma_supported(int D, int G);
int mma_tokens_per_tile();
int mma_occupancy(int device, int D, int gsub, bool qsplit);

// Plan: split count etc. Returns workspace bytes needed.
struct DecodePlan {
  int variant;
  int gsub;          // query heads per CTA (<= G)
  int nsub;          // G / gsub
  int tokens_per_tile;
  int splits;
  int tiles_per_split;
  size_t ws_bytes;
  size_t ws_o_off, ws_ml_off, ws_cnt_off;
};

// Bytes reserved at the start of every decode workspace for merge counters.
extern const size_t kCounterRegionBytes;

// splits == -1 marks a problem with more (batch x head-group) units than
// counters.
// qsplit: f32/bf16 queries (their kernels run fewer CTAs per SM, so they get
// no more splits than the f16 plan the workspace size is computed from).
DecodePlan plan_decode(int device, int B, int H, int Hkv, int D, int n_visible_max,
                       bool windowed, bool qsplit = false);
cudaError_t launch_decode_mma(const DecodeArgs& a, const DecodePlan& plan, cudaStream_t stream);
cudaError_t launch_decode(const DecodeArgs& a, const DecodePlan& plan, cudaStream_t stream);

cudaError_t launch_lse_merge(const float* parts, int n_parts, int B, int H, int D, void* out,
                             int out_dtype, cudaStream_t stream);

int device_sm_count(int device);

// Whether launch_pdl sets programmatic stream serialization on this thread
// (true by default). A host decode step turns it off while it captures its
// graph, where the kernel follows a host-to-device copy: there is no
// preceding kernel whose tail a launch could overlap.
bool& pdl_launches();

// Launch `kernel` with programmatic stream serialization, so it may start
// while the preceding kernel of the stream finishes (the kernel must call
// pdl_wait() before it touches global memory; without the attribute that
// wait returns at once).
template <typename... K, typename... A>
cudaError_t launch_pdl(void (*kernel)(K...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t stream, A&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_launches() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<A&&>(args)...);
}

// Why the last launch_* call on this thread failed before reaching the GPU
// ("" if it did not); the C ABI appends it to tq_last_error().
std::string& launch_detail();

// The current device's error word (kernels record bounded-wait timeouts in it).
uint32_t* device_error_word();

// Set the calling thread's tq_last_error() message (printf-style).
void set_last_error(const char* fmt, ...);

}  // namespace tq
