// Sequence-split merge over peer memory (NVLink / NVSwitch P2P stores), in
// place of an NCCL all-gather of the per-GPU partial states followed by the
// merge kernel: one launch pushes this rank's partial (B, H*(D+2)) fp32 into
// every rank's exchange buffer, raises a per-rank flag there, waits for all
// ranks' flags of this step and merges the states it received -- the same
// log-sum-exp merge as lse_merge.cu (the reference merges simdgroup states the
// same way, lib/turboquant.metal:838-888).
//
// A second form skips the push: the decode kernel stores its state as
// {value, step} pairs straight into every rank's buffer
// (tq_sdpa_int4_partial_publish) and peer_merge_published_kernel merges once
// the pairs of this step are in.
//
// Exchange buffer of one rank (allocated here, shared through CUDA IPC; the
// layout is in peer_layout.cuh):
//   header: [0] this rank's step counter, [32 * (1 + k)] flag of rank k (its
//           last pushed step; one 128 B line per rank), [32 * 65] grid counter
//   data:   [2 step parities][world][B * H * (D + 2)] fp32 (or pairs)
// Flags only grow and the ranks advance in lockstep (a rank's step e + 1
// needs every rank's push of e + 1, which follows that rank's merge of e), so
// a rank is at most one step ahead and the parity slots never collide. Every
// wait is bounded. On timeout the kernel records kErrPeerTimeout in the device
// error word, writes NaN to the outputs of the items whose states it could not
// gather (never a merge of stale slots), marks the exchange failed in its own
// header and leaves its step counter where it was; every later merge on a
// failed exchange records the timeout again and writes NaN. A failed exchange
// is out of step with the other ranks for good: the caller closes it and
// builds a new one.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>

#include "../../include/turboquant_c.h"
#include "tq_common.cuh"
#include "tq_internal.h"
#include "peer_layout.cuh"

namespace tq {
namespace {

constexpr int kGridCounter = kPeerGridCounter;
constexpr int kFailedWord = kPeerFailedWord;
constexpr int kMaxWorld = kPeerMaxWorld;
constexpr int kPeerThreads = 256;
__device__ __forceinline__ int flag_word(int k) { return peer_flag_word(k); }
#ifndef TQ_PEER_MERGE_PDL
#define TQ_PEER_MERGE_PDL 1
#endif
constexpr bool kPublishedMergePdl = TQ_PEER_MERGE_PDL != 0;

struct PeerParams {
  const float* part;      // this rank's partial state (B, H*(D+2)) (whole-state merge)
  void* const* bufs;      // device array: exchange buffer of every rank (own at [rank])
  int world, rank;
  int B, H, D;
  void* out;
  int out_dtype;
  long long budget;       // SM clocks a CTA may wait in all
  uint32_t* err;
};

// Reads this rank's step counter and failed word; returns the step. Lets the
// next kernel of the stream launch now (its griddepcontrol.wait still waits
// for this grid to complete): a decode kernel after the merge runs its
// prologue while the merge waits for the other ranks.
__device__ __forceinline__ uint32_t begin_step(uint32_t* own, uint32_t* s_step, int* s_failed) {
  pdl_trigger();
  if (threadIdx.x == 0) {
    *s_step = *reinterpret_cast<volatile uint32_t*>(own) + 1u;
    *s_failed = *reinterpret_cast<volatile uint32_t*>(own + kFailedWord) != 0u;
  }
  __syncthreads();
  return *s_step;
}

__device__ __forceinline__ void record_timeout(uint32_t* own, const PeerParams& p, int* s_failed) {
  *s_failed = 1;
  atomicOr(own + kFailedWord, 1u);
  atomicOr(p.err, kErrPeerTimeout);
}

// The last CTA to finish advances this rank's step counter (every CTA read it
// at its start, before any CTA could finish); a failed exchange keeps its
// step: it is out of step with the others for good.
__device__ __forceinline__ void end_step(uint32_t* own, uint32_t step) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned done = atomicAdd(own + kGridCounter, 1u);
    if (done == gridDim.x - 1) {
      own[kGridCounter] = 0u;
      if (*reinterpret_cast<volatile uint32_t*>(own + kFailedWord) == 0u)
        *reinterpret_cast<volatile uint32_t*>(own) = step;
    }
  }
}

__device__ __forceinline__ void store_nan(const PeerParams& p, int b, int h) {
  for (int d = threadIdx.x; d < p.D; d += kPeerThreads)
    store_from_float(p.out, (static_cast<long long>(b) * p.H + h) * p.D + d, p.out_dtype, NAN);
}

__global__ void __launch_bounds__(kPeerThreads) peer_merge_kernel(const PeerParams p) {
  __shared__ uint32_t s_step;
  __shared__ float s_w[kMaxWorld];
  __shared__ float s_L;
  __shared__ int s_failed;
  uint32_t* own = static_cast<uint32_t*>(p.bufs[p.rank]);
  const uint32_t step = begin_step(own, &s_step, &s_failed);
  const long long blk = static_cast<long long>(p.B) * p.H * (p.D + 2);  // floats per state
  const int par = static_cast<int>(step & 1u);

  // ---- push: CTA j copies the state into rank j's slot [par][rank]
  for (int j = blockIdx.x; j < p.world; j += gridDim.x) {
    float* dst = reinterpret_cast<float*>(static_cast<uint32_t*>(p.bufs[j]) + peer_data_word()) +
                 (static_cast<long long>(par) * p.world + p.rank) * blk;
    if ((blk & 3) == 0) {
      const float4* s4 = reinterpret_cast<const float4*>(p.part);
      float4* d4 = reinterpret_cast<float4*>(dst);
      for (long long i = threadIdx.x; i < blk / 4; i += kPeerThreads) d4[i] = s4[i];
    } else {
      for (long long i = threadIdx.x; i < blk; i += kPeerThreads) dst[i] = p.part[i];
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) st_release_sys(static_cast<uint32_t*>(p.bufs[j]) + flag_word(p.rank), step);
  }

  // ---- wait for every rank's state of this step (bounded; none on a failed exchange)
  const long long t0 = clock64();
  for (int k = threadIdx.x; k < p.world && !s_failed; k += kPeerThreads) {
    while (static_cast<int>(ld_acquire_sys(own + flag_word(k)) - step) < 0) {
      if (clock64() - t0 > p.budget) {
        record_timeout(own, p, &s_failed);
        break;
      }
    }
  }
  __syncthreads();
  const bool failed = s_failed != 0;
  if (failed && threadIdx.x == 0) atomicOr(p.err, kErrPeerTimeout);  // (again, on a failed exchange)

  // ---- merge: CTA c takes (sequence, head) items c, c + grid, ...
  const float* data = reinterpret_cast<const float*>(own + peer_data_word()) +
                      static_cast<long long>(par) * p.world * blk;
  const long long hd = static_cast<long long>(p.H) * p.D;
  for (int item = blockIdx.x; item < p.B * p.H; item += gridDim.x) {
    const int b = item / p.H, h = item % p.H;
    const float* base = data + static_cast<long long>(b) * p.H * (p.D + 2);
    if (failed) {  // no complete set of states: NaN, never stale slots
      store_nan(p, b, h);
      continue;
    }
    if (threadIdx.x == 0) {
      float M = -INFINITY;
      for (int k = 0; k < p.world; ++k) M = fmaxf(M, __ldcg(base + k * blk + hd + 2 * h));
      float L = 0.0f;
      for (int k = 0; k < p.world; ++k) {
        const float m = __ldcg(base + k * blk + hd + 2 * h);
        const float l = __ldcg(base + k * blk + hd + 2 * h + 1);
        // an empty state (m = -inf) weighs 0; a NaN state makes the result NaN
        const float w = m == -INFINITY ? 0.0f : __expf(m - M);
        s_w[k] = w;
        L += w * l;
      }
      s_L = L;
    }
    __syncthreads();
    const float L = s_L;
    for (int d = threadIdx.x; d < p.D; d += kPeerThreads) {
      float acc = 0.0f;
      for (int k = 0; k < p.world; ++k)  // an empty state's o is never read
        if (s_w[k] != 0.0f) acc += s_w[k] * __ldcg(base + k * blk + static_cast<long long>(h) * p.D + d);
      store_from_float(p.out, (static_cast<long long>(b) * p.H + h) * p.D + d, p.out_dtype,
                       L == 0.0f ? 0.0f : acc / L);
    }
    __syncthreads();
  }
  end_step(own, step);
}

// Merge of states the decode kernel published as {value, step} pairs
// (peer_layout.cuh): a value counts once its pair carries this step, so no
// flag or fence is needed on either side. Per item, the 2 * world (m, l)
// pairs are awaited first (with a short back-off: this kernel may start while
// the decode kernel still runs), then the o pairs, each read whole. The slot
// parity keeps a rank that is one step ahead from overwriting pairs a slower
// rank still reads (its step e + 2 needs every rank's pairs of e + 1, which
// follow that rank's merge of e). One bound for all of a CTA's waits.
__global__ void __launch_bounds__(kPeerThreads) peer_merge_published_kernel(const PeerParams p) {
  __shared__ uint32_t s_step;
  __shared__ float s_ml[2 * kMaxWorld];
  __shared__ float s_w[kMaxWorld];
  __shared__ float s_L;
  __shared__ int s_failed;
  uint32_t* own = static_cast<uint32_t*>(p.bufs[p.rank]);
  const uint32_t step = begin_step(own, &s_step, &s_failed);
  if (s_failed && threadIdx.x == 0) atomicOr(p.err, kErrPeerTimeout);  // (again, on a failed exchange)
  const long long blk = static_cast<long long>(p.B) * p.H * (p.D + 2);  // pairs per state
  const uint2* data = reinterpret_cast<const uint2*>(own + peer_data_word()) +
                      static_cast<long long>(step & 1u) * p.world * blk;
  const long long hd = static_cast<long long>(p.H) * p.D;
  const long long t0 = clock64();
  for (int item = blockIdx.x; item < p.B * p.H; item += gridDim.x) {
    const int b = item / p.H, h = item % p.H;
    const uint2* base = data + static_cast<long long>(b) * p.H * (p.D + 2);
    for (int t = threadIdx.x; t < 2 * p.world && !s_failed; t += kPeerThreads) {
      const uint2* q = base + (t >> 1) * blk + hd + 2 * h + (t & 1);
      uint2 v = ld_pair(q);
      while (v.y != step) {
        if (clock64() - t0 > p.budget) {
          record_timeout(own, p, &s_failed);
          break;
        }
        __nanosleep(64);
        v = ld_pair(q);
      }
      s_ml[t] = __uint_as_float(v.x);
    }
    __syncthreads();
    if (s_failed) {  // no complete set of states: NaN, never stale pairs
      store_nan(p, b, h);
      continue;
    }
    if (threadIdx.x == 0) {
      float M = -INFINITY;
      for (int k = 0; k < p.world; ++k) M = fmaxf(M, s_ml[2 * k]);
      float L = 0.0f;
      for (int k = 0; k < p.world; ++k) {
        // an empty state (m = -inf) weighs 0; a NaN state makes the result NaN
        const float w = s_ml[2 * k] == -INFINITY ? 0.0f : __expf(s_ml[2 * k] - M);
        s_w[k] = w;
        L += w * s_ml[2 * k + 1];
      }
      s_L = L;
    }
    __syncthreads();
    const float L = s_L;
    for (int d = threadIdx.x; d < p.D; d += kPeerThreads) {
      float acc = 0.0f;
      bool ok = true;
      for (int k = 0; k < p.world && ok; ++k) {  // an empty state's o is never read
        if (s_w[k] == 0.0f) continue;
        const uint2* q = base + k * blk + static_cast<long long>(h) * p.D + d;
        uint2 v = ld_pair(q);
        while (v.y != step) {
          if (clock64() - t0 > p.budget) {
            record_timeout(own, p, &s_failed);
            ok = false;
            break;
          }
          v = ld_pair(q);
        }
        acc += s_w[k] * __uint_as_float(v.x);
      }
      store_from_float(p.out, (static_cast<long long>(b) * p.H + h) * p.D + d, p.out_dtype,
                       !ok ? NAN : L == 0.0f ? 0.0f : acc / L);
    }
    __syncthreads();
  }
  end_step(own, step);
}

// Gather of states the decode kernel published as {value, step} pairs when
// the ranks split the heads rather than the sequence: rank k's slot holds
// the complete state of its p.H heads, so each (sequence, rank, head) item is
// normalised on its own (o / l) into head k * p.H + j of the (B, world * p.H,
// D) output -- no merge across ranks. Waits, bound, NaN and failed-exchange
// rules as for the merge.
__global__ void __launch_bounds__(kPeerThreads) peer_gather_published_kernel(const PeerParams p) {
  __shared__ uint32_t s_step;
  __shared__ float s_l;
  __shared__ int s_failed;
  uint32_t* own = static_cast<uint32_t*>(p.bufs[p.rank]);
  const uint32_t step = begin_step(own, &s_step, &s_failed);
  if (s_failed && threadIdx.x == 0) atomicOr(p.err, kErrPeerTimeout);  // (again, on a failed exchange)
  const long long blk = static_cast<long long>(p.B) * p.H * (p.D + 2);  // pairs per state
  const uint2* data = reinterpret_cast<const uint2*>(own + peer_data_word()) +
                      static_cast<long long>(step & 1u) * p.world * blk;
  const long long hd = static_cast<long long>(p.H) * p.D;
  const int Hout = p.world * p.H;
  const long long t0 = clock64();
  for (int item = blockIdx.x; item < p.B * Hout; item += gridDim.x) {
    const int b = item / Hout, k = (item % Hout) / p.H, j = item % p.H;
    const uint2* base = data + k * blk + static_cast<long long>(b) * p.H * (p.D + 2);
    const long long ob = (static_cast<long long>(b) * Hout + k * p.H + j) * p.D;
    if (threadIdx.x == 0 && !s_failed) {
      const uint2* q = base + hd + 2 * j + 1;  // l
      uint2 v = ld_pair(q);
      while (v.y != step) {
        if (clock64() - t0 > p.budget) {
          record_timeout(own, p, &s_failed);
          break;
        }
        __nanosleep(64);
        v = ld_pair(q);
      }
      s_l = __uint_as_float(v.x);
    }
    __syncthreads();
    if (s_failed) {  // no complete state: NaN, never stale pairs
      for (int d = threadIdx.x; d < p.D; d += kPeerThreads)
        store_from_float(p.out, ob + d, p.out_dtype, NAN);
      continue;
    }
    const float L = s_l;
    for (int d = threadIdx.x; d < p.D; d += kPeerThreads) {
      const uint2* q = base + static_cast<long long>(j) * p.D + d;
      uint2 v = ld_pair(q);
      bool ok = true;
      while (v.y != step) {
        if (clock64() - t0 > p.budget) {
          record_timeout(own, p, &s_failed);
          ok = false;
          break;
        }
        v = ld_pair(q);
      }
      store_from_float(p.out, ob + d, p.out_dtype,
                       !ok ? NAN : L == 0.0f ? 0.0f : __uint_as_float(v.x) / L);
    }
    __syncthreads();
  }
  end_step(own, step);
}

size_t state_floats(int world, int B, int H, int D) {
  return 2ull * world * B * H * (D + 2);
}

}  // namespace
}  // namespace tq

using namespace tq;

extern "C" {

TQ_API size_t tq_peer_buffer_bytes(int world, int batch, int num_heads, int head_dim) {
  if (world < 1 || world > kMaxWorld || batch < 1 || num_heads < 1 || head_dim < 1) return 0;
  // the data region holds {value, step} pairs for published states
  return static_cast<size_t>(peer_data_word()) * sizeof(uint32_t) +
         state_floats(world, batch, num_heads, head_dim) * 2 * sizeof(float);
}

TQ_API int tq_peer_buffer_alloc(size_t bytes, void** buf) {
  if (!buf || bytes == 0) {
    set_last_error("tq_peer_buffer_alloc: bad arguments");
    return TQ_ERR_INVALID;
  }
  cudaError_t e = cudaMalloc(buf, bytes);
  if (e == cudaSuccess) e = cudaMemset(*buf, 0, bytes);
  if (e != cudaSuccess) {
    set_last_error("tq_peer_buffer_alloc: %s", cudaGetErrorString(e));
    return TQ_ERR_CUDA;
  }
  return TQ_OK;
}

TQ_API int tq_peer_buffer_free(void* buf) {
  const cudaError_t e = cudaFree(buf);
  if (e != cudaSuccess) {
    set_last_error("tq_peer_buffer_free: %s", cudaGetErrorString(e));
    return TQ_ERR_CUDA;
  }
  return TQ_OK;
}

TQ_API int tq_ipc_handle(void* buf, void* handle) {
  if (!buf || !handle) {
    set_last_error("tq_ipc_handle: null pointer");
    return TQ_ERR_INVALID;
  }
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, buf);
  if (e != cudaSuccess) {
    set_last_error("tq_ipc_handle: %s", cudaGetErrorString(e));
    return TQ_ERR_CUDA;
  }
  static_assert(sizeof(h) == TQ_IPC_HANDLE_BYTES, "IPC handle size");
  memcpy(handle, &h, sizeof(h));
  return TQ_OK;
}

TQ_API int tq_ipc_open(const void* handle, void** peer_buf) {
  if (!handle || !peer_buf) {
    set_last_error("tq_ipc_open: null pointer");
    return TQ_ERR_INVALID;
  }
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(peer_buf, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    set_last_error("tq_ipc_open: %s", cudaGetErrorString(e));
    return TQ_ERR_CUDA;
  }
  return TQ_OK;
}

TQ_API int tq_ipc_close(void* peer_buf) {
  const cudaError_t e = cudaIpcCloseMemHandle(peer_buf);
  if (e != cudaSuccess) {
    set_last_error("tq_ipc_close: %s", cudaGetErrorString(e));
    return TQ_ERR_CUDA;
  }
  return TQ_OK;
}

static int peer_merge_common(const float* part, void* const* peer_bufs, int world, int rank,
                             int batch, int num_heads, int head_dim, bool published, void* out,
                             tq_dtype out_dtype, int timeout_us, void* stream);

TQ_API int tq_peer_merge(const float* part, void* const* peer_bufs, int world, int rank,
                         int batch, int num_heads, int head_dim, void* out, tq_dtype out_dtype,
                         int timeout_us, void* stream) {
  if (!part) {
    set_last_error("tq_peer_merge: null pointer");
    return TQ_ERR_INVALID;
  }
  return peer_merge_common(part, peer_bufs, world, rank, batch, num_heads, head_dim, false, out,
                           out_dtype, timeout_us, stream);
}

TQ_API int tq_peer_merge_published(void* const* peer_bufs, int world, int rank, int batch,
                                   int num_heads, int head_dim, void* out, tq_dtype out_dtype,
                                   int timeout_us, void* stream) {
  return peer_merge_common(nullptr, peer_bufs, world, rank, batch, num_heads, head_dim, true, out,
                           out_dtype, timeout_us, stream);
}

TQ_API int tq_peer_gather_published(void* const* peer_bufs, int world, int rank, int batch,
                                    int num_heads, int head_dim, void* out, tq_dtype out_dtype,
                                    int timeout_us, void* stream) {
  if (!peer_bufs || !out) {
    set_last_error("tq_peer_gather_published: null pointer");
    return TQ_ERR_INVALID;
  }
  if (world < 1 || world > kMaxWorld || rank < 0 || rank >= world || batch < 1 || num_heads < 1 ||
      head_dim < 1 || timeout_us < 1) {
    set_last_error("tq_peer_gather_published: bad sizes");
    return TQ_ERR_INVALID;
  }
  int dev = 0, khz = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&khz, cudaDevAttrClockRate, dev);
  PeerParams p{};
  p.bufs = peer_bufs;
  p.world = world;
  p.rank = rank;
  p.B = batch;
  p.H = num_heads;
  p.D = head_dim;
  p.out = out;
  p.out_dtype = out_dtype;
  p.budget = static_cast<long long>(timeout_us) * (khz > 0 ? khz : 2000000) / 1000;
  p.err = device_error_word();
  int grid = batch * num_heads * world;
  if (grid > 148) grid = 148;
  const cudaError_t e = launch_pdl(peer_gather_published_kernel, dim3(grid), dim3(kPeerThreads), 0,
                                   static_cast<cudaStream_t>(stream), p);
  if (e != cudaSuccess) {
    set_last_error("tq_peer_gather_published: %s", cudaGetErrorString(e));
    return TQ_ERR_CUDA;
  }
  return TQ_OK;
}

static int peer_merge_common(const float* part, void* const* peer_bufs, int world, int rank,
                             int batch, int num_heads, int head_dim, bool published, void* out,
                             tq_dtype out_dtype, int timeout_us, void* stream) {
  const char* fn = published ? "tq_peer_merge_published" : "tq_peer_merge";
  if (!peer_bufs || !out) {
    set_last_error("%s: null pointer", fn);
    return TQ_ERR_INVALID;
  }
  if (world < 1 || world > kMaxWorld || rank < 0 || rank >= world || batch < 1 || num_heads < 1 ||
      head_dim < 1 || timeout_us < 1) {
    set_last_error("%s: bad sizes", fn);
    return TQ_ERR_INVALID;
  }
  if (part && (reinterpret_cast<uintptr_t>(part) & 15u)) {
    set_last_error("%s: part must be 16-byte aligned", fn);
    return TQ_ERR_INVALID;
  }
  int dev = 0, khz = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&khz, cudaDevAttrClockRate, dev);
  PeerParams p{};
  p.part = part;
  p.bufs = peer_bufs;
  p.world = world;
  p.rank = rank;
  p.B = batch;
  p.H = num_heads;
  p.D = head_dim;
  p.out = out;
  p.out_dtype = out_dtype;
  p.budget = static_cast<long long>(timeout_us) * (khz > 0 ? khz : 2000000) / 1000;
  p.err = device_error_word();
  int grid = batch * num_heads;
  if (!published && grid < world) grid = world;  // one pushing CTA per rank
  if (grid > 148) grid = 148;
  cudaError_t e;
  if (published && kPublishedMergePdl) {
    // nothing of the preceding decode kernel is read but through pairs that
    // carry this step, so the merge may start once that kernel's CTAs have
    // all started and merge each item as soon as its pairs are in
    e = launch_pdl(peer_merge_published_kernel, dim3(grid), dim3(kPeerThreads), 0,
                   static_cast<cudaStream_t>(stream), p);
  } else if (published) {
    peer_merge_published_kernel<<<grid, kPeerThreads, 0, static_cast<cudaStream_t>(stream)>>>(p);
    e = cudaGetLastError();
  } else {
    peer_merge_kernel<<<grid, kPeerThreads, 0, static_cast<cudaStream_t>(stream)>>>(p);
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) {
    set_last_error("%s: %s", fn, cudaGetErrorString(e));
    return TQ_ERR_CUDA;
  }
  return TQ_OK;
}

}  // extern "C"
