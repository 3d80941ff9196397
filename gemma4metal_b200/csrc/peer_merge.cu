// Sequence-split merge over peer memory (NVLink / NVSwitch P2P stores), in
// place of an NCCL all-gather of the per-GPU partial states followed by the
// merge kernel: one launch pushes this rank's partial (B, H*(D+2)) fp32 into
// every rank's exchange buffer, raises a per-rank flag there, waits for all
// ranks' flags of this step and merges the states it received -- the same
// log-sum-exp merge as lse_merge.cu (the reference merges simdgroup states the
// same way, lib/turboquant.metal:838-888).
//
// Exchange buffer of one rank (allocated here, shared through CUDA IPC):
//   header: [0] this rank's step counter, [32 * (1 + k)] flag of rank k (its
//           last pushed step; one 128 B line per rank), [32 * 65] grid counter
//   data:   [2 step parities][world][B * H * (D + 2)] fp32
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
// back-off between flag polls: a waiting CTA shares its SM with decode CTAs
#ifndef TQ_PEER_POLL_NS
#define TQ_PEER_POLL_NS 0
#endif
constexpr unsigned kPollSleepNs = TQ_PEER_POLL_NS;

struct PeerParams {
  const float* part;      // this rank's partial state (B, H*(D+2))
  void* const* bufs;      // device array: exchange buffer of every rank (own at [rank])
  int world, rank;
  int B, H, D;
  void* out;
  int out_dtype;
  long long budget;       // SM clocks a wait may take
  uint32_t* err;
  int units;              // > 0: the decode kernel published the states per unit (no push here)
};

__global__ void __launch_bounds__(kPeerThreads) peer_merge_kernel(const PeerParams p) {
  __shared__ uint32_t s_step;
  __shared__ float s_w[kMaxWorld];
  __shared__ float s_L;
  __shared__ int s_failed;
  uint32_t* own = static_cast<uint32_t*>(p.bufs[p.rank]);
  if (threadIdx.x == 0) {
    s_step = *reinterpret_cast<volatile uint32_t*>(own) + 1u;
    s_failed = *reinterpret_cast<volatile uint32_t*>(own + kFailedWord) != 0u;
  }
  __syncthreads();
  const uint32_t step = s_step;
  const long long blk = static_cast<long long>(p.B) * p.H * (p.D + 2);  // floats per state
  const int par = static_cast<int>(step & 1u);

  // ---- push: CTA j copies the state into rank j's slot [par][rank] (when the
  // decode kernel did not publish it per unit already)
  for (int j = blockIdx.x; j < p.world && p.units == 0; j += gridDim.x) {
    float* dst = reinterpret_cast<float*>(static_cast<uint32_t*>(p.bufs[j]) + peer_data_word(p.B, p.H)) +
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

  // ---- wait (bounded; none on a failed exchange) for the states of this step:
  // whole states, every rank's flag before any item; published states, the
  // flags of an item's (sequence, KV head) unit before that item, so items
  // merge while other units are still being published
  auto wait_flags = [&](int n, int unit) {
    for (int k = threadIdx.x; k < n && !s_failed; k += kPeerThreads) {
      const uint32_t* flag =
          unit >= 0 ? own + peer_unit_flag_word(k, unit, p.B, p.H) : own + flag_word(k);
      const long long t0 = clock64();
      while (static_cast<int>(ld_acquire_sys(flag) - step) < 0) {
        if (kPollSleepNs > 0) __nanosleep(kPollSleepNs);
        if (clock64() - t0 > p.budget) {
          s_failed = 1;
          atomicOr(own + kFailedWord, 1u);
          atomicOr(p.err, kErrPeerTimeout);
          break;
        }
      }
    }
    __syncthreads();
  };
  if (p.units == 0) wait_flags(p.world, -1);
  if (s_failed && threadIdx.x == 0) atomicOr(p.err, kErrPeerTimeout);  // (again, on a failed exchange)

  // ---- merge: CTA c takes (sequence, head) items c, c + grid, ...
  const float* data = reinterpret_cast<const float*>(own + peer_data_word(p.B, p.H)) +
                      static_cast<long long>(par) * p.world * blk;
  const long long hd = static_cast<long long>(p.H) * p.D;
  for (int item = blockIdx.x; item < p.B * p.H; item += gridDim.x) {
    const int b = item / p.H, h = item % p.H;
    const float* base = data + static_cast<long long>(b) * p.H * (p.D + 2);
    if (p.units > 0) wait_flags(p.world, b * (p.units / p.B) + h / (p.H / (p.units / p.B)));
    if (s_failed) {  // no complete set of states: NaN, never stale slots
      for (int d = threadIdx.x; d < p.D; d += kPeerThreads)
        store_from_float(p.out, (static_cast<long long>(b) * p.H + h) * p.D + d, p.out_dtype, NAN);
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

  // ---- the last CTA to finish advances this rank's step counter (every CTA
  // read it at its start, before any CTA could finish)
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned done = atomicAdd(own + kGridCounter, 1u);
    if (done == gridDim.x - 1) {
      own[kGridCounter] = 0u;
      // a failed exchange keeps its step: it is out of step with the others for good
      if (*reinterpret_cast<volatile uint32_t*>(own + kFailedWord) == 0u)
        *reinterpret_cast<volatile uint32_t*>(own) = step;
    }
  }
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
  return static_cast<size_t>(peer_data_word(batch, num_heads)) * sizeof(uint32_t) +
         state_floats(world, batch, num_heads, head_dim) * sizeof(float);
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
                             int batch, int num_heads, int head_dim, int units, void* out,
                             tq_dtype out_dtype, int timeout_us, void* stream);

TQ_API int tq_peer_merge(const float* part, void* const* peer_bufs, int world, int rank,
                         int batch, int num_heads, int head_dim, void* out, tq_dtype out_dtype,
                         int timeout_us, void* stream) {
  if (!part) {
    set_last_error("tq_peer_merge: null pointer");
    return TQ_ERR_INVALID;
  }
  return peer_merge_common(part, peer_bufs, world, rank, batch, num_heads, head_dim, 0, out,
                           out_dtype, timeout_us, stream);
}

TQ_API int tq_peer_merge_published(void* const* peer_bufs, int world, int rank, int batch,
                                   int num_heads, int num_kv_heads, int head_dim, void* out,
                                   tq_dtype out_dtype, int timeout_us, void* stream) {
  if (num_kv_heads < 1 || num_heads % num_kv_heads != 0 || batch < 1) {
    set_last_error("tq_peer_merge_published: bad sizes");
    return TQ_ERR_INVALID;
  }
  return peer_merge_common(nullptr, peer_bufs, world, rank, batch, num_heads, head_dim,
                           batch * num_kv_heads, out, out_dtype, timeout_us, stream);
}

static int peer_merge_common(const float* part, void* const* peer_bufs, int world, int rank,
                             int batch, int num_heads, int head_dim, int units, void* out,
                             tq_dtype out_dtype, int timeout_us, void* stream) {
  if (!peer_bufs || !out) {
    set_last_error("tq_peer_merge: null pointer");
    return TQ_ERR_INVALID;
  }
  if (world < 1 || world > kMaxWorld || rank < 0 || rank >= world || batch < 1 || num_heads < 1 ||
      head_dim < 1 || timeout_us < 1) {
    set_last_error("tq_peer_merge: bad sizes");
    return TQ_ERR_INVALID;
  }
  if (part && (reinterpret_cast<uintptr_t>(part) & 15u)) {
    set_last_error("tq_peer_merge: part must be 16-byte aligned");
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
  p.units = units;
  int grid = batch * num_heads;
  if (grid < world) grid = world;
  if (grid > 148) grid = 148;
  cudaError_t e;
  if (units > 0 && kPublishedMergePdl) {
    // published states: nothing of the preceding decode kernel is read
    // without a flag, so the merge may start once that kernel's CTAs have all
    // started and merge each unit as soon as its flags are up
    e = launch_pdl(peer_merge_kernel, dim3(grid), dim3(kPeerThreads), 0,
                   static_cast<cudaStream_t>(stream), p);
  } else {
    peer_merge_kernel<<<grid, kPeerThreads, 0, static_cast<cudaStream_t>(stream)>>>(p);
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) {
    set_last_error("tq_peer_merge: %s", cudaGetErrorString(e));
    return TQ_ERR_CUDA;
  }
  return TQ_OK;
}

}  // extern "C"
