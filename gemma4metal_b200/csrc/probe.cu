// tq_read_probe: a read-only HBM stream, the practical ceiling the decode
// kernels are measured against (a plain copy reads and writes, so its figure
// understates what a pure read stream reaches).
//
// Each of `ctas` CTAs reads one contiguous range of [src, src + bytes):
//   mode 0 -- one thread issues 1-D bulk copies (cp.async.bulk, the decode
//             kernel's own load path) of 16 KB chunks into a 4-stage
//             shared-memory ring, four consumer warps read every stage and
//             release it (the decode kernel's pipeline without the math);
//   mode 1 -- every thread issues 16-byte non-caching loads, eight in flight.
// The XOR of everything read goes to sink[cta] (XOR-accumulated across
// launches), so no load can be dropped.
#include "../../include/turboquant_c.h"
#include "tq_common.cuh"
#include "tq_internal.h"

namespace tq {
namespace {

constexpr int kProbeChunk = 16384;
constexpr int kProbeStages = 4;
constexpr int kProbeConsumers = 4;  // warps
constexpr int kProbeBulkThreads = (kProbeConsumers + 1) * 32;
constexpr int kProbeBulkSmem = kProbeStages * kProbeChunk + 2 * kProbeStages * 8 + 128;
constexpr int kProbeLdgThreads = 512;

__global__ void __launch_bounds__(kProbeBulkThreads)
    read_probe_bulk_kernel(const unsigned char* src, long long bytes, long long per_cta,
                           uint32_t* sink, uint32_t* err) {
  extern __shared__ __align__(128) unsigned char smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kProbeStages * kProbeChunk);
  uint64_t* empty = full + kProbeStages;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const long long begin = static_cast<long long>(blockIdx.x) * per_cta;
  const long long end = min(bytes, begin + per_cta);
  const int nchunks = end > begin ? static_cast<int>((end - begin + kProbeChunk - 1) / kProbeChunk) : 0;
  if (tid == 0) {
    for (int s = 0; s < kProbeStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kProbeConsumers);
    }
    fence_barrier_init();
  }
  __syncthreads();
  if (warp == kProbeConsumers) {
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      int st = 0;
      uint32_t par = 0;
      for (int i = 0; i < nchunks; ++i) {
        if (i >= kProbeStages) mbar_wait_bounded(&empty[st], par ^ 1u, err);
        const long long off = begin + static_cast<long long>(i) * kProbeChunk;
        const uint32_t n = static_cast<uint32_t>(min(static_cast<long long>(kProbeChunk), end - off));
        mbar_arrive_expect_tx(&full[st], n);
        bulk_g2s(smem + st * kProbeChunk, src + off, n, &full[st], pol);
        if (++st == kProbeStages) {
          st = 0;
          par ^= 1u;
        }
      }
    }
    return;
  }
  uint32_t acc = 0;
  int st = 0;
  uint32_t par = 0;
  for (int i = 0; i < nchunks; ++i) {
    mbar_wait_bounded(&full[st], par, err);
    const long long off = begin + static_cast<long long>(i) * kProbeChunk;
    const int n = static_cast<int>(min(static_cast<long long>(kProbeChunk), end - off));
    const uint4* w = reinterpret_cast<const uint4*>(smem + st * kProbeChunk);
    for (int j = tid; j < n / 16; j += kProbeConsumers * 32) {
      const uint4 v = w[j];
      acc ^= v.x ^ v.y ^ v.z ^ v.w;
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);
    if (++st == kProbeStages) {
      st = 0;
      par ^= 1u;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc ^= __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) atomicXor(&sink[blockIdx.x], acc);
}

__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__global__ void __launch_bounds__(kProbeLdgThreads)
    read_probe_ldg_kernel(const unsigned char* src, long long bytes, long long per_cta,
                          uint32_t* sink) {
  const long long begin = static_cast<long long>(blockIdx.x) * per_cta;
  const long long end = min(bytes, begin + per_cta);
  constexpr int U = 8;
  constexpr long long kStep = static_cast<long long>(kProbeLdgThreads) * 16;
  uint32_t acc = 0;
  long long off = begin + threadIdx.x * 16;
  for (; off + (U - 1) * kStep < end; off += U * kStep) {
    uint4 v[U];
#pragma unroll
    for (int u = 0; u < U; ++u) v[u] = ldg_stream(src + off + u * kStep);
#pragma unroll
    for (int u = 0; u < U; ++u) acc ^= v[u].x ^ v[u].y ^ v[u].z ^ v[u].w;
  }
  for (; off < end; off += kStep) {
    const uint4 v = ldg_stream(src + off);
    acc ^= v.x ^ v.y ^ v.z ^ v.w;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc ^= __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) atomicXor(&sink[blockIdx.x], acc);
}

}  // namespace
}  // namespace tq

extern "C" TQ_API int tq_read_probe(const void* src, size_t bytes, int ctas, int mode,
                                    uint32_t* sink, void* stream) {
  if (!src || !sink || ctas < 1 || bytes == 0 || (bytes & 15u) != 0 ||
      (reinterpret_cast<uintptr_t>(src) & 15u) != 0 || (mode != 0 && mode != 1)) {
    tq::set_last_error("tq_read_probe: need src 16-byte aligned, bytes a positive multiple of 16, "
                       "ctas >= 1, mode 0 or 1 and a sink of ctas words");
    return TQ_ERR_INVALID;
  }
  const long long per = ((static_cast<long long>(bytes) + ctas - 1) / ctas + 15) / 16 * 16;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (mode == 0) {
    // per device (the attribute belongs to the current context); cheap enough per call
    cudaFuncSetAttribute(tq::read_probe_bulk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         tq::kProbeBulkSmem);
    tq::read_probe_bulk_kernel<<<ctas, tq::kProbeBulkThreads, tq::kProbeBulkSmem, s>>>(
        static_cast<const unsigned char*>(src), static_cast<long long>(bytes), per, sink,
        tq::device_error_word());
  } else {
    tq::read_probe_ldg_kernel<<<ctas, tq::kProbeLdgThreads, 0, s>>>(
        static_cast<const unsigned char*>(src), static_cast<long long>(bytes), per, sink);
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    tq::set_last_error("tq_read_probe launch: %s", cudaGetErrorString(e));
    return TQ_ERR_CUDA;
  }
  return TQ_OK;
}
