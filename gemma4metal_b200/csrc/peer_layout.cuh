// Layout of a sequence-split exchange buffer (one per rank, shared with the
// other ranks through CUDA IPC), used by the peer-merge kernels
// (peer_merge.cu) and by the decode kernel when it publishes its partial
// state straight into the buffers (sdpa_decode_mma.cu).
//
//   header (32-bit words): [0] this rank's step counter; [32 * (1 + k)] the
//          step rank k last pushed as a whole state (one 128 B line per
//          rank); [32 * 65] grid counter; [32 * 65 + 16] failed word
//   data:  whole states (tq_peer_merge): [2 step parities][world][B * H * (D + 2)]
//          fp32 in the layout of tq_sdpa_int4_partial (o (H, D), then (m, l)
//          per head), released by the per-rank flags above;
//          published states (tq_sdpa_int4_partial_publish): the same index
//          space, but every value is an 8-byte pair {fp32 bits, step} written
//          by one store, so a reader knows a value is this step's from the
//          pair alone (no fence or flag; the scheme of NCCL's LL protocol).
//          Either use makes the data region twice the fp32 state size.
#pragma once

#include <stdint.h>

namespace tq {

constexpr int kPeerHeaderWords = 32 * 66;
constexpr int kPeerGridCounter = 32 * 65;
constexpr int kPeerFailedWord = 32 * 65 + 16;  // nonzero once a wait of this rank timed out
constexpr int kPeerMaxWorld = 64;

__host__ __device__ __forceinline__ int peer_flag_word(int k) { return 32 * (1 + k); }

// First word of the state data (16-byte aligned).
__host__ __device__ __forceinline__ long long peer_data_word() { return kPeerHeaderWords; }
static_assert(kPeerHeaderWords % 4 == 0, "state data must start 16-byte aligned");

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// {value, step} pairs: one 8-byte (or two in one 16-byte) volatile access, so
// each pair is read or written whole.
__device__ __forceinline__ void st_pair(void* p, float v, uint32_t step) {
  asm volatile("st.volatile.global.v2.u32 [%0], {%1, %2};" ::"l"(p), "r"(__float_as_uint(v)),
               "r"(step)
               : "memory");
}

__device__ __forceinline__ void st_pair2(void* p, float v0, float v1, uint32_t step) {
  asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p),
               "r"(__float_as_uint(v0)), "r"(step), "r"(__float_as_uint(v1)), "r"(step)
               : "memory");
}

__device__ __forceinline__ uint2 ld_pair(const void* p) {
  uint2 v;
  asm volatile("ld.volatile.global.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p) : "memory");
  return v;
}

}  // namespace tq
