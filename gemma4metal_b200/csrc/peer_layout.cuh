// Layout of a sequence-split exchange buffer (one per rank, shared with the
// other ranks through CUDA IPC), used by the peer-merge kernels
// (peer_merge.cu) and by the decode kernel when it publishes its partial
// state straight into the buffers (sdpa_decode_mma.cu).
//
//   header (32-bit words): [0] this rank's step counter; [32 * (1 + k)] the
//          step rank k last pushed as a whole state (one 128 B line per
//          rank); [32 * 65] grid counter; [32 * 65 + 16] failed word
//   unit flags: the step at which rank k published unit u (a (sequence, KV
//          head) slice of the state), at kPeerHeaderWords + k * B * H + u
//   data: [2 step parities][world][B * H * (D + 2)] fp32 states in the
//          layout of tq_sdpa_int4_partial (o (H, D) then (m, l) per head)
#pragma once

#include <stdint.h>

namespace tq {

constexpr int kPeerHeaderWords = 32 * 66;
constexpr int kPeerGridCounter = 32 * 65;
constexpr int kPeerFailedWord = 32 * 65 + 16;  // nonzero once a wait of this rank timed out
constexpr int kPeerMaxWorld = 64;

__host__ __device__ __forceinline__ int peer_flag_word(int k) { return 32 * (1 + k); }

__host__ __device__ __forceinline__ long long peer_unit_flag_word(int k, int u, int B, int H) {
  return kPeerHeaderWords + static_cast<long long>(k) * B * H + u;
}

// First word of the state data (16-byte aligned).
__host__ __device__ __forceinline__ long long peer_data_word(int B, int H) {
  const long long w = kPeerHeaderWords + static_cast<long long>(kPeerMaxWorld) * B * H;
  return (w + 3) & ~3LL;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

}  // namespace tq
