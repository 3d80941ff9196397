// Device helpers shared by the sm_100a kernels: dtype loads/stores, the int4
// unpack, and the mbarrier / bulk-copy (TMA, non-tensor) primitives.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace tq {

enum Dtype : int { kF32 = 0, kF16 = 1, kBF16 = 2 };

// Error codes written to the device error word (see tq_device_error).
enum DeviceError : uint32_t { kErrNone = 0, kErrBarrierTimeout = 1u, kErrPeerTimeout = 2u };

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

__device__ __forceinline__ float load_as_float(const void* p, long long i, int dtype) {
  if (dtype == kF16) return __half2float(reinterpret_cast<const __half*>(p)[i]);
  if (dtype == kBF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  return reinterpret_cast<const float*>(p)[i];
}

__device__ __forceinline__ void store_from_float(void* p, long long i, int dtype, float v) {
  if (dtype == kF16) {
    reinterpret_cast<__half*>(p)[i] = __float2half_rn(v);
  } else if (dtype == kBF16) {
    reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  } else {
    reinterpret_cast<float*>(p)[i] = v;
  }
}

// Scale/bias element types of the cache.
template <typename SB>
__device__ __forceinline__ float sb_to_float(SB v);
template <>
__device__ __forceinline__ float sb_to_float<float>(float v) { return v; }
template <>
__device__ __forceinline__ float sb_to_float<__half>(__half v) { return __half2float(v); }

// ---- int4 unpack without integer->float conversion instructions ------------
// Nibble j of a word is OR-ed into the mantissa of 2^23 at its own bit
// position (j <= 4) or, for j = 5..7, from the word shifted right by 12, so
// the float equals 2^23 + c * 2^e(j) exactly; subtracting 2^23 (packed
// fp32x2 add) leaves c * 2^e(j), e(j) = {0,4,8,12,16,8,12,16}. Dot products
// use q_d * 2^-e(d) (exact power-of-two rescale), V sums are rescaled by
// 2^-e(d) once at the end, so the result is the exact integer code path.
constexpr uint32_t kMagic = 0x4B000000u;  // 2^23
__host__ __device__ constexpr int nib_exp(int j) { return j <= 4 ? 4 * j : 4 * (j - 3); }

__device__ __forceinline__ void unpack_word(uint32_t w, float2 (&c)[4]) {
  const uint32_t hi = w >> 12;
  const float2 m = make_float2(-8388608.0f, -8388608.0f);
  c[0] = __fadd2_rn(make_float2(__uint_as_float(kMagic | (w & 0xFu)),
                                __uint_as_float(kMagic | (w & 0xF0u))), m);
  c[1] = __fadd2_rn(make_float2(__uint_as_float(kMagic | (w & 0xF00u)),
                                __uint_as_float(kMagic | (w & 0xF000u))), m);
  c[2] = __fadd2_rn(make_float2(__uint_as_float(kMagic | (w & 0xF0000u)),
                                __uint_as_float(kMagic | (hi & 0xF00u))), m);
  c[3] = __fadd2_rn(make_float2(__uint_as_float(kMagic | (hi & 0xF000u)),
                                __uint_as_float(kMagic | (hi & 0xF0000u))), m);
}

// ---- shared-memory address + mbarrier + bulk async copy --------------------
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

// Plain arrival (release at CTA scope) on a shared-memory mbarrier.
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// try_wait blocks for a hardware-chosen interval while the phase is
// incomplete (no suspend-time hint: the default interval measured faster
// here than a long hint), so a waiting warp does not spin on the issue slots.
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Bounded wait: gives up after ~`budget_cycles` SM clocks, records
// kErrBarrierTimeout in the device error word and returns false. Callers keep
// running (on stale shared memory) so the kernel always terminates; the host
// reads the error word through tq_device_error().
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, uint32_t* err,
                                                  long long budget_cycles = 4000000000LL) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long start = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - start > budget_cycles) {
      if (err) atomicOr(err, kErrBarrierTimeout);
      return false;
    }
  }
  return true;
}

// cp.async.bulk global -> shared (1-D, non-tensor TMA), completion counted on
// `bar` in bytes. dst/src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1], %2, [%3], %4;" ::"r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

// Bulk prefetch of [src, src + bytes) into L2 (16-byte aligned, bytes a
// multiple of 16). Only warms the cache: it reads nothing into the kernel.
__device__ __forceinline__ void prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// L2 eviction-priority policy for data that is streamed once per step.
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// L2 priority for data that many CTAs read (kept over streamed data).
__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// Prefetch a TMA descriptor (kernel parameter) so the first copy does not wait for it.
__device__ __forceinline__ void prefetch_tensormap(const void* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Programmatic dependent launch. pdl_wait blocks until the kernels this grid
// depends on (launched before it on the stream) have completed and their
// writes are visible; without the launch attribute it returns at once.
// pdl_trigger lets the next kernel on the stream start launching (its CTAs
// then wait in their own pdl_wait), which hides its launch latency behind
// this kernel's tail.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Atomic add with acquire-release semantics at GPU scope (a split-merge ticket:
// releases this CTA's partials, acquires the other CTAs').
__device__ __forceinline__ unsigned atomic_add_acq_rel(unsigned* p, unsigned v) {
  unsigned old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 8 consecutive elements [i, i + 8) of a 16-byte aligned row as float.
__device__ __forceinline__ void load8_aligned(const void* p, long long i, int dtype, float (&v)[8]) {
  if (dtype == kF16) {
    const uint4 raw = *reinterpret_cast<const uint4*>(reinterpret_cast<const __half*>(p) + i);
    const __half2* h = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 f = __half22float2(h[k]);
      v[2 * k] = f.x;
      v[2 * k + 1] = f.y;
    }
  } else if (dtype == kBF16) {
    const uint4 raw =
        *reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(p) + i);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 f = __bfloat1622float2(h[k]);
      v[2 * k] = f.x;
      v[2 * k + 1] = f.y;
    }
  } else {
    const float4 a = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p) + i);
    const float4 b = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p) + i + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
}

// Orders this thread's generic-proxy global writes before later async-proxy
// accesses (TMA / bulk copies) of the same data.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// ---- MLX affine group-64 4-bit quantization (mlx quantize(x, 64, 4)) ----------
// A lane holds 8 consecutive values of a row (one packed word); the 8 lanes
// 8k..8k+7 of a warp hold one 64-value group. All arithmetic is IEEE
// round-to-nearest (explicit __fsub_rn/__fdiv_rn, rintf = ties-to-even), so
// the codes, scales and biases are bit-identical to the CPU oracle.

// Group min/max over the 8 lanes of the group (warp-collective: all 32 lanes).
__device__ __forceinline__ void group_minmax8(const float (&v)[8], float& mn, float& mx) {
  mn = v[0];
  mx = v[0];
#pragma unroll
  for (int j = 1; j < 8; ++j) {
    mn = fminf(mn, v[j]);
    mx = fmaxf(mx, v[j]);
  }
#pragma unroll
  for (int o = 1; o < 8; o <<= 1) {
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  }
}

// Round to the scale/bias storage type, store (if write), and return the value
// read back.
__device__ __forceinline__ float round_store(float v, int dtype, void* dst, long long i,
                                             bool write) {
  if (dtype == kF16) {
    const __half h = __float2half_rn(v);
    if (write) reinterpret_cast<__half*>(dst)[i] = h;
    return __half2float(h);
  }
  if (dtype == kBF16) {
    const __nv_bfloat16 h = __float2bfloat16_rn(v);
    if (write) reinterpret_cast<__nv_bfloat16*>(dst)[i] = h;
    return __bfloat162float(h);
  }
  if (write) reinterpret_cast<float*>(dst)[i] = v;
  return v;
}

// Scale = (max - min) / 15 and bias = min, rounded to the storage type and
// written at sidx by the group's leader; returns the packed word of the 8
// codes round((x - bias) / scale) clamped to 0..15, low nibble first (all
// zero when the scale is zero).
__device__ __forceinline__ uint32_t quantize_word8(const float (&v)[8], float mn, float mx,
                                                   int sb_dtype, void* scales, void* biases,
                                                   long long sidx, bool leader) {
  const float scale_f = __fdiv_rn(__fsub_rn(mx, mn), 15.0f);
  const float s = round_store(scale_f, sb_dtype, scales, sidx, leader);
  const float bb = round_store(mn, sb_dtype, biases, sidx, leader);
  uint32_t packed = 0;
  if (s != 0.0f) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float c = rintf(__fdiv_rn(__fsub_rn(v[j], bb), s));
      c = fminf(fmaxf(c, 0.0f), 15.0f);
      packed |= static_cast<uint32_t>(c) << (4 * j);
    }
  }
  return packed;
}

}  // namespace tq
