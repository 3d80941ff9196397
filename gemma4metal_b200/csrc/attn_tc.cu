// Tensor-core (tcgen05 + TMEM) int4 attention for many query rows per KV
// head: the batched-decode case (B sequences x 1 query against one shared
// cache) and the causal prefill chunk (n_q queries at positions pos0.. of one
// sequence). The reference runs both through MLX dequantize + fast::sdpa with
// a CPU-built mask (engine/gemma4_multilayer.cpp:307-308,347-367,441-464).
//
// CTA = 128 query rows of one KV head (row = (query, GQA head) pair; TMEM lane
// = row), one CTA per SM, warp-specialized, tiles of 64 tokens:
//   * unpack warps (2 for K, 2 for V, one token per thread) turn the int4
//     codes into exact fp16 in shared memory: K as 1 + c/64 (UMMA canonical
//     K-major, 128B swizzle, one 8 KB region per 64-dim scale group), V as
//     (c - 8)/64 (MN-major); per-token score terms and value terms go beside
//     them. K and V have two stages each, with separate lifetimes (K(i) is
//     free once the softmax of tile i is done, V(i) once PV(i) is), each
//     paced by its own warps, and the next tile's codes wait in registers.
//   * the MMA warp (one thread) issues S'_g = Q_g K_g'^T for tile i into one of
//     two TMEM S buffers, then PV for tile i-1 into the TMEM O accumulator,
//     committing each group to an mbarrier -- the tensor pipe works on the
//     next tile's scores while the softmax finishes the current one.
//   * softmax warps (8, two threads per row on the two 32-token halves of a
//     tile) read S' (tcgen05.ld) and form
//       score = 64 s_0 S'_0 + 64 s_1 S'_1 + (b_0 - 64 s_0) sum q_0 + (b_1 - 64 s_1) sum q_1 - m
//     (the int4 scale/bias factored out of the dot product, as
//     lib/turboquant.metal:803 does; the running max m folded into the FMA
//     chain), mask only tiles that cross a boundary, exchange the half-row
//     max, and write P'_g = fp16(p s_g(token)) (K-major A operand) while
//     accumulating the bias term sum p (b_g + 8 s_g) in fp32.
// out_g = (64 O'_g + bias term_g) / l: the weights' fp16 rounding error is
// multiplied by c - 8 (|c - 8| <= 8), not by the code's full value. The
// running max moves (and O is rescaled in TMEM) only when a row's max grows by
// more than 8 in log2 units. The 8-element dim order inside each code word
// follows the unpack (d = 0,4,1,5,2,6,3,7), applied to Q as well and undone
// when O is written. Splits over the cache (when row tiles alone leave SMs
// idle) write column-major partials merged by attn_tc_merge_kernel.
#include <cuda.h>

#include <cstdint>

#include "../../include/turboquant_c.h"
#include "tq_common.cuh"
#include "tq_internal.h"

namespace tq {
namespace {

constexpr int kRows = 128;     // query rows per CTA (TMEM lanes)
constexpr int kTok = 64;       // tokens per tile
constexpr int kD = 128;        // head_dim (two 64-dim scale groups)
// warp roles: warp 0 issues the MMAs (and owns TMEM); warps 1-2 unpack the K
// codes and warps 3-4 the V codes (one token per thread); warps 5-12 run the
// softmax, two threads per query row (warp % 4 is the TMEM lane quarter a
// warp may access, so each quarter has one warp per half). A warp runs on
// sub-partition warp % 4, so every sub-partition holds two softmax warps and
// one unpack warp: with two unpack warps (K and V work each), the softmax
// warps sharing their sub-partitions finished each tile 20% after the others
// and set the tile period (prefill 251 -> 232 us with four). 13 warps = 4 on
// one sub-partition, which caps registers at 128 per thread. (Four threads
// per row, 19 warps at 96 registers, measured slower: more per-thread fixed
// cost per tile.)
constexpr int kMmaWarp = 0;
constexpr int kUnpackBase = 1, kUnpackWarps = 4;
constexpr int kSoftmaxWarps = 8;
constexpr int kSoftmaxBase = (kUnpackBase + kUnpackWarps) * 32;
constexpr int kSoftmaxThreads = kSoftmaxWarps * 32;
constexpr int kThreads = kSoftmaxBase + kSoftmaxThreads;  // 416
constexpr int kTmemCols = 512; // S[0], S[1] (2 groups x 64 tokens each), O (2 groups x 64 dims)
// an MMA group finishes in microseconds; give up (and record the error) after
// ~10 ms of SM clocks so a wait that cannot complete still ends the kernel
constexpr long long kWaitBudget = 20000000LL;

struct TLayout {
  static constexpr int KVB = 2 * 2 * kTok * 128;  // one K/V stage: K [2 groups][64][128 B] + V, 32 KB
  static constexpr int Q = 0;                     // [2 groups][128 rows][128 B]  32 KB
  static constexpr int K = Q + 2 * kRows * 128;   // stage b at K + b * KVB
  static constexpr int V = K + 2 * kTok * 128;    // stage b at V + b * KVB
  static constexpr int PB = 2 * kRows * 128;      // one P buffer [2 groups][128 rows][128 B], 32 KB
  static constexpr int P = K + 2 * KVB;           // buffer b at P + b * PB
  static constexpr int TS = P + 2 * PB;           // [2][64 tokens] {A0, A1, B0, B1} (score terms)
  static constexpr int TV = TS + 2 * kTok * 16;   // [2][64] {vs0, vs1, vb0 + 8 vs0, vb1 + 8 vs1}
  static constexpr int MX = TV + 2 * kTok * 16;   // [2 tiles][2 halves][128 rows] maxima (q sums first)
  static constexpr int RED = MX + 2 * kSoftmaxThreads * 4;  // [3][2][128] epilogue sums
  static constexpr int BAR = RED + 3 * kSoftmaxThreads * 4; // 12 mbarriers
  static constexpr int TMEM = BAR + 12 * 8;                 // allocated TMEM base address
  static constexpr int BYTES = TMEM + 16 + 1024;            // + alignment slack
  // f32 queries: Q = hi + lo, both fp16; the lo part follows (32 KB)
  static constexpr int QL = (TMEM + 16 + 1023) / 1024 * 1024;
  static constexpr int BYTES_QLO = QL + 2 * kRows * 128 + 1024;
};
static_assert(TLayout::P % 1024 == 0 && TLayout::K % 1024 == 0, "UMMA operands need 1 KB alignment");

struct TCParams {
  const void* q;       // (n_q, H, D) for prefill; (B, H, D) for batched decode
  int q_dtype;
  const uint32_t* kq;  // (Hkv, cap, D/8)
  const void* ks;
  const void* kb;
  const uint32_t* vq;
  const void* vs;
  const void* vb;
  int sb_f32;
  int H, Hkv, G;
  int n_q;             // query rows per KV head = n_q * G
  int n_tokens;        // visible cache length (all queries)
  int capacity;
  int causal;          // 1: query i at position pos0 + i sees tokens t <= pos0 + i
  int pos0;
  int window;          // > 0: and pos - t < window
  float qscale;        // scale * log2(e)
  int splits, tiles_per_split;
  void* out;           // (n_q, H, D)
  int out_dtype;
  float* ws;           // split partials: (units, splits, D + 2, 128 rows)
  uint32_t* err;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// UMMA shared-memory descriptor, 128B swizzle, SBO = 1024 B (8 rows of 128 B).
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((1024u >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1u) << 46;  // descriptor version (sm_100)
  d |= static_cast<uint64_t>(2u) << 61;  // SWIZZLE_128B
  return d;
}

// Instruction descriptor: kind::f16, fp16 A/B, fp32 D, M = 128, N = 64.
__host__ __device__ constexpr uint32_t idesc_f16(bool b_mn_major) {
  return (1u << 4)                               // D format f32
         | (0u << 7) | (0u << 10)                // A, B format f16
         | (0u << 15)                            // A K-major
         | ((b_mn_major ? 1u : 0u) << 16)        // B major
         | ((64u >> 3) << 17)                    // N
         | ((128u >> 4) << 24);                  // M
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(tmem_d), "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// 32 consecutive fp32 TMEM columns of this thread's lane
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// tcgen05.ld of 32 columns without the wait: the registers are valid only
// after tmem_wait_ld(), and reg_fence() keeps their uses behind it
__device__ __forceinline__ void tmem_ld32_raw(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void reg_fence(uint32_t (&r)[N]) {
#pragma unroll
  for (int i = 0; i < N; ++i) asm volatile("" : "+r"(r[i]));
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
      "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
      "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// byte offset of 16-byte chunk `ch` of row `r` in a 128B-swizzled region
__device__ __forceinline__ uint32_t sw128(int r, int ch) {
  return static_cast<uint32_t>(r * 128 + ((ch ^ (r & 7)) << 4));
}

// nibbles j and j+4 of x -> fp16x2 1 + c/64 (see the decode kernel's nib64)
template <int J>
__device__ __forceinline__ uint32_t nib64h(uint32_t x) {
  const uint32_t s = (J == 0) ? (x << 4) : (J == 1) ? x : (J == 2) ? (x >> 4) : (x >> 8);
  return (s & 0x00F000F0u) | 0x3C003C00u;
}

// dim held by element e (0..7) of a word's unpacked chunk: 0,4,1,5,2,6,3,7
__device__ __forceinline__ int perm8(int e) { return (e >> 1) + 4 * (e & 1); }

// fp16x2 (1 + c/64) -> (c - 8)/64; exact (both operands and the result are
// multiples of 2^-6 below 2). 0x3C80 is fp16 1.125 (a literal: a runtime
// conversion would cost an XU-pipe instruction per call).
__device__ __forceinline__ uint32_t center8(uint32_t x) {
  const uint32_t k = 0x3C803C80u;
  __half2 h = *reinterpret_cast<const __half2*>(&x);
  h = __hsub2(h, *reinterpret_cast<const __half2*>(&k));
  return *reinterpret_cast<const uint32_t*>(&h);
}

// 8 consecutive elements [i, i + 8) as float; vec: 16-byte aligned base
__device__ __forceinline__ void load8(const void* p, long long i, int dtype, bool vec, float (&v)[8]) {
  if (vec && dtype != kF32) {
    load8_aligned(p, i, dtype, v);
  } else {
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] = load_as_float(p, i + k, dtype);
  }
}

// 8 consecutive elements [i, i + 8) from float; vec: 16-byte aligned base
__device__ __forceinline__ void store8(void* p, long long i, int dtype, bool vec, const float (&v)[8]) {
  if (vec && dtype != kF32) {
    uint32_t w[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      if (dtype == kF16) {
        const __half2 h = __floats2half2_rn(v[2 * k], v[2 * k + 1]);
        w[k] = *reinterpret_cast<const uint32_t*>(&h);
      } else {
        const __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * k], v[2 * k + 1]);
        w[k] = *reinterpret_cast<const uint32_t*>(&h);
      }
    }
    *reinterpret_cast<uint4*>(static_cast<unsigned short*>(p) + i) = make_uint4(w[0], w[1], w[2], w[3]);
  } else {
#pragma unroll
    for (int k = 0; k < 8; ++k) store_from_float(p, i + k, dtype, v[k]);
  }
}

// Paired fp32 arithmetic (fma/mul/add .rn.f32x2: two IEEE fp32 operations per
// instruction, each rounded exactly as the scalar one): the softmax works on
// two tokens at a time.
__device__ __forceinline__ unsigned long long pk2(float2 v) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(v.x), "f"(v.y));
  return r;
}
__device__ __forceinline__ float2 upk2(unsigned long long r) {
  float2 v;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(v.x), "=f"(v.y) : "l"(r));
  return v;
}
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
  unsigned long long d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(pk2(a)), "l"(pk2(b)), "l"(pk2(c)));
  return upk2(d);
}
__device__ __forceinline__ float2 mul2(float2 a, float2 b) {
  unsigned long long d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(pk2(a)), "l"(pk2(b)));
  return upk2(d);
}
__device__ __forceinline__ float2 add2(float2 a, float2 b) {
  unsigned long long d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(pk2(a)), "l"(pk2(b)));
  return upk2(d);
}

// shared-memory float4 load kept in program order with the tcgen05 loads (a
// plain load may be hoisted above them, which costs registers)
__device__ __forceinline__ float4 lds4(const float4* p) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(static_cast<uint32_t>(__cvta_generic_to_shared(p))));
  return v;
}

// Per-token terms {x, y, z, w} of a tile stored pair-interleaved: tokens 2u
// and 2u + 1 share 8 floats {x_2u, x_2u+1, y_2u, y_2u+1, z.., z.., w.., w..},
// so one 16-byte load gives two tokens' (x, y) or (z, w) as register pairs.
// Lanes 2u and 2u + 1 (tokens t, t ^ 1 of one warp) swap halves by shuffles
// and each writes one float4.
__device__ __forceinline__ void store_term_pair(unsigned char* base, int tok, int lane, float4 v) {
  const bool odd = (lane & 1) != 0;
  const float r0 = __shfl_xor_sync(0xffffffffu, odd ? v.x : v.z, 1);
  const float r1 = __shfl_xor_sync(0xffffffffu, odd ? v.y : v.w, 1);
  float4* dst = reinterpret_cast<float4*>(base) + 2 * (tok >> 1) + (odd ? 1 : 0);
  *dst = odd ? make_float4(r0, v.z, r1, v.w) : make_float4(v.x, r0, v.y, r1);
}

template <bool kQLo>
__global__ void __launch_bounds__(kThreads, 1) attn_tc_kernel(const TCParams p) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + TLayout::BAR);
  // K and V stages have separate lifetimes: K(i) and the score terms are free
  // once softmax(i) is done (p_full), V(i) and the value terms once PV(i) is
  uint64_t* k_full = bars;       // [2] unpack warps: K codes + score terms in smem
  uint64_t* v_full = bars + 2;   // [2] unpack warps: V codes + value terms in smem
  uint64_t* s_full = bars + 4;   // [2] S MMA done
  uint64_t* s_free = bars + 6;   // [2] softmax warps have read S
  uint64_t* p_full = bars + 8;   // [2] P written (and O rescaled): K stage free
  uint64_t* pv_done = bars + 10; // [2] PV MMA done: P buffer and V stage free
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + TLayout::TMEM);
  const uint32_t sbase = smem_u32(smem);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int split = blockIdx.x, mt = blockIdx.y, kv = blockIdx.z;
  const int rows_total = p.n_q * p.G;

  pdl_wait();
  pdl_trigger();

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(s_tmem)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 0) {
    for (int b = 0; b < 2; ++b) {
      mbar_init(&k_full[b], kUnpackWarps / 2);
      mbar_init(&v_full[b], kUnpackWarps / 2);
      mbar_init(&s_full[b], 1);
      mbar_init(&s_free[b], kSoftmaxWarps);
      mbar_init(&p_full[b], kSoftmaxWarps);
      mbar_init(&pv_done[b], 1);
    }
    fence_barrier_init();
  }

  // ---- token range of this split (tiles of 64 tokens), cut to what the CTA's
  // rows can see: causal rows end at pos0 + last query, windows start at
  // (first row's position) - window + 1
  const int row_last = min(rows_total, (mt + 1) * kRows) - 1;
  const int qpos_lo = p.causal ? p.pos0 + (mt * kRows) / p.G : p.n_tokens - 1;
  const int qpos_hi = p.causal ? p.pos0 + row_last / p.G : p.n_tokens - 1;
  const int n_vis = min(p.n_tokens, qpos_hi + 1);
  const int t_lo = p.window > 0 ? max(0, qpos_lo - p.window + 1) : 0;
  const int t_begin = max(split * p.tiles_per_split * kTok, t_lo);
  const int t_end = min(n_vis, split * p.tiles_per_split * kTok + p.tiles_per_split * kTok);
  const int n_tiles = t_end > t_begin ? (t_end - t_begin + kTok - 1) / kTok : 0;
  const long long tok_base = static_cast<long long>(kv) * p.capacity;

  // ---- softmax threads: (token half hf, row rl); warp % 4 is the TMEM lane
  // quarter a warp may access
  const int sid = tid - kSoftmaxBase;
  const bool is_softmax = sid >= 0;
  const int rl = 32 * (warp & 3) + lane;
  const int hf = is_softmax ? sid / kRows : 0;
  // exchange slot of (half, row): the partner of slot x is x ^ kRows (a
  // warp's threads need not have sid == row: warp % 4 fixes the rows)
  const int xs = hf * kRows + rl;
  const int row = mt * kRows + rl;
  const bool row_ok = row < rows_total;
  const int qi = row_ok ? row / p.G : 0;
  const int h = kv * p.G + (row_ok ? row % p.G : 0);
  // position of the query: causal rows at pos0 + qi; otherwise every query
  // sits at the end of the shared cache (the window counts back from there)
  const int qpos = p.causal ? p.pos0 + qi : p.n_tokens - 1;
  float* s_mx = reinterpret_cast<float*>(smem + TLayout::MX);  // [2 tiles][256]
  if (is_softmax) {
    // Q row, scale group hf -> smem (fp16, dims permuted inside each 8-dim
    // word like the codes; f32 queries as fp16 hi + lo); the group's sum goes
    // to the partner through s_mx
    const long long qb = (static_cast<long long>(qi) * p.H + h) * kD + hf * 64;
    const bool qvec = (reinterpret_cast<uintptr_t>(p.q) & 15u) == 0;
    float qsum = 0.0f;
    // all eight 8-dim chunks are loaded before any is converted and stored,
    // so their global-memory latencies overlap
    float qx[8][8];
#pragma unroll
    for (int ch = 0; ch < 8; ++ch) {
      if (row_ok) {
        load8(p.q, qb + ch * 8, p.q_dtype, qvec, qx[ch]);
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) qx[ch][e] = 0.0f;
      }
    }
#pragma unroll
    for (int ch = 0; ch < 8; ++ch) {
      const float* x = qx[ch];
      // fp16 copies (exact for fp16 and bf16 inputs in range)
      __half2 hh[4], hl[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float xa = x[perm8(2 * e)], xb = x[perm8(2 * e + 1)];
        hh[e] = __floats2half2_rn(xa, xb);
        const float2 f = __half22float2(hh[e]);
        qsum += f.x + f.y;
        if (kQLo) {
          hl[e] = __floats2half2_rn(xa - f.x, xb - f.y);
          const float2 fl = __half22float2(hl[e]);
          qsum += fl.x + fl.y;
        }
      }
      *reinterpret_cast<uint4*>(smem + TLayout::Q + hf * kRows * 128 + sw128(rl, ch)) =
          *reinterpret_cast<uint4*>(hh);
      if (kQLo)
        *reinterpret_cast<uint4*>(smem + TLayout::QL + hf * kRows * 128 + sw128(rl, ch)) =
            *reinterpret_cast<uint4*>(hl);
    }
    s_mx[xs] = qsum;
    fence_async_smem();
  }
  // ---- unpack warps' state: warps 1-2 unpack K (paced by the softmax), warps
  // 3-4 V (paced by PV), thread = token ptok; the codes and scales of the tile
  // being unpacked next wait in registers. The first tile's are requested
  // before the set-up barrier, while the softmax warps stage the queries.
  const bool is_unpack = warp >= kUnpackBase && warp < kUnpackBase + kUnpackWarps;
  const bool vside = warp >= kUnpackBase + kUnpackWarps / 2;
  const int ptok = tid - (kUnpackBase + (vside ? kUnpackWarps / 2 : 0)) * 32;
  uint4 cf[4];
  uint32_t sr[4] = {0u, 0u, 0u, 0u};  // scale, bias (raw: 1 or 2 words each)
  int tcur = t_end;  // the tile held in registers
  auto prefetch = [&](int t0) {
    const int t = t0 + ptok;
    const long long rowi = tok_base + (t < t_end ? t : t0);
    const uint4* cp = reinterpret_cast<const uint4*>((vside ? p.vq : p.kq) + rowi * (kD / 8));
#pragma unroll
    for (int k = 0; k < 4; ++k) cf[k] = cp[k];
    auto load_pair = [&](const void* src, int k) {
      if (p.sb_f32) {
        const uint2 a = reinterpret_cast<const uint2*>(src)[rowi];
        sr[2 * k] = a.x;
        sr[2 * k + 1] = a.y;
      } else {
        sr[2 * k] = reinterpret_cast<const uint32_t*>(src)[rowi];
      }
    };
    load_pair(vside ? p.vs : p.ks, 0);
    load_pair(vside ? p.vb : p.kb, 1);
    tcur = t0;
  };
  if (is_unpack && n_tiles > 0) prefetch(t_begin);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;
  // TMEM columns: S[b] at 128 b (group g at + 64 g), O at 256 (group g at + 64 g)
  const uint32_t t_o = tmem + 256;

  // ======================= MMA warp (one thread issues) =========================
  // S(i) is issued before PV(i-1), so the tensor pipe works on the next tile's
  // scores while the softmax warps still finish the current one.
  if (warp == kMmaWarp) {
    if (lane == 0) {
      constexpr uint32_t idS = idesc_f16(false);
      constexpr uint32_t idO = idesc_f16(true);
      auto issue_pv = [&](int i) {
        const int b = i & 1;
        const uint32_t use = static_cast<uint32_t>(i >> 1);
        mbar_wait_bounded(&v_full[b], use & 1u, p.err, kWaitBudget);
        mbar_wait_bounded(&p_full[b], use & 1u, p.err, kWaitBudget);
        tc_fence_after();
#pragma unroll
        for (int g = 0; g < 2; ++g)
#pragma unroll
          for (int ks = 0; ks < 4; ++ks) {
            const uint64_t a = umma_desc(sbase + TLayout::P + b * TLayout::PB + g * kRows * 128 + ks * 32, 16);
            const uint64_t v = umma_desc(sbase + TLayout::V + b * TLayout::KVB + g * kTok * 128 + ks * 16 * 128, 16);
            umma_f16(t_o + 64 * g, a, v, idO, (i > 0 || ks > 0) ? 1u : 0u);
          }
        umma_commit(&pv_done[b]);
      };
      for (int i = 0; i < n_tiles; ++i) {
        const int b = i & 1;
        const uint32_t use = static_cast<uint32_t>(i >> 1);
        mbar_wait_bounded(&k_full[b], use & 1u, p.err, kWaitBudget);
        if (i >= 2) mbar_wait_bounded(&s_free[b], (use - 1) & 1u, p.err, kWaitBudget);
        tc_fence_after();
        const uint32_t t_s = tmem + 128 * b;
#pragma unroll
        for (int g = 0; g < 2; ++g)
#pragma unroll
          for (int ks = 0; ks < 4; ++ks) {
            const uint64_t kd = umma_desc(sbase + TLayout::K + b * TLayout::KVB + g * kTok * 128 + ks * 32, 16);
            const uint64_t a = umma_desc(sbase + TLayout::Q + g * kRows * 128 + ks * 32, 16);
            umma_f16(t_s + 64 * g, a, kd, idS, ks > 0 ? 1u : 0u);
            if (kQLo) {
              const uint64_t al = umma_desc(sbase + TLayout::QL + g * kRows * 128 + ks * 32, 16);
              umma_f16(t_s + 64 * g, al, kd, idS, 1u);
            }
          }
        umma_commit(&s_full[b]);
        if (i >= 1) issue_pv(i - 1);
      }
      if (n_tiles > 0) issue_pv(n_tiles - 1);
    }
  }

  // ======================= unpack warps =========================================
  // Thread = token ptok: 64 B of K (warps 1-2) or V (warps 3-4) codes per
  // tile (both scale groups), the next tile's held in registers while this
  // one is unpacked; K as exact fp16 1 + c/64 (K-major), V as exact fp16
  // (c - 8)/64 (MN-major), both 128B-swizzled; the token's score or value
  // terms.
  if (is_unpack) {
    auto pair = [&](int k) {
      if (p.sb_f32) return make_float2(__uint_as_float(sr[2 * k]), __uint_as_float(sr[2 * k + 1]));
      return __half22float2(*reinterpret_cast<const __half2*>(&sr[2 * k]));
    };
    auto unpack_codes = [&](uint4 c0, uint4 c1, unsigned char* dst, bool centre) {
      const uint32_t w[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
#pragma unroll
      for (int ch = 0; ch < 8; ++ch) {
        uint4 o;
        o.x = nib64h<0>(w[ch]);
        o.y = nib64h<1>(w[ch]);
        o.z = nib64h<2>(w[ch]);
        o.w = nib64h<3>(w[ch]);
        if (centre) {
          o.x = center8(o.x);
          o.y = center8(o.y);
          o.z = center8(o.z);
          o.w = center8(o.w);
        }
        *reinterpret_cast<uint4*>(dst + sw128(ptok, ch)) = o;
      }
    };
    for (int i = 0; i < n_tiles; ++i) {
      const int b = i & 1;
      const uint32_t use = static_cast<uint32_t>(i >> 1);
      const int t0 = tcur;
      unsigned char* stage = smem + b * TLayout::KVB;
      const bool tv = t0 + ptok < t_end;
      const float2 sc2 = pair(0), bc2 = pair(1);
      const uint4 c0 = cf[0], c1 = cf[1], c2 = cf[2], c3 = cf[3];
      if (!vside) {
        // K(i) and the score terms: the stage is free once softmax(i-2) is done
        if (i >= 2) mbar_wait_bounded(&p_full[b], (use - 1) & 1u, p.err, kWaitBudget);
        if (i + 1 < n_tiles) prefetch(t0 + kTok);
        unpack_codes(c0, c1, stage + TLayout::K, false);
        unpack_codes(c2, c3, stage + TLayout::K + kTok * 128, false);
        const float qs = p.qscale;
        const float4 t4 = tv ? make_float4(64.0f * sc2.x * qs, 64.0f * sc2.y * qs,
                                           (bc2.x - 64.0f * sc2.x) * qs, (bc2.y - 64.0f * sc2.y) * qs)
                             : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        store_term_pair(smem + TLayout::TS + b * kTok * 16, ptok, lane, t4);
        fence_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&k_full[b]);
      } else {
        // V(i) and the value terms: free once PV(i-2) is done
        if (i >= 2) mbar_wait_bounded(&pv_done[b], (use - 1) & 1u, p.err, kWaitBudget);
        if (i + 1 < n_tiles) prefetch(t0 + kTok);
        unpack_codes(c0, c1, stage + TLayout::V, true);
        unpack_codes(c2, c3, stage + TLayout::V + kTok * 128, true);
        const float4 t4 = tv ? make_float4(sc2.x, sc2.y, fmaf(8.0f, sc2.x, bc2.x), fmaf(8.0f, sc2.y, bc2.y))
                             : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        store_term_pair(smem + TLayout::TV + b * kTok * 16, ptok, lane, t4);
        fence_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&v_full[b]);
      }
    }
  }

  // ======================= softmax warps ========================================
  if (is_softmax) {
    const float qsum0 = s_mx[rl], qsum1 = s_mx[rl + kRows];
    const float2 qs0p = make_float2(qsum0, qsum0), qs1p = make_float2(qsum1, qsum1);
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    // the two threads of a row meet on named barrier 1 + warp % 4 (64 threads)
    auto pair_sync = [&]() { asm volatile("bar.sync %0, 64;" ::"r"(1 + (warp & 3)) : "memory"); };
    float m_run = -INFINITY, l_run = 0.0f;
    // bias-term sums per scale group, as (even tokens, odd tokens) pairs
    float2 corr0 = make_float2(0.0f, 0.0f), corr1 = make_float2(0.0f, 0.0f);
    pair_sync();  // both halves have read the q sums before s_mx is reused
    for (int i = 0; i < n_tiles; ++i) {
      const int b = i & 1;
      const uint32_t use = static_cast<uint32_t>(i >> 1);
      const int t0 = t_begin + i * kTok;
      const float4* s_ts = reinterpret_cast<const float4*>(smem + TLayout::TS + b * kTok * 16);
      const float4* s_tv = reinterpret_cast<const float4*>(smem + TLayout::TV + b * kTok * 16);
      mbar_wait_bounded(&s_full[b], use & 1u, p.err, kWaitBudget);
      mbar_wait_bounded(&k_full[b], use & 1u, p.err, kWaitBudget);  // score terms (done: S(i) needed them)
      tc_fence_after();
      // scores of this thread's 32 tokens (both scale groups' S' halves)
      // scores relative to the running max (the previous tile's; 0 before
      // any): sc = score - mref, the subtraction folded into the FMA chain
      const float mref = m_run == -INFINITY ? 0.0f : m_run;
      float sc[32];
      {
        uint32_t r0[32], r1[32];
        tmem_ld32_raw(tmem + 128 * b + lane_off + 32 * hf, r0);
        tmem_ld32_raw(tmem + 128 * b + 64 + lane_off + 32 * hf, r1);
        tmem_wait_ld();
        reg_fence(r0);
        reg_fence(r1);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_free[b]);  // S[b] may take tile i + 2
        const float2 nm = make_float2(-mref, -mref);
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          const float4 a = lds4(&s_ts[2 * (16 * hf + j / 2)]);      // (A0, A0', A1, A1')
          const float4 bz = lds4(&s_ts[2 * (16 * hf + j / 2) + 1]); // (B0, B0', B1, B1')
          const float2 s2 = fma2(make_float2(a.x, a.y),
                                 make_float2(__uint_as_float(r0[j]), __uint_as_float(r0[j + 1])),
                                 fma2(make_float2(a.z, a.w),
                                      make_float2(__uint_as_float(r1[j]), __uint_as_float(r1[j + 1])),
                                      fma2(make_float2(bz.x, bz.y), qs0p,
                                           fma2(make_float2(bz.z, bz.w), qs1p, nm))));
          sc[j] = s2.x;
          sc[j + 1] = s2.y;
        }
      }
      const bool full = t0 + kTok <= t_end && (!p.causal || t0 + kTok - 1 <= qpos_lo) &&
                        (p.window <= 0 || qpos_hi - t0 < p.window);
      if (!full) {
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int t = t0 + 32 * hf + j;
          const bool vis = t < t_end && t <= qpos && (p.window <= 0 || qpos - t < p.window);
          sc[j] = vis ? sc[j] : -INFINITY;
        }
      }
      float mx = sc[0];
#pragma unroll
      for (int j = 1; j < 32; ++j) mx = fmaxf(mx, sc[j]);
      float* mxb = s_mx + b * kSoftmaxThreads;  // by tile parity: a partner may lag one tile
      mxb[xs] = mx;
      pair_sync();
      mx = fmaxf(mxb[rl], mxb[rl + kRows]);
      // move the running max only when it grows by more than 8 (2^8 headroom;
      // mx is relative to mref); both threads of the row take the same
      // decision, and then shift their scores to the new max
      bool rescale = false;
      float alpha = 1.0f;
      if (mx > 8.0f || (m_run == -INFINITY && mx > -INFINITY)) {
        const float m_new = fmaxf(mx + mref, m_run);
        alpha = (m_run == -INFINITY) ? 0.0f : fast_exp2(m_run - m_new);
        rescale = i > 0 && m_run != -INFINITY;
        const float delta = m_new - mref;
#pragma unroll
        for (int j = 0; j < 32; ++j) sc[j] -= delta;
        m_run = m_new;
        l_run *= alpha;
        corr0 = mul2(corr0, make_float2(alpha, alpha));
        corr1 = mul2(corr1, make_float2(alpha, alpha));
      }
      // O_hf *= alpha once PV(i-1) is done; tcgen05.ld/st are warp-wide, so the
      // whole warp takes the branch with alpha = 1 on the other rows
      if (__any_sync(0xffffffffu, rescale)) {
        const int pb = (i - 1) & 1;
        mbar_wait_bounded(&pv_done[pb], static_cast<uint32_t>((i - 1) >> 1) & 1u, p.err, kWaitBudget);
        tc_fence_after();
        const float a = rescale ? alpha : 1.0f;
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
          float o[32];
          const uint32_t ta = t_o + lane_off + 64 * hf + 32 * c;
          tmem_ld32(ta, o);
#pragma unroll
          for (int k = 0; k < 32; ++k) o[k] *= a;
          tmem_st32(ta, o);
        }
      }
      // P[b] is free once PV(i-2) is done; the value terms of tile i are in
      if (i >= 2) mbar_wait_bounded(&pv_done[b], (use - 1) & 1u, p.err, kWaitBudget);
      mbar_wait_bounded(&v_full[b], use & 1u, p.err, kWaitBudget);
      float2 lsum = make_float2(0.0f, 0.0f);  // masked scores give exp2(-inf) = 0
      unsigned char* prow = smem + TLayout::P + b * TLayout::PB;
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        const int ch = 4 * hf + cc;
        uint32_t w0[4], w1[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int j = 8 * cc + 2 * e;
          const float2 pp = make_float2(fast_exp2(sc[j]), fast_exp2(sc[j + 1]));
          lsum = add2(lsum, pp);
          const float4 vs = lds4(&s_tv[2 * (16 * hf + j / 2)]);      // (vs0, vs0', vs1, vs1')
          const float4 vc = lds4(&s_tv[2 * (16 * hf + j / 2) + 1]);  // (c0, c0', c1, c1')
          const float2 p0 = mul2(pp, make_float2(vs.x, vs.y));
          const float2 p1 = mul2(pp, make_float2(vs.z, vs.w));
          const __half2 h0 = __floats2half2_rn(p0.x, p0.y);
          const __half2 h1 = __floats2half2_rn(p1.x, p1.y);
          corr0 = fma2(pp, make_float2(vc.x, vc.y), corr0);
          corr1 = fma2(pp, make_float2(vc.z, vc.w), corr1);
          w0[e] = *reinterpret_cast<const uint32_t*>(&h0);
          w1[e] = *reinterpret_cast<const uint32_t*>(&h1);
        }
        *reinterpret_cast<uint4*>(prow + sw128(rl, ch)) = make_uint4(w0[0], w0[1], w0[2], w0[3]);
        *reinterpret_cast<uint4*>(prow + kRows * 128 + sw128(rl, ch)) =
            make_uint4(w1[0], w1[1], w1[2], w1[3]);
      }
      l_run += lsum.x + lsum.y;
      fence_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[b]);
    }

    // ---- epilogue: the row's two halves add their l and bias terms; thread hf
    // writes scale group hf: out = (64 O'_hf + corr_hf) / l
    const bool o_init = n_tiles > 0;
    if (o_init) {
      const int lb = (n_tiles - 1) & 1;
      mbar_wait_bounded(&pv_done[lb], static_cast<uint32_t>((n_tiles - 1) >> 1) & 1u, p.err,
                        kWaitBudget);
      tc_fence_after();
    }
    float* s_red = reinterpret_cast<float*>(smem + TLayout::RED);  // [3][256]
    s_red[xs] = l_run;
    const float corr0s = corr0.x + corr0.y, corr1s = corr1.x + corr1.y;
    s_red[kSoftmaxThreads + xs] = corr0s;
    s_red[2 * kSoftmaxThreads + xs] = corr1s;
    pair_sync();
    const int pt = xs ^ kRows;  // partner's slot
    const float l_tot = l_run + s_red[pt];
    const float corr = (hf ? corr1s : corr0s) + s_red[(hf ? 2 : 1) * kSoftmaxThreads + pt];
    const bool direct = p.splits == 1;
    const long long unit = static_cast<long long>(kv) * gridDim.y + mt;
    // split partials, column-major so a warp's 32 rows are one 128 B store:
    // ws[unit][split][d or m or l][row]
    float* wsr = p.ws + (unit * p.splits + split) * (kD + 2) * kRows + rl;
    const float inv = l_tot == 0.0f ? 0.0f : 1.0f / l_tot;
    const long long ob = (static_cast<long long>(qi) * p.H + h) * kD;
    const bool ovec = (reinterpret_cast<uintptr_t>(p.out) & 15u) == 0;
#pragma unroll 1
    for (int c = 0; c < 2; ++c) {
      float o[32];
      if (o_init) {
        tmem_ld32(t_o + lane_off + 64 * hf + 32 * c, o);
      } else {
#pragma unroll
        for (int k = 0; k < 32; ++k) o[k] = 0.0f;
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int d0 = 64 * hf + 32 * c + 8 * k;  // first dim of this 8-column chunk
        float v[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) v[perm8(e)] = fmaf(64.0f, o[8 * k + e], corr);
        if (direct) {
          if (row_ok) {
#pragma unroll
            for (int e = 0; e < 8; ++e) v[e] *= inv;
            store8(p.out, ob + d0, p.out_dtype, ovec, v);
          }
        } else {
#pragma unroll
          for (int e = 0; e < 8; ++e) __stcg(wsr + (d0 + e) * kRows, v[e]);
        }
      }
    }
    if (!direct && hf == 0) {
      __stcg(wsr + kD * kRows, l_tot == 0.0f ? -INFINITY : m_run);
      __stcg(wsr + (kD + 1) * kRows, l_tot);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols)
                 : "memory");
  }
}

// Merge of the split partials (log-sum-exp weights), launched after the
// attention grid with programmatic dependent launch. Grid (D/32, 128/32,
// units); 256 threads: lane = row of a 32-row block, warp = 4 of the block's
// 32 dims; the block is transposed through shared memory so the output rows
// are written 64 B at a time.
__global__ void __launch_bounds__(256) attn_tc_merge_kernel(const TCParams p, int mtiles) {
  pdl_wait();
  pdl_trigger();
  __shared__ float tile[32][33];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int db = blockIdx.x * 32, rb = blockIdx.y * 32;
  const long long unit = blockIdx.z;
  const int kv = static_cast<int>(unit / mtiles), mt = static_cast<int>(unit % mtiles);
  const int S = p.splits;
  const long long sstride = static_cast<long long>(kD + 2) * kRows;
  const float* base = p.ws + unit * S * sstride + rb + lane;
  // Up to kOne splits: every split's (m, l, o) is loaded in one round (one
  // L2 latency), then merged from registers; the batched case's 9 splits
  // took 7.1 us of merge with the max loaded first and the rest after it,
  // 3.2 us this way. More splits: the max first, then the rest, both
  // loops unrolled so several splits' loads are in flight.
  float L = 0.0f, acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  const float* col = base + (db + 4 * warp) * kRows;
  constexpr int kOne = 16;
  if (S <= kOne) {
    float ms[kOne], ls[kOne], v[kOne][4];
#pragma unroll
    for (int s = 0; s < kOne; ++s) {
      if (s < S) {
        const float* ps = base + s * sstride;
        ms[s] = __ldcg(ps + kD * kRows);
        ls[s] = __ldcg(ps + (kD + 1) * kRows);
#pragma unroll
        for (int k = 0; k < 4; ++k) v[s][k] = __ldcg(col + s * sstride + k * kRows);
      }
    }
    float M = -INFINITY;
#pragma unroll
    for (int s = 0; s < kOne; ++s) if (s < S) M = fmaxf(M, ms[s]);
#pragma unroll
    for (int s = 0; s < kOne; ++s) {
      if (s < S) {
        const float e = (ms[s] == -INFINITY) ? 0.0f : fast_exp2(ms[s] - M);
        L = fmaf(e, ls[s], L);
#pragma unroll
        for (int k = 0; k < 4; ++k) acc[k] = fmaf(e, v[s][k], acc[k]);
      }
    }
  } else {
    float M = -INFINITY;
#pragma unroll 8
    for (int s = 0; s < S; ++s) M = fmaxf(M, __ldcg(base + s * sstride + kD * kRows));
#pragma unroll 8
    for (int s = 0; s < S; ++s) {
      const float* ps = base + s * sstride;
      const float ms = __ldcg(ps + kD * kRows);
      const float ls = __ldcg(ps + (kD + 1) * kRows);
      float v[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) v[k] = __ldcg(col + s * sstride + k * kRows);
      const float e = (ms == -INFINITY) ? 0.0f : fast_exp2(ms - M);
      L = fmaf(e, ls, L);
#pragma unroll
      for (int k = 0; k < 4; ++k) acc[k] = fmaf(e, v[k], acc[k]);
    }
  }
  const float invL = L == 0.0f ? 0.0f : 1.0f / L;
#pragma unroll
  for (int k = 0; k < 4; ++k) tile[lane][4 * warp + k] = acc[k] * invL;
  __syncthreads();
  const int rows_total = p.n_q * p.G;
#pragma unroll
  for (int rr = warp; rr < 32; rr += 8) {
    const int row = mt * kRows + rb + rr;
    if (row < rows_total) {
      const int qi = row / p.G, h = kv * p.G + row % p.G;
      store_from_float(p.out, (static_cast<long long>(qi) * p.H + h) * kD + db + lane, p.out_dtype,
                       tile[rr][lane]);
    }
  }
}

int tc_splits(int units, int tiles) {
  int dev = 0;
  cudaGetDevice(&dev);
  const int target = device_sm_count(dev);  // one CTA per SM (512 TMEM columns, 170 KB smem)
  int s = target / (units > 0 ? units : 1);
  if (s < 1) s = 1;
  if (s > tiles) s = tiles > 0 ? tiles : 1;
  if (s > 64) s = 64;
  return s;
}

}  // namespace
}  // namespace tq

using namespace tq;

extern "C" {

TQ_API size_t tq_sdpa_int4_multi_workspace_size(int n_q, int num_heads, int num_kv_heads,
                                                int head_dim, int n_tokens) {
  if (n_q < 1 || num_kv_heads < 1 || num_heads % num_kv_heads || head_dim != kD || n_tokens < 0)
    return 0;
  const int G = num_heads / num_kv_heads;
  const int mtiles = (n_q * G + kRows - 1) / kRows;
  const int units = mtiles * num_kv_heads;
  const int tiles = (n_tokens + kTok - 1) / kTok;
  const int s = tc_splits(units, tiles);
  if (s <= 1) return 0;
  return kCounterRegionBytes + static_cast<size_t>(units) * s * kRows * (kD + 2) * sizeof(float);
}

TQ_API int tq_sdpa_int4_multi(const void* queries, tq_dtype q_dtype, const uint32_t* k_quant,
                              const void* k_scales, const void* k_biases, const uint32_t* v_quant,
                              const void* v_scales, const void* v_biases, tq_dtype sb_dtype,
                              int gqa_factor, float scale, int sliding_window, int num_kv_heads,
                              int head_dim, int n_q, int n_tokens, int capacity, int causal,
                              int pos0, void* out, tq_dtype out_dtype, void* workspace,
                              size_t workspace_bytes, void* stream) {
  auto fail = [](int code, const char* m) {
    set_last_error("tq_sdpa_int4_multi: %s", m);
    return code;
  };
  if (head_dim != kD) return fail(TQ_ERR_UNSUPPORTED, "head_dim must be 128");
  if (!queries || !k_quant || !k_scales || !k_biases || !v_quant || !v_scales || !v_biases || !out)
    return fail(TQ_ERR_INVALID, "null pointer argument");
  if (gqa_factor < 1 || num_kv_heads < 1 || n_q < 1 || n_tokens < 0 || n_tokens > capacity ||
      capacity % 4 || sliding_window < 0)
    return fail(TQ_ERR_INVALID, "bad sizes");
  if (sb_dtype != TQ_F16 && sb_dtype != TQ_F32) return fail(TQ_ERR_UNSUPPORTED, "scales must be f16 or f32");
  const uintptr_t a = reinterpret_cast<uintptr_t>(k_quant) | reinterpret_cast<uintptr_t>(v_quant);
  if (a & 15u) return fail(TQ_ERR_INVALID, "cache pointers must be 16-byte aligned");
  const int H = num_kv_heads * gqa_factor;
  const int mtiles = (n_q * gqa_factor + kRows - 1) / kRows;
  const int units = mtiles * num_kv_heads;
  const int tiles = (n_tokens + kTok - 1) / kTok;
  int splits = tc_splits(units, tiles);
  const int tps = tiles > 0 ? (tiles + splits - 1) / splits : 1;
  splits = tiles > 0 ? (tiles + tps - 1) / tps : 1;
  TCParams p{};
  p.q = queries;
  p.q_dtype = q_dtype;
  p.kq = k_quant;
  p.ks = k_scales;
  p.kb = k_biases;
  p.vq = v_quant;
  p.vs = v_scales;
  p.vb = v_biases;
  p.sb_f32 = sb_dtype == TQ_F32;
  p.H = H;
  p.Hkv = num_kv_heads;
  p.G = gqa_factor;
  p.n_q = n_q;
  p.n_tokens = n_tokens;
  p.capacity = capacity;
  p.causal = causal;
  p.pos0 = pos0;
  p.window = sliding_window;
  p.qscale = scale * kLog2e;
  p.splits = splits;
  p.tiles_per_split = tps;
  p.out = out;
  p.out_dtype = out_dtype;
  if (splits > 1) {
    const size_t need = kCounterRegionBytes + static_cast<size_t>(units) * splits * kRows * (kD + 2) * sizeof(float);
    if (!workspace || workspace_bytes < need) {
      set_last_error("tq_sdpa_int4_multi: workspace of %zu bytes needed", need);
      return TQ_ERR_WORKSPACE;
    }
    p.ws = reinterpret_cast<float*>(static_cast<unsigned char*>(workspace) + kCounterRegionBytes);
  }
  int dev = 0;
  cudaGetDevice(&dev);
  static int attr_set[64] = {0};
  if (dev < 64 && !attr_set[dev]) {
    cudaFuncSetAttribute(attn_tc_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, TLayout::BYTES);
    cudaFuncSetAttribute(attn_tc_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         TLayout::BYTES_QLO);
    attr_set[dev] = 1;
  }
  p.err = device_error_word();
  const bool qlo = q_dtype == TQ_F32;
  const cudaError_t e =
      qlo ? launch_pdl(attn_tc_kernel<true>, dim3(splits, mtiles, num_kv_heads), dim3(kThreads),
                       static_cast<size_t>(TLayout::BYTES_QLO), static_cast<cudaStream_t>(stream), p)
          : launch_pdl(attn_tc_kernel<false>, dim3(splits, mtiles, num_kv_heads), dim3(kThreads),
                       static_cast<size_t>(TLayout::BYTES), static_cast<cudaStream_t>(stream), p);
  if (e != cudaSuccess) {
    set_last_error("tq_sdpa_int4_multi: %s", cudaGetErrorString(e));
    return TQ_ERR_CUDA;
  }
  if (splits > 1) {
    const cudaError_t e2 = launch_pdl(attn_tc_merge_kernel, dim3(kD / 32, kRows / 32, units), dim3(256), 0,
                                      static_cast<cudaStream_t>(stream), p, mtiles);
    if (e2 != cudaSuccess) {
      set_last_error("tq_sdpa_int4_multi (merge): %s", cudaGetErrorString(e2));
      return TQ_ERR_CUDA;
    }
  }
  return TQ_OK;
}

// The two config-2 cases under their own names (the multi-query kernel serves
// both): batched decode of n_seq single queries over one shared cache, and a
// causal prefill chunk of n_q queries whose first sits at position pos0.
TQ_API int tq_sdpa_int4_batched(const void* queries, tq_dtype q_dtype, const uint32_t* k_quant,
                                const void* k_scales, const void* k_biases,
                                const uint32_t* v_quant, const void* v_scales,
                                const void* v_biases, tq_dtype sb_dtype, int gqa_factor,
                                float scale, int sliding_window, int num_kv_heads, int head_dim,
                                int n_seq, int n_tokens, int capacity, void* out,
                                tq_dtype out_dtype, void* workspace, size_t workspace_bytes,
                                void* stream) {
  return tq_sdpa_int4_multi(queries, q_dtype, k_quant, k_scales, k_biases, v_quant, v_scales,
                            v_biases, sb_dtype, gqa_factor, scale, sliding_window, num_kv_heads,
                            head_dim, n_seq, n_tokens, capacity, 0, 0, out, out_dtype, workspace,
                            workspace_bytes, stream);
}

TQ_API int tq_sdpa_int4_prefill(const void* queries, tq_dtype q_dtype, const uint32_t* k_quant,
                                const void* k_scales, const void* k_biases,
                                const uint32_t* v_quant, const void* v_scales,
                                const void* v_biases, tq_dtype sb_dtype, int gqa_factor,
                                float scale, int sliding_window, int num_kv_heads, int head_dim,
                                int n_q, int pos0, int capacity, void* out, tq_dtype out_dtype,
                                void* workspace, size_t workspace_bytes, void* stream) {
  return tq_sdpa_int4_multi(queries, q_dtype, k_quant, k_scales, k_biases, v_quant, v_scales,
                            v_biases, sb_dtype, gqa_factor, scale, sliding_window, num_kv_heads,
                            head_dim, n_q, pos0 + n_q, capacity, 1, pos0, out, out_dtype, workspace,
                            workspace_bytes, stream);
}

}  // extern "C"
