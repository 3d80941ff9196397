// Tensor-core (tcgen05 + TMEM) int4 attention for many query rows per KV
// head: the batched-decode case (B sequences x 1 query against one shared
// cache) and the causal prefill chunk (n_q queries at positions pos0.. of one
// sequence). The reference runs both through MLX dequantize + fast::sdpa with
// a CPU-built mask (engine/gemma4_multilayer.cpp:307-308,347-367,441-464).
//
// CTA = 128 query rows of one KV head (row = (query, GQA head) pair; TMEM lane
// = row), 4 warps, 2 CTAs per SM. Per 64-token tile of the int4 cache:
//   1. all threads unpack the K and V codes into shared memory as exact fp16
//      values 1 + c/64, in the UMMA canonical 128B-swizzled layout (K: K-major
//      B operand of S = Q K^T; V: MN-major B operand of O = P V), one 8 KB
//      region per 64-dim scale group; per-token scale/bias terms go to smem;
//   2. thread 0 issues tcgen05.mma S'_g = Q_g (1 + C_g/64)^T per scale group g
//      (fp16 x fp16 -> fp32 in TMEM; exact products), commit -> mbarrier;
//   3. each thread reads its row of S'_0, S'_1 (tcgen05.ld), forms the scores
//      score = 64 s_0 S'_0 + 64 s_1 S'_1 + (b_0 - 64 s_0) sum q_0 + (b_1 - 64 s_1) sum q_1
//      (the int4 scale/bias factored out of the dot product, as
//      lib/turboquant.metal:803 does), masks (causal / window / length),
//      online softmax in log2 units, writes P'_g = p * s_g(token) as fp16
//      (K-major A operand) and accumulates the bias term
//      sum p b + 8 p s - 72 fp16(p s) (exact for the rounded weights);
//   4. thread 0 issues O'_g += P'_g (1 + C_g/64) per group into TMEM.
// The running max is only moved (and O rescaled in TMEM) when a row's max
// grows by more than 8 (log2 units), so most tiles skip the rescale.
// out = (64 O' + bias term) / l. The 8-element dim order inside each
// code word follows the unpack (d = 0,4,1,5,2,6,3,7), applied to Q as well and
// undone when O is written.
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
constexpr int kThreads = 128;
constexpr int kTmemCols = 256; // S'_0, S'_1, O'_0, O'_1 (64 fp32 columns each)
// an MMA group finishes in microseconds; give up (and record the error) after
// ~10 ms of SM clocks so a wait that cannot complete still ends the kernel
constexpr long long kWaitBudget = 20000000LL;

struct TLayout {
  static constexpr int Q = 0;                   // [2 groups][128 rows][128 B]  32 KB
  static constexpr int K = Q + 2 * kRows * 128; // [2][64 tokens][128 B]        16 KB
  static constexpr int V = K + 2 * kTok * 128;  // [2][64][128 B]               16 KB
  static constexpr int P = V + 2 * kTok * 128;  // [2][128 rows][128 B]         32 KB
  static constexpr int TS = P + 2 * kRows * 128;  // per token: {A0, A1, B0, B1} (score terms)
  static constexpr int TV = TS + kTok * 16;        // per token: {vs0, vs1, vbm0, vbm1}
  static constexpr int BAR = TV + kTok * 16;       // mbarriers: S done, O done
  static constexpr int TMEM = BAR + 16;            // allocated TMEM base address
  static constexpr int BYTES = TMEM + 16 + 1024;   // + alignment slack
};

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
  float* ws;           // split partials: (units, splits, 128 rows, D + 2)
  unsigned* counters;
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

__device__ __forceinline__ float sbload(const void* p, long long i, int f32) {
  return f32 ? reinterpret_cast<const float*>(p)[i] : __half2float(reinterpret_cast<const __half*>(p)[i]);
}

__global__ void __launch_bounds__(kThreads, 2) attn_tc_kernel(const TCParams p) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bar_s = reinterpret_cast<uint64_t*>(smem + TLayout::BAR);
  uint64_t* bar_o = bar_s + 1;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + TLayout::TMEM);
  float4* s_ts = reinterpret_cast<float4*>(smem + TLayout::TS);
  float4* s_tv = reinterpret_cast<float4*>(smem + TLayout::TV);
  const uint32_t sbase = smem_u32(smem);

  const int tid = threadIdx.x, warp = tid >> 5;
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
    mbar_init(bar_s, 1);
    mbar_init(bar_o, 1);
    fence_barrier_init();
  }

  // ---- this thread's row: query qi, head h (rows past the end compute on zeros)
  const int row = mt * kRows + tid;
  const bool row_ok = row < rows_total;
  const int qi = row_ok ? row / p.G : 0;
  const int h = kv * p.G + (row_ok ? row % p.G : 0);
  // position of the query: causal rows at pos0 + qi; otherwise every query
  // sits at the end of the shared cache (the window counts back from there)
  const int qpos = p.causal ? p.pos0 + qi : p.n_tokens - 1;
  // Q row -> smem (fp16, dims permuted inside each 8-dim word like the codes)
  float qsum0 = 0.0f, qsum1 = 0.0f;
  {
    const long long qb = (static_cast<long long>(qi) * p.H + h) * kD;
#pragma unroll
    for (int g = 0; g < 2; ++g)
#pragma unroll
      for (int ch = 0; ch < 8; ++ch) {
        float v[8];
#pragma unroll
        for (int e = 0; e < 8; ++e)
          v[e] = row_ok ? load_as_float(p.q, qb + g * 64 + ch * 8 + perm8(e), p.q_dtype) : 0.0f;
        // fp16 copies (exact for fp16 and bf16 inputs in range)
        __half2 hh[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          hh[e] = __floats2half2_rn(v[2 * e], v[2 * e + 1]);
          const float2 f = __half22float2(hh[e]);
          if (g == 0) qsum0 += f.x + f.y; else qsum1 += f.x + f.y;
        }
        *reinterpret_cast<uint4*>(smem + TLayout::Q + g * kRows * 128 + sw128(tid, ch)) =
            *reinterpret_cast<uint4*>(hh);
      }
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;
  const uint32_t t_s0 = tmem, t_s1 = tmem + 64, t_o0 = tmem + 128, t_o1 = tmem + 192;
  const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;

  // ---- token range of this split (tiles of 64 tokens)
  int n_vis = p.n_tokens;
  const int t_begin = split * p.tiles_per_split * kTok;
  const int t_end = min(n_vis, t_begin + p.tiles_per_split * kTok);
  const long long tok_base = static_cast<long long>(kv) * p.capacity;

  float m_run = -INFINITY, l_run = 0.0f, corr0 = 0.0f, corr1 = 0.0f;
  bool o_init = false;  // TMEM O holds accumulated values
  uint32_t ph = 0;

  for (int t0 = t_begin; t0 < t_end; t0 += kTok) {
    // ---- 1. unpack K and V codes of 64 tokens into the canonical layouts ----
    {
      const int tok = tid & 63, grp = tid >> 6;
      const int t = t0 + tok;
      const bool tv = t < t_end;
      const long long rowi = tok_base + (tv ? t : t0);
#pragma unroll
      for (int kvs = 0; kvs < 2; ++kvs) {
        const uint32_t* src = (kvs ? p.vq : p.kq) + rowi * (kD / 8) + grp * 8;
        const uint4 w0 = reinterpret_cast<const uint4*>(src)[0];
        const uint4 w1 = reinterpret_cast<const uint4*>(src)[1];
        const uint32_t w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
        unsigned char* dst = smem + (kvs ? TLayout::V : TLayout::K) + grp * kTok * 128;
#pragma unroll
        for (int ch = 0; ch < 8; ++ch) {
          uint4 o;
          o.x = nib64h<0>(w[ch]);
          o.y = nib64h<1>(w[ch]);
          o.z = nib64h<2>(w[ch]);
          o.w = nib64h<3>(w[ch]);
          *reinterpret_cast<uint4*>(dst + sw128(tok, ch)) = o;
        }
      }
      if (tid < kTok) {
        const long long gi = (tok_base + (tv ? t : t0)) * 2;
        const float ks0 = sbload(p.ks, gi, p.sb_f32), ks1 = sbload(p.ks, gi + 1, p.sb_f32);
        const float kb0 = sbload(p.kb, gi, p.sb_f32), kb1 = sbload(p.kb, gi + 1, p.sb_f32);
        const float vs0 = sbload(p.vs, gi, p.sb_f32), vs1 = sbload(p.vs, gi + 1, p.sb_f32);
        const float vb0 = sbload(p.vb, gi, p.sb_f32), vb1 = sbload(p.vb, gi + 1, p.sb_f32);
        const float qs = p.qscale;
        s_ts[tok] = tv ? make_float4(64.0f * ks0 * qs, 64.0f * ks1 * qs, (kb0 - 64.0f * ks0) * qs,
                                     (kb1 - 64.0f * ks1) * qs)
                       : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        s_tv[tok] = tv ? make_float4(vs0, vs1, vb0, vb1) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      }
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();

    // ---- 2. S'_g = Q_g (1 + C_g/64)^T ------------------------------------------
    if (tid == 0) {
      constexpr uint32_t idS = idesc_f16(false);
#pragma unroll
      for (int g = 0; g < 2; ++g)
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
          const uint64_t a = umma_desc(sbase + TLayout::Q + g * kRows * 128 + ks * 32, 16);
          const uint64_t b = umma_desc(sbase + TLayout::K + g * kTok * 128 + ks * 32, 16);
          umma_f16(g ? t_s1 : t_s0, a, b, idS, ks > 0 ? 1u : 0u);
        }
      umma_commit(bar_s);
    }
    mbar_wait_bounded(bar_s, ph, p.err, kWaitBudget);
    tc_fence_after();

    // ---- 3. scores, online softmax, P' and the bias terms ----------------------
    const bool need_mask = p.causal || p.window > 0 || t0 + kTok > t_end;
    float s0[64];
    float mx = -INFINITY;
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      float a0[32], a1[32];
      tmem_ld32(t_s0 + lane_off + 32 * c, a0);
      tmem_ld32(t_s1 + lane_off + 32 * c, a1);
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int i = 32 * c + j;
        const float4 a = s_ts[i];
        float v = fmaf(a.x, a0[j], fmaf(a.y, a1[j], fmaf(a.z, qsum0, a.w * qsum1)));
        if (need_mask) {
          const int t = t0 + i;
          const bool vis = t < t_end && t <= qpos && (p.window <= 0 || qpos - t < p.window) && row_ok;
          v = vis ? v : -INFINITY;
        }
        s0[i] = v;
        mx = fmaxf(mx, v);
      }
    }
    // move the running max only when it grows by more than 8 (2^8 headroom)
    bool rescale = false;
    float alpha = 1.0f;
    if (mx > m_run + 8.0f || (m_run == -INFINITY && mx > -INFINITY)) {
      const float m_new = fmaxf(mx, m_run);
      alpha = (m_run == -INFINITY) ? 0.0f : fast_exp2(m_run - m_new);
      rescale = o_init && m_run != -INFINITY;
      m_run = m_new;
      l_run *= alpha;
      corr0 *= alpha;
      corr1 *= alpha;
    }
    float lsum = 0.0f;
    unsigned char* prow = smem + TLayout::P;
#pragma unroll
    for (int ch = 0; ch < 8; ++ch) {
      uint32_t w0[4], w1[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int i = ch * 8 + 2 * e;
        const float pa = (s0[i] == -INFINITY) ? 0.0f : fast_exp2(s0[i] - m_run);
        const float pb = (s0[i + 1] == -INFINITY) ? 0.0f : fast_exp2(s0[i + 1] - m_run);
        lsum += pa + pb;
        const float4 va = s_tv[i], vb = s_tv[i + 1];
        const float wa0 = pa * va.x, wb0 = pb * vb.x, wa1 = pa * va.y, wb1 = pb * vb.y;
        const __half2 h0 = __floats2half2_rn(wa0, wb0);
        const __half2 h1 = __floats2half2_rn(wa1, wb1);
        // bias term with the fp16 weights r the mma sees (out = 64 O' + corr):
        // corr = sum p b + 8 w - 72 r, which leaves the weights' rounding error
        // multiplied by (c - 8), |c - 8| <= 8, instead of by c
        const float2 r0 = __half22float2(h0), r1 = __half22float2(h1);
        corr0 = fmaf(pa, va.z, fmaf(pb, vb.z, fmaf(8.0f, wa0 + wb0, fmaf(-72.0f, r0.x + r0.y, corr0))));
        corr1 = fmaf(pa, va.w, fmaf(pb, vb.w, fmaf(8.0f, wa1 + wb1, fmaf(-72.0f, r1.x + r1.y, corr1))));
        w0[e] = *reinterpret_cast<const uint32_t*>(&h0);
        w1[e] = *reinterpret_cast<const uint32_t*>(&h1);
      }
      *reinterpret_cast<uint4*>(prow + sw128(tid, ch)) = make_uint4(w0[0], w0[1], w0[2], w0[3]);
      *reinterpret_cast<uint4*>(prow + kRows * 128 + sw128(tid, ch)) =
          make_uint4(w1[0], w1[1], w1[2], w1[3]);
    }
    l_run += lsum;
    // O *= alpha for the rows whose max moved; tcgen05.ld/st are warp-wide
    // (.sync.aligned), so the whole warp takes the branch with alpha = 1 on
    // the other rows
    if (__any_sync(0xffffffffu, rescale)) {
      const float a = rescale ? alpha : 1.0f;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        float o[32];
        const uint32_t ta = t_o0 + lane_off + c * 32;
        tmem_ld32(ta, o);
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] *= a;
        tmem_st32(ta, o);
      }
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();

    // ---- 4. O'_g += P'_g (1 + C_g/64) ---------------------------------------------
    if (tid == 0) {
      constexpr uint32_t idO = idesc_f16(true);
#pragma unroll
      for (int g = 0; g < 2; ++g)
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
          const uint64_t a = umma_desc(sbase + TLayout::P + g * kRows * 128 + ks * 32, 16);
          const uint64_t b = umma_desc(sbase + TLayout::V + g * kTok * 128 + ks * 16 * 128, 16);
          umma_f16(g ? t_o1 : t_o0, a, b, idO, (o_init || ks > 0) ? 1u : 0u);
        }
      umma_commit(bar_o);
    }
    o_init = true;
    mbar_wait_bounded(bar_o, ph, p.err, kWaitBudget);
    tc_fence_after();
    ph ^= 1u;
  }

  // ---- epilogue: out = (64 O' + corr) / l, 32 TMEM columns at a time ---------------
  // TMEM column j of group g holds dim g*64 + 8*(j/8) + perm8(j%8)
  const bool direct = p.splits == 1;
  const long long unit = static_cast<long long>(kv) * gridDim.y + mt;
  float* wsr = p.ws + ((unit * p.splits + split) * kRows + tid) * (kD + 2);
  const float inv = l_run > 0.0f ? 1.0f / l_run : 0.0f;
  const long long ob = (static_cast<long long>(qi) * p.H + h) * kD;
#pragma unroll 1
  for (int c = 0; c < 4; ++c) {
    float o[32];
    if (o_init) {
      tmem_ld32(t_o0 + lane_off + c * 32, o);
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i) o[i] = 0.0f;
    }
    const float corr = (c >> 1) ? corr1 : corr0;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const int j = 32 * c + i;
      const int d = (j & ~7) + perm8(j & 7);
      const float v = fmaf(64.0f, o[i], corr);
      if (direct) {
        if (row_ok) store_from_float(p.out, ob + d, p.out_dtype, l_run > 0.0f ? v * inv : 0.0f);
      } else {
        wsr[d] = v;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols)
                 : "memory");
  }
  if (direct) return;
  // split partial: (o unnormalised, m in log2 units, l), row-major per CTA
  wsr[kD] = l_run > 0.0f ? m_run : -INFINITY;
  wsr[kD + 1] = l_run;
  __syncthreads();
  __shared__ int s_last;
  if (tid == 0) {
    const unsigned prev = atomic_add_acq_rel(&p.counters[unit], 1u);
    s_last = prev == static_cast<unsigned>(p.splits - 1);
  }
  __syncthreads();
  if (!s_last || !row_ok) {
    if (s_last && tid == 0) p.counters[unit] = 0u;
    return;
  }
  const float* base = p.ws + (unit * p.splits * kRows + tid) * (kD + 2);
  const long long sstride = static_cast<long long>(kRows) * (kD + 2);
  float M = -INFINITY;
  for (int s = 0; s < p.splits; ++s) M = fmaxf(M, __ldcg(base + s * sstride + kD));
  float L = 0.0f;
  for (int s = 0; s < p.splits; ++s) {
    const float ms = __ldcg(base + s * sstride + kD);
    const float e = (ms == -INFINITY) ? 0.0f : fast_exp2(ms - M);
    L = fmaf(e, __ldcg(base + s * sstride + kD + 1), L);
  }
  const float invL = L > 0.0f ? 1.0f / L : 0.0f;
#pragma unroll 1
  for (int c = 0; c < 4; ++c) {
    float acc[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) acc[i] = 0.0f;
    for (int s = 0; s < p.splits; ++s) {
      const float ms = __ldcg(base + s * sstride + kD);
      const float e = (ms == -INFINITY) ? 0.0f : fast_exp2(ms - M);
#pragma unroll
      for (int i = 0; i < 32; ++i) acc[i] = fmaf(e, __ldcg(base + s * sstride + 32 * c + i), acc[i]);
    }
#pragma unroll
    for (int i = 0; i < 32; ++i) store_from_float(p.out, ob + 32 * c + i, p.out_dtype, acc[i] * invL);
  }
  if (tid == 0) p.counters[unit] = 0u;
}

int tc_splits(int units, int tiles) {
  int dev = 0;
  cudaGetDevice(&dev);
  const int target = device_sm_count(dev) * 2;
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
    if (units * sizeof(unsigned) > kCounterRegionBytes) return fail(TQ_ERR_UNSUPPORTED, "too many row tiles");
    p.counters = static_cast<unsigned*>(workspace);
    p.ws = reinterpret_cast<float*>(static_cast<unsigned char*>(workspace) + kCounterRegionBytes);
  }
  int dev = 0;
  cudaGetDevice(&dev);
  static int attr_set[64] = {0};
  if (dev < 64 && !attr_set[dev]) {
    cudaFuncSetAttribute(attn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, TLayout::BYTES);
    attr_set[dev] = 1;
  }
  p.err = device_error_word();
  const cudaError_t e = launch_pdl(attn_tc_kernel, dim3(splits, mtiles, num_kv_heads), dim3(kThreads),
                                   static_cast<size_t>(TLayout::BYTES),
                                   static_cast<cudaStream_t>(stream), p);
  if (e != cudaSuccess) {
    set_last_error("tq_sdpa_int4_multi: %s", cudaGetErrorString(e));
    return TQ_ERR_CUDA;
  }
  return TQ_OK;
}

}  // extern "C"
