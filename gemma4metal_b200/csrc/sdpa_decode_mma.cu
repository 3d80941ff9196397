// Tensor-core (warp-level mma.sync m16n8k16, f16 x f16 -> f32) split-KV decode
// attention straight from the int4 KV cache. Same contract and partial/merge
// format as decode_kernel in sdpa_decode.cu; this variant exists because the
// CUDA-core kernel is instruction-bound at GQA >= 2, and a
// single mma consumes 128 (K side) or 256 (V side) 4-bit codes per warp
// instruction.
//
// Data path per CTA (grid = splits x KV-head groups x batch):
//   * producer warp: 2-D TMA tensor copies of the K and V code tiles
//     (64 tokens x D/2 bytes, 64B/128B-swizzled so the transposed ldmatrix
//     reads below are bank-conflict free) + 1-D bulk copies of the fp16
//     scales/biases, into a 4-stage full/empty mbarrier ring;
//   * 4 consumer warps, 16 tokens of every tile each, each with its own
//     online-softmax state (no CTA barrier in the main loop):
//       K side:  S[head][token] = sum_d q[head][d] * (1 + c[token][d]/16)
//                as mma(A = q (rows = query heads), B = codes); the codes are
//                made exact fp16 values 1 + c/16 by one shift + one LOP3 per
//                two nibbles, and the offset is removed through sum_d q:
//                score = s*(16*S - 16*sum q) + b*sum q per 64-group;
//       softmax: exp2 in log2 units; weights w = p*s split into fp16 hi+lo
//                (22 significant bits) -- the K-side accumulator layout is
//                exactly the B-operand layout the V side needs;
//       V side:  O[dim][head] += (1 + c/16)^T * w as mma(A = codes read
//                transposed by ldmatrix.trans, B = w hi/lo); the constant part
//                is removed with corr = sum_t p*(b - 16*s) at the end:
//                out = 16*O + corr.
//   * the 4 warp states are LSE-merged in shared memory; the CTA writes its
//     split partial and the last CTA of the KV head merges all splits.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>
#include <unordered_map>

#include "tq_common.cuh"
#include "tq_internal.h"

namespace tq {

namespace {

constexpr int kConsumerWarps = 4;
constexpr int kMThreads = (kConsumerWarps + 1) * 32;  // + one TMA producer warp
constexpr int kMTile = 64;                             // tokens per stage
constexpr int kMStages = 4;
constexpr int kMMaxSplits = 1024;

template <int D, int G, typename SB>
struct MLayout {
  static constexpr int NG = D / 64;
  static constexpr int ROWB = D / 2;                     // code bytes per token
  static constexpr int CODE = kMTile * ROWB;             // one code tile
  static constexpr int SBB = kMTile * NG * static_cast<int>(sizeof(SB));
  static constexpr int STAGE = (2 * CODE + 4 * SBB + 1023) / 1024 * 1024;
  static constexpr int STAGES = kMStages * STAGE;
  static constexpr int BAR = STAGES;                     // full[kMStages], empty[kMStages]
  static constexpr int FLAG = BAR + 2 * kMStages * 8;
  static constexpr int RED = FLAG + 16;                  // float scratch (merge reductions)
  static constexpr int BYTES = RED + 2 * 4 * 8 * 4 + 1024;  // + alignment slack
  // end-of-range combine: per warp m, l, corr[NG], o[D] for G heads
  static constexpr int WST = G * (2 + NG + D);
  static_assert(kConsumerWarps * WST * 4 <= STAGES, "warp states reuse the stages");
  static_assert(G * kMMaxSplits * 4 <= STAGES, "merge weights reuse the stages");
};

struct MParams {
  const void* q;
  int q_dtype;
  const void* ks;
  const void* kb;
  const void* vs;
  const void* vb;
  const int32_t* seq_lens;
  int n_tokens;
  int H, Hkv, Gtot, nsub;
  int capacity;
  long long bstride_tok;
  float qscale;  // scale * log2(e)
  int window;
  int token_offset;
  int n_total;
  int partial;
  void* out;
  int out_dtype;
  float* part_out;
  int splits, tiles_per_split;
  float* ws_o;
  float* ws_ml;
  unsigned* counters;
  uint32_t* err;
};

// ---- PTX wrappers -------------------------------------------------------------
__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t (&d)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
               : "r"(addr));
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void consumers_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory");
}

// Two nibbles (bits 4j and 16+4j of x) -> fp16x2 (1 + c/16): the nibble is
// moved to mantissa bits 6..9 of each half and OR-ed into 1.0 (0x3C00).
template <int J>
__device__ __forceinline__ uint32_t nib2h(uint32_t x) {
  const uint32_t s = (J == 0) ? (x << 6) : (J == 1) ? (x << 2) : (J == 2) ? (x >> 2) : (x >> 6);
  return (s & 0x03C003C0u) | 0x3C003C00u;
}

// Byte offset of 16-byte chunk k of tile row t (TMA swizzle of the code tile).
template <int D>
__device__ __forceinline__ int swz(int t, int k) {
  if constexpr (D == 128) {
    return t * 64 + ((k ^ ((t >> 1) & 3)) << 4);  // SWIZZLE_64B on 64-byte rows
  } else {
    return t * 128 + ((k ^ (t & 7)) << 4);         // SWIZZLE_128B on 128-byte rows
  }
}

__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

__device__ __forceinline__ float2 unpack_h2(uint32_t v) {
  return __half22float2(*reinterpret_cast<const __half2*>(&v));
}

// scales/biases of two consecutive tokens (2*NG values) as floats
template <typename SB, int NG>
__device__ __forceinline__ void load_sb2(const SB* p, float (&v)[2][NG]) {
  if constexpr (sizeof(SB) == 2 && NG == 2) {
    const uint2 raw = *reinterpret_cast<const uint2*>(p);
    const float2 a = unpack_h2(raw.x), b = unpack_h2(raw.y);
    v[0][0] = a.x; v[0][1] = a.y; v[1][0] = b.x; v[1][1] = b.y;
  } else if constexpr (sizeof(SB) == 2 && NG == 4) {
    const uint4 raw = *reinterpret_cast<const uint4*>(p);
    float2 f;
    f = unpack_h2(raw.x); v[0][0] = f.x; v[0][1] = f.y;
    f = unpack_h2(raw.y); v[0][2] = f.x; v[0][3] = f.y;
    f = unpack_h2(raw.z); v[1][0] = f.x; v[1][1] = f.y;
    f = unpack_h2(raw.w); v[1][2] = f.x; v[1][3] = f.y;
  } else {
#pragma unroll
    for (int e = 0; e < 2; ++e)
#pragma unroll
      for (int g = 0; g < NG; ++g) v[e][g] = sb_to_float<SB>(p[e * NG + g]);
  }
}

__device__ __forceinline__ float wmax(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float wsum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <int D, int G, typename SB, bool QSPLIT>
__global__ void __launch_bounds__(kMThreads, D == 128 ? 3 : 1)
    decode_mma_kernel(const __grid_constant__ CUtensorMap tmk,
                      const __grid_constant__ CUtensorMap tmv, const MParams p) {
  using Lyt = MLayout<D, G, SB>;
  constexpr int NG = Lyt::NG;
  constexpr int NCH = D / 32;          // 16-byte code chunks per token
  constexpr bool kPaired = G <= 4;     // hi/lo weights share one mma (N = 2G <= 8)
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Lyt::BAR);
  uint64_t* empty = full + kMStages;
  int* s_flag = reinterpret_cast<int*>(smem + Lyt::FLAG);
  float* s_red = reinterpret_cast<float*>(smem + Lyt::RED);

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int split = blockIdx.x;
  const int hg = blockIdx.y;
  const int b = blockIdx.z;
  const int kv = hg / p.nsub;
  const int h0 = kv * p.Gtot + (hg % p.nsub) * G;

  // ---- visible token range (local coordinates), as in decode_kernel --------
  const int n_local = max(0, min(p.seq_lens ? p.seq_lens[b] : p.n_tokens, p.capacity));
  int t_lo = 0;
  const int t_hi = n_local;
  if (p.window > 0) {
    const int n_glob = p.n_total > 0 ? p.n_total : n_local + p.token_offset;
    t_lo = max(0, n_glob - p.window - p.token_offset);
  }
  int ntiles = 0, tile_begin = 0;
  if (t_hi > t_lo) {
    const int tb = t_lo / kMTile;
    const int te = (t_hi + kMTile - 1) / kMTile;
    tile_begin = tb + split * p.tiles_per_split;
    ntiles = max(0, min(te, tile_begin + p.tiles_per_split) - tile_begin);
  }
  const long long tok_base =
      static_cast<long long>(b) * p.bstride_tok + static_cast<long long>(kv) * p.capacity;

  if (tid == 0) {
    for (int s = 0; s < kMStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    fence_barrier_init();
  }
  __syncthreads();

  // ======================= producer warp ========================================
  if (warp == kConsumerWarps) {
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      const int t_hi4 = (t_hi + 3) & ~3;
      const SB* ksb = reinterpret_cast<const SB*>(p.ks) + tok_base * NG;
      const SB* kbb = reinterpret_cast<const SB*>(p.kb) + tok_base * NG;
      const SB* vsb = reinterpret_cast<const SB*>(p.vs) + tok_base * NG;
      const SB* vbb = reinterpret_cast<const SB*>(p.vb) + tok_base * NG;
      for (int i = 0; i < ntiles; ++i) {
        const int st = i % kMStages;
        if (i >= kMStages) mbar_wait_bounded(&empty[st], ((i / kMStages) + 1) & 1, p.err);
        const int t0 = (tile_begin + i) * kMTile;
        const int nt = min(kMTile, t_hi4 - t0);
        const uint32_t sbb = static_cast<uint32_t>(nt * NG * sizeof(SB));
        unsigned char* sb = smem + st * Lyt::STAGE;
        mbar_arrive_expect_tx(&full[st], 2 * Lyt::CODE + 4 * sbb);
        const int row = static_cast<int>(tok_base + t0);
#pragma unroll
        for (int half = 0; half < (D > 256 ? 2 : 1); ++half) {
          tma_load_2d(sb + half * (Lyt::CODE / 2), &tmk, half * 32, row, &full[st], pol);
          tma_load_2d(sb + Lyt::CODE + half * (Lyt::CODE / 2), &tmv, half * 32, row, &full[st], pol);
        }
        unsigned char* sbp = sb + 2 * Lyt::CODE;
        bulk_g2s(sbp, ksb + static_cast<long long>(t0) * NG, sbb, &full[st], pol);
        bulk_g2s(sbp + Lyt::SBB, kbb + static_cast<long long>(t0) * NG, sbb, &full[st], pol);
        bulk_g2s(sbp + 2 * Lyt::SBB, vsb + static_cast<long long>(t0) * NG, sbb, &full[st], pol);
        bulk_g2s(sbp + 3 * Lyt::SBB, vbb + static_cast<long long>(t0) * NG, sbb, &full[st], pol);
      }
    }
    return;
  }

  // ======================= consumer warps =======================================
  const int r = lane >> 2;  // mma groupID
  const int c = lane & 3;   // mma thread-in-group
  const int hr = kPaired ? (r >> 1) : r;  // query head of K-side row r
  const bool hr_ok = hr < G;

  // q as the K-side A operand: row r = head hr; k-step ks of group g covers
  // word w = 8g + 2c + ks/2, nibbles jb, jb+4 (cols 2c, 2c+1) and jb+1, jb+5
  // (cols 2c+8, 2c+9), jb = 2*(ks%2).
  uint32_t qa[NG][4][2];
  uint32_t qa_lo[QSPLIT ? NG : 1][4][2];
  float qsum[NG];
  {
    const long long qrow = (static_cast<long long>(b) * p.H + h0 + (hr_ok ? hr : 0)) * D;
#pragma unroll
    for (int g = 0; g < NG; ++g) {
      float part = 0.0f;
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        const int w = 8 * g + 2 * c + (ks >> 1);
        const int jb = 2 * (ks & 1);
        float v[4];
        const int dd[4] = {8 * w + jb, 8 * w + jb + 4, 8 * w + jb + 1, 8 * w + jb + 5};
#pragma unroll
        for (int e = 0; e < 4; ++e) v[e] = hr_ok ? load_as_float(p.q, qrow + dd[e], p.q_dtype) : 0.0f;
        part += (v[0] + v[1]) + (v[2] + v[3]);
        qa[g][ks][0] = pack_h2(v[0], v[1]);
        qa[g][ks][1] = pack_h2(v[2], v[3]);
        if constexpr (QSPLIT) {
          const float2 h01 = unpack_h2(qa[g][ks][0]);
          const float2 h23 = unpack_h2(qa[g][ks][1]);
          qa_lo[g][ks][0] = pack_h2(v[0] - h01.x, v[1] - h01.y);
          qa_lo[g][ks][1] = pack_h2(v[2] - h23.x, v[3] - h23.y);
        }
      }
      part += __shfl_xor_sync(0xffffffffu, part, 1);
      part += __shfl_xor_sync(0xffffffffu, part, 2);
      qsum[g] = part;
    }
  }

  // O[dim][col] accumulators: chunk kk (32 dims), sub-tile sub; rows r / r+8 =
  // dims 32kk + 4r + 2sub (+1); cols 2c, 2c+1 = (head c: hi, lo) when paired,
  // heads 2c, 2c+1 otherwise.
  float o[NCH][2][4];
#pragma unroll
  for (int kk = 0; kk < NCH; ++kk)
#pragma unroll
    for (int s = 0; s < 2; ++s)
#pragma unroll
      for (int e = 0; e < 4; ++e) o[kk][s][e] = 0.0f;
  float m_run = -INFINITY;  // for head hr (K-side layout)
  float l_run = 0.0f;       // partial over this thread's tokens
  float corr[NG];
#pragma unroll
  for (int g = 0; g < NG; ++g) corr[g] = 0.0f;

  const int wt0 = warp * 16;  // this warp's first row of every tile
  const uint32_t smem_base = smem_addr(smem);

  for (int i = 0; i < ntiles; ++i) {
    const int st = i % kMStages;
    const unsigned char* stg = smem + st * Lyt::STAGE;
    const uint32_t stg_addr = smem_base + st * Lyt::STAGE;
    const SB* s_ks = reinterpret_cast<const SB*>(stg + 2 * Lyt::CODE);
    const SB* s_kb = s_ks + kMTile * NG;
    const SB* s_vs = s_kb + kMTile * NG;
    const SB* s_vb = s_vs + kMTile * NG;
    const int tile_t0 = (tile_begin + i) * kMTile;
    mbar_wait_bounded(&full[st], static_cast<uint32_t>((i / kMStages) & 1), p.err);

    // ---- K side: S[head][token], then the scores of (head hr, tokens
    // 8nt + 2c + e), one n-tile at a time to keep few accumulators live -------
    float sc[2][2];
    float bmax = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      const int trow = wt0 + 8 * nt + r;  // token (B-operand column r) of this n-tile
      float acc[NG][4];
#pragma unroll
      for (int g = 0; g < NG; ++g) {
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[g][e] = 0.0f;
        const int word = 8 * g + 2 * c;
        const uint2 wv = *reinterpret_cast<const uint2*>(stg + swz<D>(trow, word >> 2) + 4 * (word & 3));
        mma16816(acc[g], qa[g][0][0], 0u, qa[g][0][1], 0u, nib2h<0>(wv.x), nib2h<1>(wv.x));
        mma16816(acc[g], qa[g][1][0], 0u, qa[g][1][1], 0u, nib2h<2>(wv.x), nib2h<3>(wv.x));
        mma16816(acc[g], qa[g][2][0], 0u, qa[g][2][1], 0u, nib2h<0>(wv.y), nib2h<1>(wv.y));
        mma16816(acc[g], qa[g][3][0], 0u, qa[g][3][1], 0u, nib2h<2>(wv.y), nib2h<3>(wv.y));
        if constexpr (QSPLIT) {
          mma16816(acc[g], qa_lo[g][0][0], 0u, qa_lo[g][0][1], 0u, nib2h<0>(wv.x), nib2h<1>(wv.x));
          mma16816(acc[g], qa_lo[g][1][0], 0u, qa_lo[g][1][1], 0u, nib2h<2>(wv.x), nib2h<3>(wv.x));
          mma16816(acc[g], qa_lo[g][2][0], 0u, qa_lo[g][2][1], 0u, nib2h<0>(wv.y), nib2h<1>(wv.y));
          mma16816(acc[g], qa_lo[g][3][0], 0u, qa_lo[g][3][1], 0u, nib2h<2>(wv.y), nib2h<3>(wv.y));
        }
      }
      const int tt = wt0 + 8 * nt + 2 * c;
      float sk[2][NG], bk[2][NG];
      load_sb2<SB, NG>(s_ks + tt * NG, sk);
      load_sb2<SB, NG>(s_kb + tt * NG, bk);
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        float s = 0.0f;
#pragma unroll
        for (int g = 0; g < NG; ++g)
          s += sk[e][g] * (16.0f * acc[g][e] - 16.0f * qsum[g]) + bk[e][g] * qsum[g];
        const int tg = tile_t0 + tt + e;
        const bool ok = hr_ok && tg >= t_lo && tg < t_hi;
        sc[nt][e] = ok ? s * p.qscale : -INFINITY;
        bmax = fmaxf(bmax, sc[nt][e]);
      }
    }
    bmax = fmaxf(bmax, __shfl_xor_sync(0xffffffffu, bmax, 1));
    bmax = fmaxf(bmax, __shfl_xor_sync(0xffffffffu, bmax, 2));

    // ---- online softmax for head hr -------------------------------------------
    const float m_new = fmaxf(m_run, bmax);
    const float alpha = (m_new == -INFINITY) ? 1.0f : fast_exp2(m_run - m_new);
    m_run = m_new;
    float pr[2][2];
    float lsum = 0.0f;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        pr[nt][e] = (sc[nt][e] == -INFINITY) ? 0.0f : fast_exp2(sc[nt][e] - m_new);
        lsum += pr[nt][e];
      }
    l_run = l_run * alpha + lsum;

    // weights w = p*s (V-side B operand, hi/lo) and the constant correction
    uint32_t bw[NG][2];
    uint32_t bw_lo[kPaired ? 1 : NG][2];
#pragma unroll
    for (int g = 0; g < NG; ++g) corr[g] *= alpha;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      const int tt = wt0 + 8 * nt + 2 * c;
      float sv[2][NG], bv[2][NG];
      load_sb2<SB, NG>(s_vs + tt * NG, sv);
      load_sb2<SB, NG>(s_vb + tt * NG, bv);
#pragma unroll
      for (int g = 0; g < NG; ++g) {
        // masked tokens have p == 0 but their scales may be stale: select
        const float w0 = pr[nt][0] > 0.0f ? pr[nt][0] * sv[0][g] : 0.0f;
        const float w1 = pr[nt][1] > 0.0f ? pr[nt][1] * sv[1][g] : 0.0f;
        corr[g] += (pr[nt][0] > 0.0f ? pr[nt][0] * (bv[0][g] - 16.0f * sv[0][g]) : 0.0f) +
                   (pr[nt][1] > 0.0f ? pr[nt][1] * (bv[1][g] - 16.0f * sv[1][g]) : 0.0f);
        const uint32_t hi = pack_h2(w0, w1);
        const float2 hf = unpack_h2(hi);
        const uint32_t lo = pack_h2(w0 - hf.x, w1 - hf.y);
        if constexpr (kPaired) {
          bw[g][nt] = (r & 1) ? lo : hi;
        } else {
          bw[g][nt] = hi;
          bw_lo[g][nt] = lo;
        }
      }
    }

    // rescale O when any head's max moved (warp-uniform decision)
    if (__any_sync(0xffffffffu, alpha != 1.0f)) {
      float a0, a1;
      if constexpr (kPaired) {
        a0 = a1 = __shfl_sync(0xffffffffu, alpha, 8 * c);
      } else {
        a0 = __shfl_sync(0xffffffffu, alpha, 8 * c);
        a1 = __shfl_sync(0xffffffffu, alpha, 8 * c + 4);
      }
#pragma unroll
      for (int kk = 0; kk < NCH; ++kk)
#pragma unroll
        for (int s = 0; s < 2; ++s) {
          o[kk][s][0] *= a0;
          o[kk][s][1] *= a1;
          o[kk][s][2] *= a0;
          o[kk][s][3] *= a1;
        }
    }

    // ---- V side: O += V^T * w -------------------------------------------------
    const uint32_t vbase = stg_addr + Lyt::CODE;
    const int mi = lane >> 3;  // ldmatrix matrix served by this lane's row address
    const int mrow = lane & 7;
#pragma unroll
    for (int q2 = 0; q2 < NCH / 2; ++q2) {
      // matrices: (chunk 2q2, tokens 0-7), (2q2, 8-15), (2q2+1, 0-7), (2q2+1, 8-15)
      const int kk_l = 2 * q2 + (mi >> 1);
      const int trow = wt0 + 8 * (mi & 1) + mrow;
      uint32_t d[4];
      ldsm_x4_trans(vbase + swz<D>(trow, kk_l), d);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int kk = 2 * q2 + h;
        const int g = kk >> 1;
        const uint32_t R0 = d[2 * h], R1 = d[2 * h + 1];
        mma16816(o[kk][0], nib2h<0>(R0), nib2h<1>(R0), nib2h<0>(R1), nib2h<1>(R1), bw[g][0], bw[g][1]);
        mma16816(o[kk][1], nib2h<2>(R0), nib2h<3>(R0), nib2h<2>(R1), nib2h<3>(R1), bw[g][0], bw[g][1]);
        if constexpr (!kPaired) {
          mma16816(o[kk][0], nib2h<0>(R0), nib2h<1>(R0), nib2h<0>(R1), nib2h<1>(R1), bw_lo[g][0], bw_lo[g][1]);
          mma16816(o[kk][1], nib2h<2>(R0), nib2h<3>(R0), nib2h<2>(R1), nib2h<3>(R1), bw_lo[g][0], bw_lo[g][1]);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);
  }

  // ---- combine the 4 consumer warps -------------------------------------------
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
#pragma unroll
  for (int g = 0; g < NG; ++g) {
    corr[g] += __shfl_xor_sync(0xffffffffu, corr[g], 1);
    corr[g] += __shfl_xor_sync(0xffffffffu, corr[g], 2);
  }
  consumers_sync();  // every warp is past its last tile: the stage area is free
  float* wst = reinterpret_cast<float*>(smem) + warp * Lyt::WST;  // [G][2 + NG + D]
  if (c == 0 && hr_ok && (!kPaired || (r & 1) == 0)) {
    float* hs = wst + hr * (2 + NG + D);
    hs[0] = m_run;
    hs[1] = l_run;
#pragma unroll
    for (int g = 0; g < NG; ++g) hs[2 + g] = corr[g];
  }
#pragma unroll
  for (int kk = 0; kk < NCH; ++kk)
#pragma unroll
    for (int s = 0; s < 2; ++s) {
      const int d0 = 32 * kk + 4 * r + 2 * s;
      if constexpr (kPaired) {
        if (c < G) {
          float* hs = wst + c * (2 + NG + D) + 2 + NG;
          hs[d0] = o[kk][s][0] + o[kk][s][1];
          hs[d0 + 1] = o[kk][s][2] + o[kk][s][3];
        }
      } else {
        float* h0s = wst + (2 * c) * (2 + NG + D) + 2 + NG;
        float* h1s = wst + (2 * c + 1) * (2 + NG + D) + 2 + NG;
        h0s[d0] = o[kk][s][0];
        h0s[d0 + 1] = o[kk][s][2];
        h1s[d0] = o[kk][s][1];
        h1s[d0 + 1] = o[kk][s][3];
      }
    }
  consumers_sync();

  const bool direct = p.splits == 1;
  const long long unit = static_cast<long long>(b) * gridDim.y + hg;
  const float* wall = reinterpret_cast<const float*>(smem);
  for (int it = tid; it < G * D; it += kConsumerWarps * 32) {
    const int g = it / D;
    const int d = it % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, wall[w * Lyt::WST + g * (2 + NG + D)]);
    float L = 0.0f, acc = 0.0f;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) {
      const float* hs = wall + w * Lyt::WST + g * (2 + NG + D);
      const float e = (M == -INFINITY || hs[0] == -INFINITY) ? 0.0f : fast_exp2(hs[0] - M);
      L += e * hs[1];
      acc += e * (16.0f * hs[2 + NG + d] + hs[2 + d / 64]);
    }
    const int h = h0 + g;
    if (direct) {
      if (p.partial) {
        float* blk = p.part_out + static_cast<long long>(b) * p.H * (D + 2);
        blk[static_cast<long long>(h) * D + d] = acc;
        if (d == 0) {
          blk[static_cast<long long>(p.H) * D + 2 * h] = L > 0.0f ? M * kLn2 : -INFINITY;
          blk[static_cast<long long>(p.H) * D + 2 * h + 1] = L;
        }
      } else {
        store_from_float(p.out, (static_cast<long long>(b) * p.H + h) * D + d, p.out_dtype,
                         L > 0.0f ? acc / L : 0.0f);
      }
    } else {
      const long long base = (unit * p.splits + split) * G;
      p.ws_o[(base + g) * D + d] = acc;
      if (d == 0) {
        p.ws_ml[(base + g) * 2] = L > 0.0f ? M : -INFINITY;
        p.ws_ml[(base + g) * 2 + 1] = L;
      }
    }
  }
  if (direct) return;

  // ---- last CTA of this (b, head group) merges the splits -------------------
  __threadfence();
  consumers_sync();
  if (tid == 0) {
    const unsigned prev = atomicAdd(&p.counters[unit], 1u);
    s_flag[0] = (prev == static_cast<unsigned>(p.splits - 1)) ? 1 : 0;
  }
  consumers_sync();
  if (s_flag[0] == 0) return;
  __threadfence();

  constexpr int NT = kConsumerWarps * 32;
  const int S_ = p.splits;
  float* ew = reinterpret_cast<float*>(smem);  // [G][S_]
  const long long base = unit * S_ * G;
  float Mg[G];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float m = -INFINITY;
    for (int s = tid; s < S_; s += NT) m = fmaxf(m, __ldcg(&p.ws_ml[(base + s * G + g) * 2]));
    m = wmax(m);
    if (lane == 0) s_red[warp * G + g] = m;
  }
  consumers_sync();
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float m = s_red[g];
#pragma unroll
    for (int ww = 1; ww < kConsumerWarps; ++ww) m = fmaxf(m, s_red[ww * G + g]);
    Mg[g] = m;
  }
  consumers_sync();
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float l = 0.0f;
    for (int s = tid; s < S_; s += NT) {
      const float ms = __ldcg(&p.ws_ml[(base + s * G + g) * 2]);
      const float ls = __ldcg(&p.ws_ml[(base + s * G + g) * 2 + 1]);
      const float e = (ms == -INFINITY || Mg[g] == -INFINITY) ? 0.0f : fast_exp2(ms - Mg[g]);
      ew[g * S_ + s] = e;
      l += e * ls;
    }
    l = wsum(l);
    if (lane == 0) s_red[4 * G + warp * G + g] = l;
  }
  consumers_sync();
  for (int it = tid; it < G * D; it += NT) {
    const int g = it / D;
    const int d = it % D;
    float L = 0.0f;
#pragma unroll
    for (int ww = 0; ww < kConsumerWarps; ++ww) L += s_red[4 * G + ww * G + g];
    float acc = 0.0f;
    for (int s = 0; s < S_; ++s) acc += ew[g * S_ + s] * __ldcg(&p.ws_o[(base + s * G + g) * D + d]);
    const int h = h0 + g;
    float Mv = Mg[0];
#pragma unroll
    for (int gg = 1; gg < G; ++gg) Mv = (g == gg) ? Mg[gg] : Mv;
    if (p.partial) {
      float* blk = p.part_out + static_cast<long long>(b) * p.H * (D + 2);
      blk[static_cast<long long>(h) * D + d] = acc;
      if (d == 0) {
        blk[static_cast<long long>(p.H) * D + 2 * h] = L > 0.0f ? Mv * kLn2 : -INFINITY;
        blk[static_cast<long long>(p.H) * D + 2 * h + 1] = L;
      }
    } else {
      store_from_float(p.out, (static_cast<long long>(b) * p.H + h) * D + d, p.out_dtype,
                       L > 0.0f ? acc / L : 0.0f);
    }
  }
  if (tid == 0) p.counters[unit] = 0u;
}

// ---- host side ----------------------------------------------------------------

using MKernelFn = void (*)(CUtensorMap, CUtensorMap, MParams);

struct MKernelInfo {
  MKernelFn fn = nullptr;
  int smem = 0;
};

template <int D, int G, typename SB>
MKernelInfo mk(bool qsplit) {
  MKernelInfo k;
  k.fn = qsplit ? decode_mma_kernel<D, G, SB, true> : decode_mma_kernel<D, G, SB, false>;
  k.smem = MLayout<D, G, SB>::BYTES;
  return k;
}

template <int D, typename SB>
MKernelInfo mk_g(int g, bool qsplit) {
  switch (g) {
    case 1: return mk<D, 1, SB>(qsplit);
    case 2: return mk<D, 2, SB>(qsplit);
    case 4: return mk<D, 4, SB>(qsplit);
    case 8: return mk<D, 8, SB>(qsplit);
    default: return MKernelInfo{};
  }
}

MKernelInfo pick_mma(int D, int gsub, int sb_dtype, bool qsplit) {
  const bool f32 = sb_dtype == kF32;
  if (D == 128) return f32 ? mk_g<128, float>(gsub, qsplit) : mk_g<128, __half>(gsub, qsplit);
  if (D == 256) return f32 ? mk_g<256, float>(gsub, qsplit) : mk_g<256, __half>(gsub, qsplit);
  return MKernelInfo{};
}

std::mutex g_mmu;
std::unordered_map<long long, int> g_mocc;

int mma_blocks_per_sm(int device, const MKernelInfo& k) {
  const long long key = (static_cast<long long>(device) << 48) ^ reinterpret_cast<long long>(k.fn);
  std::lock_guard<std::mutex> lock(g_mmu);
  auto it = g_mocc.find(key);
  if (it != g_mocc.end()) return it->second;
  cudaFuncSetAttribute(k.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, k.smem);
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k.fn, kMThreads, k.smem) != cudaSuccess || n < 1)
    n = 1;
  g_mocc[key] = n;
  return n;
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  });
  return fn;
}

bool encode_codes_map(CUtensorMap* m, const uint32_t* base, int D, long long rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(D / 8), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(D / 2)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(D == 128 ? 16 : 32), static_cast<cuuint32_t>(kMTile)};
  cuuint32_t estr[2] = {1, 1};
  const CUtensorMapSwizzle swz = D == 128 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B;
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<uint32_t*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

}  // namespace

bool mma_supported(int D, int G) { return (D == 128 || D == 256) && G >= 1 && G <= 8 && (G & (G - 1)) == 0; }

int mma_tokens_per_tile() { return kMTile; }

int mma_occupancy(int device, int D, int gsub) {
  MKernelInfo k = pick_mma(D, gsub, kF16, false);
  return k.fn ? mma_blocks_per_sm(device, k) : 1;
}

cudaError_t launch_decode_mma(const DecodeArgs& a, const DecodePlan& pl, cudaStream_t stream) {
  const bool qsplit = a.q_dtype != kF16;
  MKernelInfo k = pick_mma(a.D, pl.gsub, a.sb_dtype, qsplit);
  if (!k.fn) return cudaErrorInvalidValue;
  int device = 0;
  cudaGetDevice(&device);
  mma_blocks_per_sm(device, k);
  const long long rows = static_cast<long long>(a.B) * a.bstride_tok;
  if (rows >= (1LL << 31)) return cudaErrorInvalidValue;
  CUtensorMap tmk, tmv;
  if (!encode_codes_map(&tmk, a.kq, a.D, rows) || !encode_codes_map(&tmv, a.vq, a.D, rows))
    return cudaErrorInvalidValue;
  MParams p{};
  p.q = a.q;
  p.q_dtype = a.q_dtype;
  p.ks = a.ks;
  p.kb = a.kb;
  p.vs = a.vs;
  p.vb = a.vb;
  p.seq_lens = a.seq_lens;
  p.n_tokens = a.n_tokens;
  p.H = a.H;
  p.Hkv = a.Hkv;
  p.Gtot = a.G;
  p.nsub = pl.nsub;
  p.capacity = a.capacity;
  p.bstride_tok = a.bstride_tok;
  p.qscale = a.scale * kLog2e;
  p.window = a.window;
  p.token_offset = a.token_offset;
  p.n_total = a.n_total;
  p.partial = a.partial;
  p.out = a.out;
  p.out_dtype = a.out_dtype;
  p.part_out = a.part_out;
  p.splits = pl.splits;
  p.tiles_per_split = pl.tiles_per_split;
  if (pl.splits > 1) {
    unsigned char* ws = static_cast<unsigned char*>(a.workspace);
    p.ws_o = reinterpret_cast<float*>(ws + pl.ws_o_off);
    p.ws_ml = reinterpret_cast<float*>(ws + pl.ws_ml_off);
    p.counters = reinterpret_cast<unsigned*>(ws + pl.ws_cnt_off);
  }
  p.err = a.err;
  dim3 grid(pl.splits, a.Hkv * pl.nsub, a.B);
  k.fn<<<grid, kMThreads, k.smem, stream>>>(tmk, tmv, p);
  return cudaGetLastError();
}

}  // namespace tq
