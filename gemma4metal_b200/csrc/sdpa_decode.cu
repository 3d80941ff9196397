// Split-KV single-query decode attention straight from the int4 KV cache.
//
// Replaces the reference's sdpa_int4_vector<D,BN> (lib/turboquant.metal:723-903,
// dispatched by lib/turboquant.cpp:367-403) with a B200 design:
//   * grid = (splits, KV-head groups, batch): one CTA streams a contiguous
//     token range of ONE KV head and serves all of its GQA query heads, so each
//     packed byte crosses HBM once (the reference launches one threadgroup per
//     query head and re-reads the KV head gqa times: lib/turboquant.cpp:400);
//   * tiles of T = 8192/D tokens (9 KB of codes+scales+biases) are staged into
//     shared memory by 1-D TMA bulk copies (cp.async.bulk + mbarrier), four
//     stages deep;
//   * K phase: token-parallel; each thread dots WK code words against the
//     query kept in registers (packed fp32x2 FMA, nibbles turned into floats
//     with the 2^23 mantissa trick, no I2F); the scale/bias of each 64-group is
//     factored out: score = s * sum(q*c) + b * sum(q) (the reference does the
//     same at lib/turboquant.metal:803);
//   * softmax phase: exact tile max, exp2 in log2 units, per-(token,group)
//     weights p*s and p*b written to shared memory;
//   * V phase: dimension-parallel; o += (p*s) * c, sum(p*b) kept per thread;
//   * the last CTA of each KV head (atomic ticket) merges the split partials
//     with a log-sum-exp merge and writes the output (or the partial state
//     when the caller asked for it, for the multi-GPU sequence split).
// All waits on barriers are bounded (see mbar_wait_bounded).
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <unordered_map>

#include "tq_common.cuh"
#include "tq_internal.h"

namespace tq {

namespace {

constexpr int kThreads = 128;
constexpr int kStages = 4;
constexpr int kMaxSplits = 1024;
constexpr int kMinBlocksPerSM = 3;
}  // namespace
const size_t kCounterRegionBytes = 64 * 1024;  // 16384 merge counters
namespace {

template <int D, int G>
struct Cfg {
  static constexpr int T = 8192 / D;          // tokens per tile
  static constexpr int WPT = D / 8;           // code words per token (K or V)
  static constexpr int NG = D / 64;           // 64-groups per token
  static constexpr int WK = 8 / G;            // K-phase words per thread (q regs = 8*WK*G = 64)
  static constexpr int LPT = WPT / WK;        // K-phase threads per token
  static constexpr int KTOK = kThreads / LPT; // tokens per K pass
  static constexpr int KP = T / KTOK;         // K passes per tile
  static constexpr int WV = G >= 4 ? 1 : 4 / G;  // V-phase words per thread
  static constexpr int VL = WPT / WV;         // V-phase threads per token
  static constexpr int VTOK = kThreads / VL;  // tokens per V pass
  static constexpr int VP = T / VTOK;         // V passes per tile
  static_assert(LPT <= 32, "a token's K words must stay inside one warp");
  static_assert(KP * KTOK == T && VP * VTOK == T, "tile mapping");
  static_assert(WK * 8 <= 64 && 8 % WK == 0, "K words of a thread stay in one group");
  static_assert(WV * 8 <= 64, "V words of a thread stay in one group");
};

struct KParams {
  const void* q;
  int q_dtype;
  const uint32_t* kq;
  const void* ks;
  const void* kb;
  const uint32_t* vq;
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

template <int D, int G, typename SB>
struct Smem {
  using C = Cfg<D, G>;
  static constexpr int kCodeBytes = C::T * D / 2;
  static constexpr int kSbBytes = C::T * C::NG * static_cast<int>(sizeof(SB));
  static constexpr int kStageBytes = 2 * kCodeBytes + 4 * kSbBytes;
  static constexpr int kStagesBytes = kStages * kStageBytes;
  static constexpr int kScOff = kStagesBytes;                       // float [T][G]
  static constexpr int kWbOff = kScOff + C::T * G * 4;              // float2 [T][NG][G]
  static constexpr int kRedOff = kWbOff + C::T * C::NG * G * 8;     // float [4][G] x 2
  static constexpr int kFlagOff = kRedOff + 2 * 4 * G * 4;          // int
  static constexpr int kBarOff = (kFlagOff + 16 + 7) / 8 * 8;       // uint64 [kStages]
  static constexpr int kBytes = kBarOff + kStages * 8;
  static constexpr int kReduceBytes = C::VTOK * G * D * 4;          // final o reduction
  static_assert(kReduceBytes <= kStagesBytes, "reduction buffer reuses the stages");
  static_assert(G * kMaxSplits * 4 <= kStagesBytes, "merge weights reuse the stages");
};

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <int WK>
__device__ __forceinline__ void load_words(const uint32_t* src, uint32_t (&w)[WK]) {
  if constexpr (WK == 8) {
    const uint4 a = reinterpret_cast<const uint4*>(src)[0];
    const uint4 b = reinterpret_cast<const uint4*>(src)[1];
    w[0] = a.x; w[1] = a.y; w[2] = a.z; w[3] = a.w;
    w[4] = b.x; w[5] = b.y; w[6] = b.z; w[7] = b.w;
  } else if constexpr (WK == 4) {
    const uint4 a = *reinterpret_cast<const uint4*>(src);
    w[0] = a.x; w[1] = a.y; w[2] = a.z; w[3] = a.w;
  } else if constexpr (WK == 2) {
    const uint2 a = *reinterpret_cast<const uint2*>(src);
    w[0] = a.x; w[1] = a.y;
  } else {
    w[0] = *src;
  }
}

template <int D, int G, typename SB>
__global__ void __launch_bounds__(kThreads, G >= 8 ? 2 : kMinBlocksPerSM) decode_kernel(const KParams p) {
  using C = Cfg<D, G>;
  using S = Smem<D, G, SB>;
  extern __shared__ __align__(128) unsigned char smem[];
  float* s_sc = reinterpret_cast<float*>(smem + S::kScOff);
  float2* s_wb = reinterpret_cast<float2*>(smem + S::kWbOff);
  float* s_red = reinterpret_cast<float*>(smem + S::kRedOff);
  int* s_flag = reinterpret_cast<int*>(smem + S::kFlagOff);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::kBarOff);

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int split = blockIdx.x;
  const int hg = blockIdx.y;
  const int b = blockIdx.z;
  const int kv = hg / p.nsub;
  const int h0 = kv * p.Gtot + (hg % p.nsub) * G;  // first query head served

  // ---- visible token range in local cache coordinates ----------------------
  // device-provided lengths are clamped so every copy stays inside the cache
  const int n_local = max(0, min(p.seq_lens ? p.seq_lens[b] : p.n_tokens, p.capacity));
  int t_lo = 0;
  const int t_hi = n_local;
  if (p.window > 0) {
    const int n_glob = p.n_total > 0 ? p.n_total : n_local + p.token_offset;
    t_lo = max(0, n_glob - p.window - p.token_offset);
  }
  int ntiles = 0, tile_begin = 0;
  if (t_hi > t_lo) {
    const int tb = t_lo / C::T;
    const int te = (t_hi + C::T - 1) / C::T;
    tile_begin = tb + split * p.tiles_per_split;
    const int tile_end = min(te, tile_begin + p.tiles_per_split);
    ntiles = max(0, tile_end - tile_begin);
  }
  const int t_hi4 = (t_hi + 3) & ~3;

  const long long tok_base = static_cast<long long>(b) * p.bstride_tok +
                             static_cast<long long>(kv) * p.capacity;
  const uint32_t* kq_base = p.kq + tok_base * C::WPT;
  const uint32_t* vq_base = p.vq + tok_base * C::WPT;
  const SB* ks_base = reinterpret_cast<const SB*>(p.ks) + tok_base * C::NG;
  const SB* kb_base = reinterpret_cast<const SB*>(p.kb) + tok_base * C::NG;
  const SB* vs_base = reinterpret_cast<const SB*>(p.vs) + tok_base * C::NG;
  const SB* vb_base = reinterpret_cast<const SB*>(p.vb) + tok_base * C::NG;

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) mbar_init(&bars[s], 1);
    fence_barrier_init();
  }

  // ---- query (K-phase layout) in registers ----------------------------------
  const int kqi = tid % C::LPT;        // which WK-word chunk of the token
  const int ktok = tid / C::LPT;       // token within a K pass
  const int kgrp = kqi * C::WK / 8;    // 64-group of that chunk
  float2 qq[G][C::WK * 4];
  float qs[G];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const long long qrow = (static_cast<long long>(b) * p.H + h0 + g) * D;
    float sum = 0.0f;
#pragma unroll
    for (int wi = 0; wi < C::WK; ++wi) {
#pragma unroll
      for (int pr = 0; pr < 4; ++pr) {
        const int d0 = (kqi * C::WK + wi) * 8 + 2 * pr;
        const float a0 = load_as_float(p.q, qrow + d0, p.q_dtype) * p.qscale;
        const float a1 = load_as_float(p.q, qrow + d0 + 1, p.q_dtype) * p.qscale;
        sum += a0 + a1;
        qq[g][wi * 4 + pr] = make_float2(ldexpf(a0, -nib_exp(2 * pr)), ldexpf(a1, -nib_exp(2 * pr + 1)));
      }
    }
    qs[g] = sum;
  }

  __syncthreads();  // barriers initialised

  const uint64_t pol = policy_evict_first();
  auto issue = [&](int rel, int st) {
    const int t0 = (tile_begin + rel) * C::T;
    const int nt = min(C::T, t_hi4 - t0);
    const uint32_t cb = static_cast<uint32_t>(nt * D / 2);
    const uint32_t sbb = static_cast<uint32_t>(nt * C::NG * sizeof(SB));
    unsigned char* st_base = smem + st * S::kStageBytes;
    mbar_arrive_expect_tx(&bars[st], 2 * cb + 4 * sbb);
    bulk_g2s(st_base, kq_base + static_cast<long long>(t0) * C::WPT, cb, &bars[st], pol);
    bulk_g2s(st_base + S::kCodeBytes, vq_base + static_cast<long long>(t0) * C::WPT, cb, &bars[st], pol);
    unsigned char* sbp = st_base + 2 * S::kCodeBytes;
    bulk_g2s(sbp, ks_base + static_cast<long long>(t0) * C::NG, sbb, &bars[st], pol);
    bulk_g2s(sbp + S::kSbBytes, kb_base + static_cast<long long>(t0) * C::NG, sbb, &bars[st], pol);
    bulk_g2s(sbp + 2 * S::kSbBytes, vs_base + static_cast<long long>(t0) * C::NG, sbb, &bars[st], pol);
    bulk_g2s(sbp + 3 * S::kSbBytes, vb_base + static_cast<long long>(t0) * C::NG, sbb, &bars[st], pol);
  };
  if (tid == 0) {
    for (int s = 0; s < kStages && s < ntiles; ++s) issue(s, s);
  }

  // ---- running state --------------------------------------------------------
  const int vw = tid % C::VL;          // V-phase word chunk
  const int vt = tid / C::VL;          // token within a V pass
  const int vgrp = vw * C::WV / 8;
  float2 o2[G][C::WV * 4];
  float bacc[G];
  float m_run[G];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    bacc[g] = 0.0f;
    m_run[g] = -INFINITY;
#pragma unroll
    for (int k = 0; k < C::WV * 4; ++k) o2[g][k] = make_float2(0.0f, 0.0f);
  }
  float l_acc = 0.0f;  // softmax denominator for head g = tid % G

  for (int i = 0; i < ntiles; ++i) {
    const int st = i % kStages;
    const unsigned char* st_base = smem + st * S::kStageBytes;
    const uint32_t* s_kc = reinterpret_cast<const uint32_t*>(st_base);
    const uint32_t* s_vc = reinterpret_cast<const uint32_t*>(st_base + S::kCodeBytes);
    const SB* s_ks = reinterpret_cast<const SB*>(st_base + 2 * S::kCodeBytes);
    const SB* s_kb = s_ks + C::T * C::NG;
    const SB* s_vs = s_kb + C::T * C::NG;
    const SB* s_vb = s_vs + C::T * C::NG;
    const int tile_t0 = (tile_begin + i) * C::T;

    mbar_wait_bounded(&bars[st], static_cast<uint32_t>((i / kStages) & 1), p.err);

    // ---- K phase: scores of the tile -----------------------------------------
    float tmax[G];
#pragma unroll
    for (int g = 0; g < G; ++g) tmax[g] = -INFINITY;
#pragma unroll
    for (int kp = 0; kp < C::KP; ++kp) {
      const int t = kp * C::KTOK + ktok;
      uint32_t w[C::WK];
      load_words<C::WK>(s_kc + t * C::WPT + kqi * C::WK, w);
      float2 acc[G];
#pragma unroll
      for (int g = 0; g < G; ++g) acc[g] = make_float2(0.0f, 0.0f);
#pragma unroll
      for (int wi = 0; wi < C::WK; ++wi) {
        float2 c[4];
        unpack_word(w[wi], c);
#pragma unroll
        for (int pr = 0; pr < 4; ++pr) {
#pragma unroll
          for (int g = 0; g < G; ++g) acc[g] = __ffma2_rn(qq[g][wi * 4 + pr], c[pr], acc[g]);
        }
      }
      const float sk = sb_to_float<SB>(s_ks[t * C::NG + kgrp]);
      const float bk = sb_to_float<SB>(s_kb[t * C::NG + kgrp]);
      const int tg = tile_t0 + t;
      const bool valid = tg >= t_lo && tg < t_hi;
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float part = sk * (acc[g].x + acc[g].y) + bk * qs[g];
#pragma unroll
        for (int o = 1; o < C::LPT; o <<= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
        const float sc = valid ? part : -INFINITY;
        if (kqi == 0) s_sc[t * G + g] = sc;
        tmax[g] = fmaxf(tmax[g], sc);
      }
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float m = warp_max(tmax[g]);
      if (lane == 0) s_red[warp * G + g] = m;
    }
    __syncthreads();  // A: scores + warp maxima visible; stage of tile i-1 free

    if (tid == 0 && i >= 1 && i - 1 + kStages < ntiles) issue(i - 1 + kStages, (i - 1) % kStages);

    // ---- softmax phase -------------------------------------------------------
    float alpha[G];
    float m_new[G];
    bool rescale = false;
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float mt = s_red[g];
#pragma unroll
      for (int ww = 1; ww < kThreads / 32; ++ww) mt = fmaxf(mt, s_red[ww * G + g]);
      m_new[g] = fmaxf(m_run[g], mt);
      alpha[g] = (m_new[g] == -INFINITY) ? 1.0f : fast_exp2(m_run[g] - m_new[g]);
      rescale |= alpha[g] != 1.0f;
      m_run[g] = m_new[g];
    }
    {
      const int g = tid % G;
      float mg = m_new[0];
#pragma unroll
      for (int gg = 1; gg < G; ++gg) mg = (g == gg) ? m_new[gg] : mg;
      float lsum = 0.0f;
      for (int it = tid; it < C::T * G; it += kThreads) {
        const int t = it / G;
        const float sc = s_sc[t * G + g];
        const bool live = sc != -INFINITY;
        const float pr = live ? fast_exp2(sc - mg) : 0.0f;
        lsum += pr;
#pragma unroll
        for (int grp = 0; grp < C::NG; ++grp) {
          const float vsv = sb_to_float<SB>(s_vs[t * C::NG + grp]);
          const float vbv = sb_to_float<SB>(s_vb[t * C::NG + grp]);
          s_wb[(t * C::NG + grp) * G + g] =
              live ? make_float2(pr * vsv, pr * vbv) : make_float2(0.0f, 0.0f);
        }
      }
      float ag = alpha[0];
#pragma unroll
      for (int gg = 1; gg < G; ++gg) ag = (g == gg) ? alpha[gg] : ag;
      l_acc = ag * l_acc + lsum;
    }
    __syncthreads();  // B: weights visible

    // ---- V phase -------------------------------------------------------------
    if (rescale) {
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float2 a2 = make_float2(alpha[g], alpha[g]);
        bacc[g] *= alpha[g];
#pragma unroll
        for (int k = 0; k < C::WV * 4; ++k) o2[g][k] = __fmul2_rn(o2[g][k], a2);
      }
    }
#pragma unroll
    for (int vp = 0; vp < C::VP; ++vp) {
      const int t = vp * C::VTOK + vt;
      uint32_t w[C::WV];
      load_words<C::WV>(s_vc + t * C::WPT + vw * C::WV, w);
      float2 wb[G];
#pragma unroll
      for (int g = 0; g < G; ++g) wb[g] = s_wb[(t * C::NG + vgrp) * G + g];
#pragma unroll
      for (int wi = 0; wi < C::WV; ++wi) {
        float2 c[4];
        unpack_word(w[wi], c);
#pragma unroll
        for (int pr = 0; pr < 4; ++pr) {
#pragma unroll
          for (int g = 0; g < G; ++g)
            o2[g][wi * 4 + pr] = __ffma2_rn(make_float2(wb[g].x, wb[g].x), c[pr], o2[g][wi * 4 + pr]);
        }
      }
#pragma unroll
      for (int g = 0; g < G; ++g) bacc[g] += wb[g].y;
    }
  }

  // ---- combine the CTA's threads ---------------------------------------------
  __syncthreads();  // all stages consumed: the stage area is free
  float* red = reinterpret_cast<float*>(smem);  // [VTOK][G][D]
#pragma unroll
  for (int g = 0; g < G; ++g) {
#pragma unroll
    for (int wi = 0; wi < C::WV; ++wi) {
#pragma unroll
      for (int pr = 0; pr < 4; ++pr) {
        const int d0 = (vw * C::WV + wi) * 8 + 2 * pr;
        const float2 v = o2[g][wi * 4 + pr];
        red[(vt * G + g) * D + d0] = ldexpf(v.x, -nib_exp(2 * pr)) + bacc[g];
        red[(vt * G + g) * D + d0 + 1] = ldexpf(v.y, -nib_exp(2 * pr + 1)) + bacc[g];
      }
    }
  }
  // l: sum over the threads that share g = tid % G
  {
    float l = l_acc;
#pragma unroll
    for (int o = G; o < 32; o <<= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
    if (lane < G) s_red[4 * G + warp * G + lane] = l;
  }
  __syncthreads();
  float l_tot[G];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float l = 0.0f;
#pragma unroll
    for (int ww = 0; ww < kThreads / 32; ++ww) l += s_red[4 * G + ww * G + g];
    l_tot[g] = l;
  }

  const bool direct = p.splits == 1;
  const long long unit = static_cast<long long>(b) * gridDim.y + hg;  // (b, head group)
  for (int it = tid; it < G * D; it += kThreads) {
    const int g = it / D;
    const int d = it % D;
    float acc = 0.0f;
#pragma unroll 4
    for (int r = 0; r < C::VTOK; ++r) acc += red[(r * G + g) * D + d];
    float lg = l_tot[0];
    float mg = m_run[0];
#pragma unroll
    for (int gg = 1; gg < G; ++gg) {
      lg = (g == gg) ? l_tot[gg] : lg;
      mg = (g == gg) ? m_run[gg] : mg;
    }
    if (direct) {
      const int h = h0 + g;
      if (p.partial) {
        float* blk = p.part_out + static_cast<long long>(b) * p.H * (D + 2);
        blk[static_cast<long long>(h) * D + d] = acc;
        if (d == 0) {
          blk[static_cast<long long>(p.H) * D + 2 * h] = lg == 0.0f ? -INFINITY : mg * kLn2;
          blk[static_cast<long long>(p.H) * D + 2 * h + 1] = lg;
        }
      } else {
        store_from_float(p.out, (static_cast<long long>(b) * p.H + h) * D + d, p.out_dtype,
                         lg == 0.0f ? 0.0f : acc / lg);
      }
    } else {
      const long long base = (unit * p.splits + split) * G;
      p.ws_o[(base + g) * D + d] = acc;
      if (d == 0) {
        p.ws_ml[(base + g) * 2] = lg == 0.0f ? -INFINITY : mg;
        p.ws_ml[(base + g) * 2 + 1] = lg;
      }
    }
  }
  if (direct) return;

  // ---- last CTA of this (b, head group) merges the splits -------------------
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const unsigned prev = atomicAdd(&p.counters[unit], 1u);
    s_flag[0] = (prev == static_cast<unsigned>(p.splits - 1)) ? 1 : 0;
  }
  __syncthreads();
  if (s_flag[0] == 0) return;
  __threadfence();

  const int S_ = p.splits;
  float* ew = reinterpret_cast<float*>(smem);  // [G][S_] merge weights
  const long long base = unit * S_ * G;
  float Mg[G];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float m = -INFINITY;
    for (int s = tid; s < S_; s += kThreads) m = fmaxf(m, __ldcg(&p.ws_ml[(base + s * G + g) * 2]));
    m = warp_max(m);
    if (lane == 0) s_red[warp * G + g] = m;
  }
  __syncthreads();
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float m = s_red[g];
#pragma unroll
    for (int ww = 1; ww < kThreads / 32; ++ww) m = fmaxf(m, s_red[ww * G + g]);
    Mg[g] = m;
  }
  __syncthreads();
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float l = 0.0f;
    for (int s = tid; s < S_; s += kThreads) {
      const float ms = __ldcg(&p.ws_ml[(base + s * G + g) * 2]);
      const float ls = __ldcg(&p.ws_ml[(base + s * G + g) * 2 + 1]);
      const float e = (ms == -INFINITY || Mg[g] == -INFINITY) ? 0.0f : fast_exp2(ms - Mg[g]);
      ew[g * S_ + s] = e;
      l += e * ls;
    }
    l = warp_sum(l);
    if (lane == 0) s_red[4 * G + warp * G + g] = l;
  }
  __syncthreads();
  for (int it = tid; it < G * D; it += kThreads) {
    const int g = it / D;
    const int d = it % D;
    float L = 0.0f;
#pragma unroll
    for (int ww = 0; ww < kThreads / 32; ++ww) L += s_red[4 * G + ww * G + g];
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
        blk[static_cast<long long>(p.H) * D + 2 * h] = L == 0.0f ? -INFINITY : Mv * kLn2;
        blk[static_cast<long long>(p.H) * D + 2 * h + 1] = L;
      }
    } else {
      store_from_float(p.out, (static_cast<long long>(b) * p.H + h) * D + d, p.out_dtype,
                       L == 0.0f ? 0.0f : acc / L);
    }
  }
  if (tid == 0) p.counters[unit] = 0u;  // ready for the next launch
}

// ---- host side --------------------------------------------------------------

using KernelFn = void (*)(KParams);

template <int D, int G, typename SB>
KernelFn kernel_ptr() {
  return decode_kernel<D, G, SB>;
}

template <int D, int G, typename SB>
int smem_bytes() {
  return Smem<D, G, SB>::kBytes;
}

struct KernelInfo {
  KernelFn fn = nullptr;
  int smem = 0;
  int tokens_per_tile = 0;
};

template <int D, typename SB>
KernelInfo pick_g(int g) {
  KernelInfo k;
  k.tokens_per_tile = 8192 / D;
  switch (g) {
    case 1: k.fn = kernel_ptr<D, 1, SB>(); k.smem = smem_bytes<D, 1, SB>(); break;
    case 2: k.fn = kernel_ptr<D, 2, SB>(); k.smem = smem_bytes<D, 2, SB>(); break;
    case 4: k.fn = kernel_ptr<D, 4, SB>(); k.smem = smem_bytes<D, 4, SB>(); break;
    case 8:
      if constexpr (D <= 256) {
        k.fn = kernel_ptr<D, 8, SB>();
        k.smem = smem_bytes<D, 8, SB>();
      }
      break;
    default: break;
  }
  return k;
}

KernelInfo pick_kernel(int D, int gsub, int sb_dtype) {
  const bool f32 = sb_dtype == kF32;
  switch (D) {
    case 128: return f32 ? pick_g<128, float>(gsub) : pick_g<128, __half>(gsub);
    case 256: return f32 ? pick_g<256, float>(gsub) : pick_g<256, __half>(gsub);
    case 512: return f32 ? pick_g<512, float>(gsub) : pick_g<512, __half>(gsub);
    default: return KernelInfo{};
  }
}

int max_gsub(int D) { return D >= 512 ? 4 : 8; }

std::mutex g_mu;
std::unordered_map<long long, int> g_occ;  // (device, kernel) -> CTAs per SM

int blocks_per_sm(int device, const KernelInfo& k) {
  const long long key = (static_cast<long long>(device) << 48) ^ reinterpret_cast<long long>(k.fn);
  std::lock_guard<std::mutex> lock(g_mu);
  auto it = g_occ.find(key);
  if (it != g_occ.end()) return it->second;
  cudaFuncSetAttribute(k.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, k.smem);
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k.fn, kThreads, k.smem) != cudaSuccess || n < 1)
    n = 1;
  g_occ[key] = n;
  return n;
}

size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

}  // namespace

int device_sm_count(int device) {
  static std::mutex mu;
  static std::unordered_map<int, int> cache;
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(device);
  if (it != cache.end()) return it->second;
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || n < 1)
    n = 148;
  cache[device] = n;
  return n;
}

int choose_decode_variant(int D, int G) {
  const char* env = getenv("TQ_DECODE_KERNEL");
  const bool force_simt = env && strcmp(env, "simt") == 0;
  if (!force_simt && mma_supported(D, std::min(G, 8))) return kDecodeMma;
  return kDecodeSimt;
}

DecodePlan plan_decode(int device, int B, int H, int Hkv, int D, int n_visible_max, bool windowed,
                       bool qsplit) {
  DecodePlan pl{};
  if ((D != 128 && D != 256 && D != 512) || Hkv < 1 || H < Hkv || B < 1) {
    pl.splits = -1;  // not a decode shape (callers validate first; nothing below may divide by 0)
    return pl;
  }
  const int G = H / Hkv;
  pl.variant = choose_decode_variant(D, G);
  pl.gsub = std::min(G, pl.variant == kDecodeMma ? 8 : max_gsub(D));
  pl.nsub = G / pl.gsub;
  pl.tokens_per_tile = pl.variant == kDecodeMma ? mma_tokens_per_tile() : 8192 / D;
  const int T = pl.tokens_per_tile;
  // +1 tile: a window that does not start on a tile boundary spans one more
  const int tiles = std::max(1, (n_visible_max + T - 1) / T + (windowed ? 1 : 0));
  const long long units = static_cast<long long>(B) * Hkv * pl.nsub;
  int per_sm = kMinBlocksPerSM;
  if (device >= 0) {
    // occupancy of the f16-scale kernel (the f32 variant differs by 1 KB smem)
    if (pl.variant == kDecodeMma) {
      per_sm = mma_occupancy(device, D, pl.gsub, qsplit);
    } else {
      KernelInfo k = pick_kernel(D, pl.gsub, kF16);
      if (k.fn) per_sm = blocks_per_sm(device, k);
    }
  }
  const long long target = static_cast<long long>(device_sm_count(device < 0 ? 0 : device)) * per_sm;
  // at most one wave: splits * units <= resident CTAs
  long long splits = target / units;
  splits = std::max<long long>(1, std::min<long long>(splits, tiles));
  int tps = static_cast<int>((tiles + splits - 1) / splits);
  splits = (tiles + tps - 1) / tps;
  if (splits > kMaxSplits) {
    tps = (tiles + kMaxSplits - 1) / kMaxSplits;
    splits = (tiles + tps - 1) / tps;
  }
  pl.splits = static_cast<int>(splits);
  pl.tiles_per_split = tps;
  if (pl.splits > 1) {
    // Merge counters live in a fixed region at the start of every workspace,
    // so that no plan's partials ever overlap another plan's counters: kernels
    // leave counters at zero, partial data is only ever written after them.
    const size_t n_part = static_cast<size_t>(units) * pl.splits * pl.gsub;
    pl.ws_cnt_off = 0;
    pl.ws_o_off = kCounterRegionBytes;
    pl.ws_ml_off = pl.ws_o_off + align256(n_part * D * sizeof(float));
    pl.ws_bytes = pl.ws_ml_off + align256(n_part * 2 * sizeof(float));
    // the tensor-core kernel merges more than 64 splits in two levels, with
    // one more counter per group of 32 splits of a unit
    const long long groups = pl.splits > 64 ? (pl.splits + 31) / 32 : 0;
    if (static_cast<size_t>(units * (1 + groups)) * sizeof(unsigned) > kCounterRegionBytes)
      pl.ws_bytes = 0, pl.splits = -1;
  }
  return pl;
}

cudaError_t launch_decode(const DecodeArgs& a, const DecodePlan& pl, cudaStream_t stream) {
  if (pl.variant == kDecodeMma) return launch_decode_mma(a, pl, stream);
  KernelInfo k = pick_kernel(a.D, pl.gsub, a.sb_dtype);
  if (!k.fn) return cudaErrorInvalidValue;
  int device = 0;
  cudaGetDevice(&device);
  blocks_per_sm(device, k);  // sets the dynamic shared-memory attribute once
  KParams p{};
  p.q = a.q;
  p.q_dtype = a.q_dtype;
  p.kq = a.kq;
  p.ks = a.ks;
  p.kb = a.kb;
  p.vq = a.vq;
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
  k.fn<<<grid, kThreads, k.smem, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace tq
