// Tensor-core (warp-level mma.sync m16n8k16, f16 x f16 -> f32) split-KV decode
// attention straight from the int4 KV cache. Same contract and partial/merge
// format as decode_kernel in sdpa_decode.cu; this variant exists because the
// CUDA-core kernel is instruction-bound at GQA >= 2 (about 2.6 instructions
// per 4-bit code; 54 us at 32K tokens against 20 us here), and a single mma
// consumes 128 (K side) or 256 (V side) 4-bit codes per warp instruction.
//
// Data path per CTA (grid = splits x KV-head groups x batch):
//   * producer warp: 2-D TMA tensor copies of the K and V code tiles
//     (64 tokens x D/2 bytes, 64B/128B-swizzled so the K-side row reads and
//     the transposed ldmatrix reads below are bank-conflict free) + 1-D bulk
//     copies of the fp16 scales/biases, into a full/empty mbarrier ring of 3
//     (D=128) or 5 (D=256) stages (64-token boxes; a CTA's token range is a
//     whole number of boxes);
//   * 4 consumer warps, 32 (D=128) or 16 (D=256) tokens of every tile each
//     (as independent 16-token blocks), each warp with its own online-softmax
//     state (no CTA barrier in the main loop), 3 (D=128) or 2 (D=256) CTAs
//     per SM:
//       K side:  S[token][col] = sum_d (1 + c[token][d]/64) * q[col][d] as
//                mma(A = codes, rows = tokens; B = q). The codes become exact
//                fp16 values 1 + c/64 with one LOP3 (and at most one shift)
//                per two nibbles; every B column holds one query head on a
//                subset of the dims, so all 8 columns work at any GQA factor
//                and a cheap in-register/one-shuffle sum completes the dot
//                products. The offset is removed through sum_d q:
//                score = s*64*(S - sum q) + b*sum q per 64-group;
//       softmax: exp2 in log2 units, one (head, token) item per lane at
//                GQA <= 2; weights w = p*s split into fp16 hi+lo (22
//                significant bits) and moved to the V-side B layout with four
//                shuffles per group;
//       V side:  O[dim][head] += (1 + c/64)^T * w as mma(A = codes read
//                transposed by ldmatrix.trans, B = w hi/lo); the constant part
//                is removed with corr = sum_t p*(b - 64*s) at the end:
//                out = 64*O + corr.
//   * the query rows are loaded by the consumer threads (plain 16-byte loads
//     into shared memory), so the producer's first TMA issues do not queue
//     behind them;
//   * the warp states are LSE-merged in shared memory; the CTA writes its
//     split partial and the last CTA of the KV head merges all splits with an
//     online LSE merge, 16 (G <= 2) or 8 splits' loads in flight per thread.
//   * launch: programmatic dependent launch; barrier init, tensor-map and L2
//     prefetches (queries, the CTA's first tiles) run before the dependency
//     wait; a fused quantize-on-append (tq_sdpa_int4_append) has consumer
//     warp 0 (and 1 at D=256) write the step's K/V row while the first tiles
//     stream in, and the producer issues the tile holding it only after that
//     write is fenced.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>
#include <string>
#include <type_traits>
#include <unordered_map>

#include "tq_common.cuh"
#include "tq_internal.h"
#include "peer_layout.cuh"

namespace tq {

namespace {

constexpr int kChunk = 64;  // tokens per TMA box; splits are whole chunks
constexpr int kMergeGroup = 32;  // splits per first-level group of a two-level merge
#ifndef TQ_DECODE_MINB_128
#define TQ_DECODE_MINB_128 3
#endif
#ifndef TQ_DECODE_STAGES_128
#define TQ_DECODE_STAGES_128 3
#endif
#ifndef TQ_DECODE_PREFETCH_TILES
#define TQ_DECODE_PREFETCH_TILES 2
#endif
// Tiles of its range a CTA warms L2 with before it waits for the preceding
// kernel (a hint: nothing is read into the kernel before the wait).
constexpr int kPrefetchTiles = TQ_DECODE_PREFETCH_TILES;

// Per head_dim: W consumer warps (+ one TMA producer warp), each taking TB
// independent 16-token blocks of every tile (two interleaved dependency
// chains at D=128); a stage of W*TB*16 tokens (18 KB at D=128 and at D=256);
// 3 CTAs per SM at D=128, 2 at D=256 (registers).
template <int D>
struct MCfg {
  static constexpr int W = 4;
  static constexpr int TB = D == 128 ? 2 : 1;  // 16-token blocks per warp per tile
  static constexpr int THREADS = (W + 1) * 32;
  static constexpr int TILE = 16 * W * TB;
  static constexpr int CPT = TILE / kChunk;  // chunks per tile
  static constexpr int MINB = D == 128 ? TQ_DECODE_MINB_128 : 2;  // CTAs per SM with f16
                                                 // queries; f32/bf16 queries (hi+lo split) run 1 per SM
  static constexpr int STAGES = D == 128 ? TQ_DECODE_STAGES_128 : 5;
};

template <int D, int G, typename SB>
struct MLayout {
  static constexpr int W = MCfg<D>::W;
  static constexpr int TILE = MCfg<D>::TILE;
  static constexpr int NG = D / 64;
  static constexpr int ROWB = D / 2;                     // code bytes per token
  static constexpr int CHUNK = kChunk * ROWB;            // code bytes of one TMA box
  static constexpr int CODE = TILE * ROWB;               // one code tile
  static constexpr int SBB = TILE * NG * static_cast<int>(sizeof(SB));
  static constexpr int STAGE = (2 * CODE + 4 * SBB + 1023) / 1024 * 1024;
  static constexpr int STAGES = MCfg<D>::STAGES * STAGE;
  // full[MCfg<D>::STAGES], empty[MCfg<D>::STAGES], q, appended token written
  static constexpr int BAR = STAGES;
  static constexpr int FLAG = BAR + ((2 * MCfg<D>::STAGES + 1) * 8 + 15) / 16 * 16;
  static constexpr int QB = FLAG + 16;                   // the CTA's G query rows (<= f32)
  static_assert(QB % 16 == 0, "the query rows are stored as 16-byte words");
  static constexpr int BYTES = QB + G * D * 4 + 1024;    // + alignment slack
  // end-of-range combine: per warp m, l, corr[NG], o[D] for G heads
  static constexpr int WST = G * (2 + NG + D);
  static_assert(W * WST * 4 <= STAGES, "warp states reuse the stages");
  // split merge: per thread (M, L) + a float4 of o
  static_assert(W * 32 * 24 <= STAGES, "merge states reuse the stages");
};

struct MParams {
  const void* q;
  int q_dtype;
  const uint32_t* kq;  // code bases (the TMA maps hold them too; used for L2 prefetch)
  const uint32_t* vq;
  const void* ks;
  const void* kb;
  const void* vs;
  const void* vb;
  const int32_t* seq_lens;
  int n_tokens;
  int B, H, Hkv, Gtot, nsub;
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
  int splits, chunks_per_split;
  // fused quantize-on-append (nullable): the step's K/V rows (B, Hkv, D) are
  // quantized into slot n_local - 1 of each sequence before it is read
  const void* k_new;
  const void* v_new;
  int new_dtype;
  int new_slot;  // < 0: n_local - 1 (the end of each sequence); else this slot (ring caches)
  const int32_t* new_slots;  // nullable: sequence b's slot in device memory (overrides new_slot)
  float* ws_o;
  float* ws_ml;
  unsigned* counters;
  uint32_t* err;
  // partial == 1 with peer_bufs: the state goes straight into slot
  // [step parity][peer_rank] of every rank's exchange buffer, then the
  // unit's flag is raised in each (peer_layout.cuh); part_out is unused
  void* const* peer_bufs;
  int peer_world, peer_rank;
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


template <int W>
__device__ __forceinline__ void consumers_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(W * 32) : "memory");
}

// Two nibbles (bits 4j and 16+4j of x) -> fp16x2 (1 + c/64): the nibble is
// moved to mantissa bits 4..7 of each half (nibble 1 is already there) and
// OR-ed into 1.0 (0x3C00). Three shifts and four LOP3 per 8 nibbles.
template <int J>
__device__ __forceinline__ uint32_t nib64(uint32_t x, uint32_t magic) {
  const uint32_t s = (J == 0) ? (x << 4) : (J == 1) ? x : (J == 2) ? (x >> 4) : (x >> 8);
  uint32_t d;  // (s & 0x00F000F0) | magic in one LOP3 (lut 0xEA = (a & b) | c)
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(s), "n"(0x00F000F0), "r"(magic));
  return d;
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

// The NG scales (or biases) of one token row as floats.
template <typename SB, int NG>
__device__ __forceinline__ void load_sb_row(const SB* p, float (&v)[NG]) {
  if constexpr (sizeof(SB) == 2 && NG == 2) {
    const float2 a = unpack_h2(*reinterpret_cast<const uint32_t*>(p));
    v[0] = a.x;
    v[1] = a.y;
  } else if constexpr (sizeof(SB) == 2 && NG == 4) {
    const uint2 raw = *reinterpret_cast<const uint2*>(p);
    const float2 a = unpack_h2(raw.x), b = unpack_h2(raw.y);
    v[0] = a.x;
    v[1] = a.y;
    v[2] = b.x;
    v[3] = b.y;
  } else if constexpr (sizeof(SB) == 4 && NG == 2) {
    const float2 a = *reinterpret_cast<const float2*>(p);
    v[0] = a.x;
    v[1] = a.y;
  } else if constexpr (sizeof(SB) == 4 && NG == 4) {
    const float4 a = *reinterpret_cast<const float4*>(p);
    v[0] = a.x;
    v[1] = a.y;
    v[2] = a.z;
    v[3] = a.w;
  } else {
#pragma unroll
    for (int g = 0; g < NG; ++g) v[g] = sb_to_float<SB>(p[g]);
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

// Token order of a warp's 16-token block: A-operand row r of the K-side mma
// and V-side contraction index k < 8 both stand for token sigma(r) (any
// permutation works for the math, both sides use the same one). It is chosen
// so the K-side 8-byte row reads are bank-conflict free: a half-warp (rows
// 4p..4p+3, 4 lanes each) reads 16-byte chunk (word chunk) ^ swizzle(row), so
// the four rows' swizzle values must differ in their chunk-pair bits --
//   D = 128 (SWIZZLE_64B, 64-byte rows, swizzle (row >> 1) & 3): bits 1 and 2
//   swapped; D = 256 (SWIZZLE_128B, 128-byte rows, swizzle row & 7): a 3-bit
//   rotation, so rows 0..3 map to 0,2,4,6 and rows 4..7 to 1,3,5,7.
// The ldmatrix reads (8 rows of one chunk) are conflict free for any
// permutation.
template <int D>
__device__ __forceinline__ int sigma8(int r) {
  if constexpr (D == 128) return (r & 1) | ((r & 2) << 1) | ((r & 4) >> 1);
  return ((r << 1) & 6) | (r >> 2);
}

template <int D, int G, typename SB, bool QSPLIT>
__global__ void __launch_bounds__(MCfg<D>::THREADS, QSPLIT ? 1 : MCfg<D>::MINB)
    decode_mma_kernel(const __grid_constant__ CUtensorMap tmk,
                      const __grid_constant__ CUtensorMap tmv, const MParams p) {
  using Lyt = MLayout<D, G, SB>;
  constexpr int W = MCfg<D>::W;
  constexpr int TILE = MCfg<D>::TILE;
  constexpr int TB = MCfg<D>::TB;
  constexpr int CPT = MCfg<D>::CPT;
  constexpr int NG = Lyt::NG;
  constexpr int NCH = D / 32;          // 16-byte code chunks per token
  constexpr bool kPaired = G <= 4;     // V side: hi/lo weights share one mma (N = 2G <= 8)
  // K side: mma(A = codes, rows = tokens; B = q, columns n = hb*P + phi). A
  // column (hb, phi) carries q_hb only on the k-rows of the lanes whose
  // thread-in-group c has c*P/4 == phi, so every accumulator column is a
  // partial dot product over a quarter (P=4), half (P=2) or all (P=1) of the
  // 64 dims of a group, and all 8 columns are used for any GQA factor.
  constexpr int P = G <= 2 ? 4 : 8 / G;
  constexpr int IPL = G <= 2 ? 1 : G / 2;  // complete (head, token) items per lane
  constexpr int IH = G == 8 ? 2 : 1;       // distinct item heads per lane
  constexpr int NTK = G <= 2 ? 1 : 2;      // distinct item tokens per lane
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Lyt::BAR);
  uint64_t* empty = full + MCfg<D>::STAGES;
  uint64_t* nbar = empty + MCfg<D>::STAGES;  // the appended token is in global memory (fused append)
  int* s_flag = reinterpret_cast<int*>(smem + Lyt::FLAG);

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int split = blockIdx.x;
  const int hg = blockIdx.y;
  const int b = blockIdx.z;
  const int kv = hg / p.nsub;
  const int h0 = kv * p.Gtot + (hg % p.nsub) * G;

  const long long tok_base =
      static_cast<long long>(b) * p.bstride_tok + static_cast<long long>(kv) * p.capacity;
  // visible token range [t_lo, t_hi) of a sequence of n_local tokens and this
  // CTA's chunks [cb, ce) of it (tiles of CPT chunks from cb, the last may be short)
  auto range = [&](int n_local, int& t_lo, int& cb, int& ce) {
    t_lo = 0;
    if (p.window > 0) {
      const int n_glob = p.n_total > 0 ? p.n_total : n_local + p.token_offset;
      t_lo = max(0, n_glob - p.window - p.token_offset);
    }
    cb = ce = 0;
    if (n_local > t_lo) {
      cb = t_lo / kChunk + split * p.chunks_per_split;
      ce = min((n_local + kChunk - 1) / kChunk, cb + p.chunks_per_split);
    }
  };

  // Before waiting for the preceding kernel: barrier init, tensor-map
  // prefetch, and L2 warmed with the query rows and the first tiles of the
  // range that n_tokens (the largest sequence) gives. A prefetch reads
  // nothing into this kernel, so data a preceding kernel still writes (the
  // queries, an appended token) is read coherently after pdl_wait.
  if (tid == 0) {
    for (int s = 0; s < MCfg<D>::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], W);
    }
    mbar_init(nbar, D / 128);  // one arrival per writer warp of a fused append
    fence_barrier_init();
  }
  if (warp == W) {
    if (lane == 0) {
      prefetch_tensormap(&tmk);
      prefetch_tensormap(&tmv);
      const int qel = p.q_dtype == kF32 ? 4 : 2;
      prefetch_l2(static_cast<const unsigned char*>(p.q) + (static_cast<long long>(b) * p.H + h0) * D * qel,
                  static_cast<uint32_t>(G * D * qel));
    }
    const int n_pf = max(0, min(p.n_tokens, p.capacity));
    const int n_pf4 = (n_pf + 3) & ~3;  // <= capacity: rows past it are never touched
    int lo, c0, c1;
    range(n_pf, lo, c0, c1);
    // the producer warp's lanes prefetch kPrefetchTiles tiles each (one tile
    // per lane); kPrefetchTiles < 0: the CTA's whole range
    const int pf_end = kPrefetchTiles < 0 ? c1 : min(c1, c0 + kPrefetchTiles * CPT);
    for (int c = c0 + lane * CPT; c < pf_end; c += 32 * CPT) {
      const int rows = min(min(CPT, c1 - c) * kChunk, n_pf4 - c * kChunk);
      const long long t0 = tok_base + static_cast<long long>(c) * kChunk;
      const uint32_t cbytes = static_cast<uint32_t>(rows * (D / 2));
      const uint32_t sbytes = static_cast<uint32_t>(rows * NG * sizeof(SB));
      prefetch_l2(p.kq + t0 * (D / 8), cbytes);
      prefetch_l2(p.vq + t0 * (D / 8), cbytes);
      prefetch_l2(reinterpret_cast<const SB*>(p.ks) + t0 * NG, sbytes);
      prefetch_l2(reinterpret_cast<const SB*>(p.kb) + t0 * NG, sbytes);
      prefetch_l2(reinterpret_cast<const SB*>(p.vs) + t0 * NG, sbytes);
      prefetch_l2(reinterpret_cast<const SB*>(p.vb) + t0 * NG, sbytes);
    }
  }

  __syncthreads();
  pdl_wait();     // inputs of the preceding kernels are visible from here on
  pdl_trigger();  // every CTA of this grid has started: the next may launch

  const int n_local = max(0, min(p.seq_lens ? p.seq_lens[b] : p.n_tokens, p.capacity));
  const int t_hi = n_local;
  int t_lo, cb, ce;
  range(n_local, t_lo, cb, ce);
  const int ntiles = ce > cb ? (ce - cb + CPT - 1) / CPT : 0;
  const int r_hi = min(t_hi, ce * kChunk);  // tokens at or past r_hi are masked
  // fused append: the CTA whose chunks hold slot n_local - 1 quantizes the
  // step's K/V row into it (CTAs of other query-head subsets of the same KV
  // head write the same bytes); its producer issues the tile holding the
  // slot only after the writers' release on nbar
  constexpr int NWW = D / 128;  // writer warps: D/8 words of K and of V, one per lane
  const int new_slot = p.new_slots ? p.new_slots[b] : p.new_slot >= 0 ? p.new_slot : n_local - 1;
  const bool has_new = p.k_new != nullptr && n_local > 0 && new_slot < n_local &&
                       new_slot >= cb * kChunk && new_slot < ce * kChunk;
  const int new_tile = has_new ? (new_slot / kChunk - cb) / CPT : -1;


  // ======================= producer warp ========================================
  if (warp == W) {
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      const int t_hi4 = (t_hi + 3) & ~3;
      const SB* ksb = reinterpret_cast<const SB*>(p.ks) + tok_base * NG;
      const SB* kbb = reinterpret_cast<const SB*>(p.kb) + tok_base * NG;
      const SB* vsb = reinterpret_cast<const SB*>(p.vs) + tok_base * NG;
      const SB* vbb = reinterpret_cast<const SB*>(p.vb) + tok_base * NG;
      int st = 0;
      uint32_t par = 0;
      for (int i = 0; i < ntiles; ++i) {
        if (i >= MCfg<D>::STAGES) mbar_wait_bounded(&empty[st], par ^ 1u, p.err);
        if (i == new_tile) {  // the appended token's codes and scales are written
          mbar_wait_bounded(nbar, 0, p.err);
          fence_proxy_async_global();
        }
        const int c0 = cb + i * CPT;
        const int nc = min(CPT, ce - c0);
        const int t0 = c0 * kChunk;
        const int nt = min(nc * kChunk, t_hi4 - t0);  // scale rows: a positive multiple of 4
        const uint32_t sbb = static_cast<uint32_t>(nt * NG * sizeof(SB));
        unsigned char* sb = smem + st * Lyt::STAGE;
        mbar_arrive_expect_tx(&full[st], 2 * nc * Lyt::CHUNK + 4 * sbb);
        const int row = static_cast<int>(tok_base + t0);
        for (int j = 0; j < nc; ++j) {
          tma_load_2d(sb + j * Lyt::CHUNK, &tmk, 0, row + j * kChunk, &full[st], pol);
          tma_load_2d(sb + Lyt::CODE + j * Lyt::CHUNK, &tmv, 0, row + j * kChunk, &full[st], pol);
        }
        unsigned char* sbp = sb + 2 * Lyt::CODE;
        bulk_g2s(sbp, ksb + static_cast<long long>(t0) * NG, sbb, &full[st], pol);
        bulk_g2s(sbp + Lyt::SBB, kbb + static_cast<long long>(t0) * NG, sbb, &full[st], pol);
        bulk_g2s(sbp + 2 * Lyt::SBB, vsb + static_cast<long long>(t0) * NG, sbb, &full[st], pol);
        bulk_g2s(sbp + 3 * Lyt::SBB, vbb + static_cast<long long>(t0) * NG, sbb, &full[st], pol);
        if (++st == MCfg<D>::STAGES) {
          st = 0;
          par ^= 1u;
        }
      }
    }
    return;
  }

  // ======================= consumer warps =======================================
  // the CTA's query rows (0.5-8 KB) into shared memory by the consumer
  // threads' own loads: the producer's first TMA issues are not queued
  // behind a copy of them
  {
    const int qel = p.q_dtype == kF32 ? 4 : 2;
    const int qwords = G * D * qel / 16;
    const uint4* qsrc = reinterpret_cast<const uint4*>(
        static_cast<const unsigned char*>(p.q) + (static_cast<long long>(b) * p.H + h0) * D * qel);
    uint4* qdst = reinterpret_cast<uint4*>(smem + Lyt::QB);
    for (int i = tid; i < qwords; i += W * 32) qdst[i] = qsrc[i];
  }
  // fused append: lane = one packed word of the K row (first D/8 writer
  // threads) or of the V row, quantized exactly as quantize_rows_kernel does
  if (has_new && warp < NWW) {
    constexpr int WPR = D / 8;
    const int wi = warp * 32 + lane;
    const bool is_v = wi >= WPR;
    const int w = wi % WPR;
    float v[8];
    load8_aligned(is_v ? p.v_new : p.k_new,
                  (static_cast<long long>(b) * p.Hkv + kv) * D + w * 8, p.new_dtype, v);
    float mn, mx;
    group_minmax8(v, mn, mx);
    const long long tok = tok_base + new_slot;
    void* sc = const_cast<void*>(is_v ? p.vs : p.ks);
    void* bi = const_cast<void*>(is_v ? p.vb : p.kb);
    constexpr int kSb = sizeof(SB) == 4 ? kF32 : kF16;
    const uint32_t packed = quantize_word8(v, mn, mx, kSb, sc, bi, tok * NG + w / 8, (w % 8) == 0);
    const_cast<uint32_t*>(is_v ? p.vq : p.kq)[tok * WPR + w] = packed;
    fence_proxy_async_global();
    __syncwarp();
    if (lane == 0) mbar_arrive(nbar);
  }
  const int r = lane >> 2;  // mma groupID
  const int c = lane & 3;   // mma thread-in-group

  // ---- q as the K-side B operand (column n = r) -----------------------------
  // k-step ks of group g covers word w = 8g + 2c + ks/2 of the token rows:
  // b0 = k-rows 2c, 2c+1 -> dims 8w+jb, 8w+jb+4; b1 = k-rows 2c+8, 2c+9 ->
  // dims 8w+jb+1, 8w+jb+5 (jb = 2*(ks%2)) -- the dims nib64<jb>/<jb+1> give
  // the A operand.
  uint32_t qb[NG][4][2];
  uint32_t qb_lo[QSPLIT ? NG : 1][4][2];
  float qs_col[NG];  // sum of q_hb over each group (identical in the 4 lanes of row r)
  consumers_sync<W>();  // the query rows are in shared memory
  {
    const int hb = r / P;
    const int phib = r % P;
    const bool on = hb < G && phib == (c * P) / 4;
    const void* sq = smem + Lyt::QB;
    const int qrow = (hb < G ? hb : 0) * D;
#pragma unroll
    for (int g = 0; g < NG; ++g) {
      float part = 0.0f;
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        const int w = 8 * g + 2 * c + (ks >> 1);
        const int jb = 2 * (ks & 1);
        const int dd[4] = {8 * w + jb, 8 * w + jb + 4, 8 * w + jb + 1, 8 * w + jb + 5};
        float v[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) v[e] = load_as_float(sq, qrow + dd[e], p.q_dtype);
        part += (v[0] + v[1]) + (v[2] + v[3]);
        const uint32_t h01 = pack_h2(v[0], v[1]), h23 = pack_h2(v[2], v[3]);
        qb[g][ks][0] = on ? h01 : 0u;
        qb[g][ks][1] = on ? h23 : 0u;
        if constexpr (QSPLIT) {
          const float2 f01 = unpack_h2(h01), f23 = unpack_h2(h23);
          qb_lo[g][ks][0] = on ? pack_h2(v[0] - f01.x, v[1] - f01.y) : 0u;
          qb_lo[g][ks][1] = on ? pack_h2(v[2] - f23.x, v[3] - f23.y) : 0u;
        }
      }
      part += __shfl_xor_sync(0xffffffffu, part, 1);
      part += __shfl_xor_sync(0xffffffffu, part, 2);
      qs_col[g] = part;
    }
  }

  // ---- this lane's items: complete (head, token) scores after the reduce ----
  // G <= 2: head c/2, token sigma(r) + 8*(c&1); G = 4: head c, tokens
  // sigma(r) + 8f; G = 8: heads 2c + e, tokens sigma(r) + 8f (item 2f + e).
  int ihead[IH];
#pragma unroll
  for (int e = 0; e < IH; ++e) ihead[e] = G <= 2 ? (c >> 1) : (G == 4 ? c : 2 * c + e);
  const bool hvalid = ihead[0] < G;  // false only for G = 1, c >= 2
  float qsum[IH][NG];                // sum of q over each group for the item heads
#pragma unroll
  for (int e = 0; e < IH; ++e)
#pragma unroll
    for (int g = 0; g < NG; ++g)
      qsum[e][g] = __shfl_sync(0xffffffffu, qs_col[g], 4 * ((hvalid ? ihead[e] : 0) * P));

  // this warp's blocks of 16 tokens start at tile rows wt0 + 16*bt; the
  // swizzle pattern repeats every 8 rows, so block bt's offsets are block 0's
  // plus 16*bt rows
  const int wt0 = warp * 16 * TB;
  constexpr int BROW = 16 * Lyt::ROWB;  // bytes of 16 code rows
  const int sr = sigma8<D>(r);
  int trow[NTK];              // tile rows of the item tokens (block 0)
#pragma unroll
  for (int f = 0; f < NTK; ++f) trow[f] = wt0 + sr + 8 * (G <= 2 ? (c & 1) : f);
  int koff[2][NG];            // K-side A operand: rows sigma(r), sigma(r)+8; words 8g+2c, +1
#pragma unroll
  for (int f = 0; f < 2; ++f)
#pragma unroll
    for (int g = 0; g < NG; ++g) {
      const int word = 8 * g + 2 * c;
      koff[f][g] = swz<D>(wt0 + sr + 8 * f, word >> 2) + 4 * (word & 3);
    }
  int voff[NCH / 2];          // ldmatrix row address of this lane (token sigma(row))
  {
    const int mi = lane >> 3, mrow = lane & 7;
#pragma unroll
    for (int q2 = 0; q2 < NCH / 2; ++q2)
      voff[q2] = swz<D>(wt0 + 8 * (mi & 1) + sigma8<D>(mrow), 2 * q2 + (mi >> 1));
  }

  // O[dim][col] accumulators: chunk kk (32 dims), sub-tile s2; rows r / r+8 =
  // dims 32kk + 4r + 2s2 (+1); cols 2c, 2c+1 = (head c: hi, lo) when paired,
  // heads 2c, 2c+1 otherwise.
  float o[NCH][2][4];
#pragma unroll
  for (int kk = 0; kk < NCH; ++kk)
#pragma unroll
    for (int s2 = 0; s2 < 2; ++s2)
#pragma unroll
      for (int e = 0; e < 4; ++e) o[kk][s2][e] = 0.0f;
  float m_run[IH], l_run[IH], corr[IH][NG];
#pragma unroll
  for (int e = 0; e < IH; ++e) {
    m_run[e] = -INFINITY;
    l_run[e] = 0.0f;
#pragma unroll
    for (int g = 0; g < NG; ++g) corr[e][g] = 0.0f;
  }

  const uint32_t smem_base = smem_addr(smem);
  uint32_t mg = 0x3C003C00u;  // fp16x2 1.0, kept in a register for the LOP3s
  asm volatile("" : "+r"(mg));

  auto tile = [&](auto masked_c, int st, int tile_t0) {
    constexpr bool MASKED = decltype(masked_c)::value;
    const unsigned char* stg = smem + st * Lyt::STAGE;
    const SB* s_ks = reinterpret_cast<const SB*>(stg + 2 * Lyt::CODE);
    const SB* s_kb = s_ks + TILE * NG;
    const SB* s_vs = s_kb + TILE * NG;
    const SB* s_vb = s_vs + TILE * NG;

    // ---- K side: partial S[token][column] per block and group ------------------
    float acc[TB][NG][4];
#pragma unroll
    for (int bt = 0; bt < TB; ++bt)
#pragma unroll
      for (int g = 0; g < NG; ++g) {
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[bt][g][e] = 0.0f;
        const uint2 w0 = *reinterpret_cast<const uint2*>(stg + bt * BROW + koff[0][g]);  // sigma(r)
        const uint2 w1 = *reinterpret_cast<const uint2*>(stg + bt * BROW + koff[1][g]);  // sigma(r)+8
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
          const uint32_t x0 = (ks >> 1) ? w0.y : w0.x;
          const uint32_t x1 = (ks >> 1) ? w1.y : w1.x;
          uint32_t a0, a1, a2, a3;
          if (ks & 1) {
            a0 = nib64<2>(x0, mg); a1 = nib64<2>(x1, mg); a2 = nib64<3>(x0, mg); a3 = nib64<3>(x1, mg);
          } else {
            a0 = nib64<0>(x0, mg); a1 = nib64<0>(x1, mg); a2 = nib64<1>(x0, mg); a3 = nib64<1>(x1, mg);
          }
          mma16816(acc[bt][g], a0, a1, a2, a3, qb[g][ks][0], qb[g][ks][1]);
          if constexpr (QSPLIT) mma16816(acc[bt][g], a0, a1, a2, a3, qb_lo[g][ks][0], qb_lo[g][ks][1]);
        }
      }

    // ---- complete S per item (sum over the dim subsets phi) ------------------
    float S[TB][IPL][NG];
#pragma unroll
    for (int bt = 0; bt < TB; ++bt)
#pragma unroll
      for (int g = 0; g < NG; ++g) {
        if constexpr (G <= 2) {
          // cols 2c, 2c+1 = phis {0,1} (c even) or {2,3} (c odd) of head c/2;
          // lane c even keeps token sigma(r), c odd keeps sigma(r)+8.
          const float x0 = acc[bt][g][0] + acc[bt][g][1];
          const float x1 = acc[bt][g][2] + acc[bt][g][3];
          const bool odd = (c & 1) != 0;
          const float keep = odd ? x1 : x0;
          const float send = odd ? x0 : x1;
          S[bt][0][g] = keep + __shfl_xor_sync(0xffffffffu, send, 1);
        } else if constexpr (G == 4) {
          S[bt][0][g] = acc[bt][g][0] + acc[bt][g][1];
          S[bt][1][g] = acc[bt][g][2] + acc[bt][g][3];
        } else {
#pragma unroll
          for (int it = 0; it < 4; ++it) S[bt][it][g] = acc[bt][g][it];  // it = 2f + e
        }
      }

    // ---- scores (log2 units) ---------------------------------------------------
    // score = sum_g s_g * sum_d q_d c_d + b_g * sum_d q_d, sum q c = 64 (S - sum q)
    float sk[TB][NTK][NG], bk[TB][NTK][NG];
#pragma unroll
    for (int bt = 0; bt < TB; ++bt)
#pragma unroll
      for (int f = 0; f < NTK; ++f) {
        load_sb_row<SB, NG>(s_ks + (trow[f] + 16 * bt) * NG, sk[bt][f]);
        load_sb_row<SB, NG>(s_kb + (trow[f] + 16 * bt) * NG, bk[bt][f]);
      }
    float sc[TB][IPL];
    float bmax[IH];
#pragma unroll
    for (int e = 0; e < IH; ++e) bmax[e] = -INFINITY;
#pragma unroll
    for (int bt = 0; bt < TB; ++bt)
#pragma unroll
      for (int it = 0; it < IPL; ++it) {
        const int f = G <= 2 ? 0 : (G == 4 ? it : it >> 1);
        const int e = G == 8 ? (it & 1) : 0;
        float a = 0.0f, bsum = 0.0f;
#pragma unroll
        for (int g = 0; g < NG; ++g) {
          a = fmaf(sk[bt][f][g], S[bt][it][g] - qsum[e][g], a);
          bsum = fmaf(bk[bt][f][g], qsum[e][g], bsum);
        }
        float v = fmaf(64.0f, a, bsum) * p.qscale;
        if constexpr (MASKED) {
          const int tg = tile_t0 + trow[f] + 16 * bt;
          v = (hvalid && tg >= t_lo && tg < r_hi) ? v : -INFINITY;
        }
        sc[bt][it] = v;
        bmax[e] = fmaxf(bmax[e], v);
      }
    // max over the lanes of each item head
#pragma unroll
    for (int e = 0; e < IH; ++e) {
      if constexpr (G <= 2) bmax[e] = fmaxf(bmax[e], __shfl_xor_sync(0xffffffffu, bmax[e], 1));
      bmax[e] = fmaxf(bmax[e], __shfl_xor_sync(0xffffffffu, bmax[e], 4));
      bmax[e] = fmaxf(bmax[e], __shfl_xor_sync(0xffffffffu, bmax[e], 8));
      bmax[e] = fmaxf(bmax[e], __shfl_xor_sync(0xffffffffu, bmax[e], 16));
    }

    // ---- online softmax -------------------------------------------------------
    float alpha[IH];
#pragma unroll
    for (int e = 0; e < IH; ++e) {
      const float m_new = fmaxf(m_run[e], bmax[e]);
      alpha[e] = (m_new == -INFINITY) ? 1.0f : fast_exp2(m_run[e] - m_new);
      m_run[e] = m_new;
      l_run[e] *= alpha[e];
#pragma unroll
      for (int g = 0; g < NG; ++g) corr[e][g] *= alpha[e];
    }
    float pr[TB][IPL];
#pragma unroll
    for (int bt = 0; bt < TB; ++bt)
#pragma unroll
      for (int it = 0; it < IPL; ++it) {
        const int e = G == 8 ? (it & 1) : 0;
        pr[bt][it] = MASKED ? ((sc[bt][it] == -INFINITY) ? 0.0f : fast_exp2(sc[bt][it] - m_run[e]))
                            : fast_exp2(sc[bt][it] - m_run[e]);
        l_run[e] += pr[bt][it];
      }

    // ---- weights w = p*s (fp16 hi + lo) and the constant correction ------------
    float sv[TB][NTK][NG], bv[TB][NTK][NG];
#pragma unroll
    for (int bt = 0; bt < TB; ++bt)
#pragma unroll
      for (int f = 0; f < NTK; ++f) {
        load_sb_row<SB, NG>(s_vs + (trow[f] + 16 * bt) * NG, sv[bt][f]);
        load_sb_row<SB, NG>(s_vb + (trow[f] + 16 * bt) * NG, bv[bt][f]);
      }
    uint32_t hl[TB][IPL][NG];  // packed (hi | lo << 16) of w per item and group
#pragma unroll
    for (int bt = 0; bt < TB; ++bt)
#pragma unroll
      for (int it = 0; it < IPL; ++it) {
        const int f = G <= 2 ? 0 : (G == 4 ? it : it >> 1);
        const int e = G == 8 ? (it & 1) : 0;
        float w[NG];
#pragma unroll
        for (int g = 0; g < NG; ++g) {
          w[g] = pr[bt][it] * sv[bt][f][g];
          float cb = pr[bt][it] * fmaf(-64.0f, sv[bt][f][g], bv[bt][f][g]);
          if constexpr (MASKED) {  // stale scales of masked tokens must not leak
            w[g] = pr[bt][it] == 0.0f ? 0.0f : w[g];
            cb = pr[bt][it] == 0.0f ? 0.0f : cb;
          }
          corr[e][g] += cb;
        }
        // hi = fp16(w), lo = fp16(w - hi), two groups per conversion
#pragma unroll
        for (int g = 0; g < NG; g += 2) {
          const uint32_t hi2 = pack_h2(w[g], w[g + 1]);
          const float2 hf = unpack_h2(hi2);
          const uint32_t lo2 = pack_h2(w[g] - hf.x, w[g + 1] - hf.y);
          hl[bt][it][g] = __byte_perm(hi2, lo2, 0x5410u);
          hl[bt][it][g + 1] = __byte_perm(hi2, lo2, 0x7632u);
        }
      }

    // ---- V-side B operand: rows k = 2c, 2c+1 (b0), 2c+8, 2c+9 (b1) stand for
    // tokens sigma(k&7) + 8(k>>3), whose items live in lanes with r' = k & 7.
    uint32_t bw[TB][NG][2];
    uint32_t bw_lo[TB][kPaired ? 1 : NG][2];
    (void)bw_lo;
#pragma unroll
    for (int bt = 0; bt < TB; ++bt) {
      if constexpr (G <= 2) {
        // column r = (head r/2, hi or lo); columns of heads >= G carry other
        // heads' weights into O columns that are never read (each mma output
        // column depends on its B column only)
        const int hp = r >> 1;
        const uint32_t sel = (r & 1) ? 0x7632u : 0x5410u;
        const int l0 = 8 * c + 2 * hp;
#pragma unroll
        for (int g = 0; g < NG; ++g) {
          const uint32_t x0 = __shfl_sync(0xffffffffu, hl[bt][0][g], l0);
          const uint32_t x1 = __shfl_sync(0xffffffffu, hl[bt][0][g], l0 + 4);
          const uint32_t x2 = __shfl_sync(0xffffffffu, hl[bt][0][g], l0 + 1);
          const uint32_t x3 = __shfl_sync(0xffffffffu, hl[bt][0][g], l0 + 5);
          bw[bt][g][0] = __byte_perm(x0, x1, sel);
          bw[bt][g][1] = __byte_perm(x2, x3, sel);
        }
      } else if constexpr (G == 4) {
        const int hp = r >> 1;
        const uint32_t sel = (r & 1) ? 0x7632u : 0x5410u;
        const int l0 = 8 * c + hp;
#pragma unroll
        for (int g = 0; g < NG; ++g) {
          const uint32_t x0 = __shfl_sync(0xffffffffu, hl[bt][0][g], l0);
          const uint32_t x1 = __shfl_sync(0xffffffffu, hl[bt][0][g], l0 + 4);
          const uint32_t x2 = __shfl_sync(0xffffffffu, hl[bt][1][g], l0);
          const uint32_t x3 = __shfl_sync(0xffffffffu, hl[bt][1][g], l0 + 4);
          bw[bt][g][0] = __byte_perm(x0, x1, sel);
          bw[bt][g][1] = __byte_perm(x2, x3, sel);
        }
      } else {
        // column r = head r: item (head r, token k) is register 2(k>>3) + (r&1)
        // of lane 4(k&7) + r/2
        const int l0 = 8 * c + (r >> 1);
        const bool odd = (r & 1) != 0;
#pragma unroll
        for (int g = 0; g < NG; ++g) {
          uint32_t y[4];
#pragma unroll
          for (int f = 0; f < 2; ++f) {
            const uint32_t u0 = __shfl_sync(0xffffffffu, hl[bt][2 * f][g], l0);
            const uint32_t u1 = __shfl_sync(0xffffffffu, hl[bt][2 * f + 1][g], l0);
            const uint32_t v0 = __shfl_sync(0xffffffffu, hl[bt][2 * f][g], l0 + 4);
            const uint32_t v1 = __shfl_sync(0xffffffffu, hl[bt][2 * f + 1][g], l0 + 4);
            y[2 * f] = odd ? u1 : u0;
            y[2 * f + 1] = odd ? v1 : v0;
          }
          bw[bt][g][0] = __byte_perm(y[0], y[1], 0x5410u);
          bw[bt][g][1] = __byte_perm(y[2], y[3], 0x5410u);
          bw_lo[bt][g][0] = __byte_perm(y[0], y[1], 0x7632u);
          bw_lo[bt][g][1] = __byte_perm(y[2], y[3], 0x7632u);
        }
      }
    }

    // rescale O when any head's max moved (warp-uniform decision)
    bool moved = false;
#pragma unroll
    for (int e = 0; e < IH; ++e) moved |= alpha[e] != 1.0f;
    if (__any_sync(0xffffffffu, moved)) {
      float a0, a1;
      if constexpr (G <= 2) {
        a0 = a1 = __shfl_sync(0xffffffffu, alpha[0], 2 * c);
      } else if constexpr (G == 4) {
        a0 = a1 = __shfl_sync(0xffffffffu, alpha[0], c);
      } else {
        a0 = __shfl_sync(0xffffffffu, alpha[0], c);
        a1 = __shfl_sync(0xffffffffu, alpha[IH - 1], c);
      }
#pragma unroll
      for (int kk = 0; kk < NCH; ++kk)
#pragma unroll
        for (int s2 = 0; s2 < 2; ++s2) {
          o[kk][s2][0] *= a0;
          o[kk][s2][1] *= a1;
          o[kk][s2][2] *= a0;
          o[kk][s2][3] *= a1;
        }
    }

    // ---- V side: O += V^T * w ---------------------------------------------------
    const uint32_t vbase = smem_base + st * Lyt::STAGE + Lyt::CODE;
#pragma unroll
    for (int bt = 0; bt < TB; ++bt)
#pragma unroll
      for (int q2 = 0; q2 < NCH / 2; ++q2) {
        uint32_t d[4];
        ldsm_x4_trans(vbase + bt * BROW + voff[q2], d);
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int kk = 2 * q2 + hh;
          const int g = kk >> 1;
          const uint32_t R0 = d[2 * hh], R1 = d[2 * hh + 1];
          const uint32_t a00 = nib64<0>(R0, mg), a01 = nib64<1>(R0, mg), a02 = nib64<2>(R0, mg), a03 = nib64<3>(R0, mg);
          const uint32_t a10 = nib64<0>(R1, mg), a11 = nib64<1>(R1, mg), a12 = nib64<2>(R1, mg), a13 = nib64<3>(R1, mg);
          mma16816(o[kk][0], a00, a01, a10, a11, bw[bt][g][0], bw[bt][g][1]);
          mma16816(o[kk][1], a02, a03, a12, a13, bw[bt][g][0], bw[bt][g][1]);
          if constexpr (!kPaired) {
            mma16816(o[kk][0], a00, a01, a10, a11, bw_lo[bt][g][0], bw_lo[bt][g][1]);
            mma16816(o[kk][1], a02, a03, a12, a13, bw_lo[bt][g][0], bw_lo[bt][g][1]);
          }
        }
      }
  };

  {
    int st = 0;
    uint32_t par = 0;
    for (int i = 0; i < ntiles; ++i) {
      mbar_wait_bounded(&full[st], par, p.err);
      const int tile_t0 = (cb + i * CPT) * kChunk;
      if (tile_t0 >= t_lo && tile_t0 + TILE <= r_hi) {
        tile(std::integral_constant<bool, false>{}, st, tile_t0);
      } else {
        tile(std::integral_constant<bool, true>{}, st, tile_t0);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
      if (++st == MCfg<D>::STAGES) {
        st = 0;
        par ^= 1u;
      }
    }
  }

  // ---- combine the 4 consumer warps -------------------------------------------
  // l and corr: sum over the lanes of each item head
#pragma unroll
  for (int e = 0; e < IH; ++e) {
    if constexpr (G <= 2) l_run[e] += __shfl_xor_sync(0xffffffffu, l_run[e], 1);
    l_run[e] += __shfl_xor_sync(0xffffffffu, l_run[e], 4);
    l_run[e] += __shfl_xor_sync(0xffffffffu, l_run[e], 8);
    l_run[e] += __shfl_xor_sync(0xffffffffu, l_run[e], 16);
#pragma unroll
    for (int g = 0; g < NG; ++g) {
      if constexpr (G <= 2) corr[e][g] += __shfl_xor_sync(0xffffffffu, corr[e][g], 1);
      corr[e][g] += __shfl_xor_sync(0xffffffffu, corr[e][g], 4);
      corr[e][g] += __shfl_xor_sync(0xffffffffu, corr[e][g], 8);
      corr[e][g] += __shfl_xor_sync(0xffffffffu, corr[e][g], 16);
    }
  }
  consumers_sync<W>();  // every warp is past its last tile: the stage area is free
  float* wst = reinterpret_cast<float*>(smem) + warp * Lyt::WST;  // [G][2 + NG + D]
  if (r == 0 && (G > 2 || (c & 1) == 0) && hvalid) {
#pragma unroll
    for (int e = 0; e < IH; ++e) {
      float* hs = wst + ihead[e] * (2 + NG + D);
      hs[0] = m_run[e];
      hs[1] = l_run[e];
#pragma unroll
      for (int g = 0; g < NG; ++g) hs[2 + g] = corr[e][g];
    }
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
  consumers_sync<W>();

  const bool direct = p.splits == 1;
  const long long unit = static_cast<long long>(b) * gridDim.y + hg;
  // a value of this sequence's partial state: to part_out, or (published) as a
  // {value, step} pair into slot [step parity][peer_rank] of every rank's
  // exchange buffer (peer_layout.cuh), which needs no fence or flag: the
  // reader takes a value once its pair carries the step
  const long long sblk = static_cast<long long>(b) * p.H * (D + 2);
  uint32_t pstep = 0;
  long long pub_off = 0;  // this sequence's block in the slot, in pairs from the data start
  if (p.peer_bufs) {
    pstep = *reinterpret_cast<volatile const uint32_t*>(p.peer_bufs[p.peer_rank]) + 1u;
    pub_off = (static_cast<long long>(pstep & 1u) * p.peer_world + p.peer_rank) *
                  p.B * p.H * (D + 2) + sblk;
  }
  auto pub_ptr = [&](int k, long long off) {
    return reinterpret_cast<uint2*>(static_cast<uint32_t*>(p.peer_bufs[k]) + peer_data_word()) +
           pub_off + off;
  };
  auto put_state = [&](long long off, float v) {
    if (!p.peer_bufs) {
      p.part_out[sblk + off] = v;
      return;
    }
    for (int k = 0; k < p.peer_world; ++k) st_pair(pub_ptr(k, off), v, pstep);
  };
  // two adjacent values, off even (one 16-byte store per rank when published)
  auto put_state2 = [&](long long off, float v0, float v1) {
    if (!p.peer_bufs) {
      p.part_out[sblk + off] = v0;
      p.part_out[sblk + off + 1] = v1;
      return;
    }
    for (int k = 0; k < p.peer_world; ++k) st_pair2(pub_ptr(k, off), v0, v1, pstep);
  };
  const float* wall = reinterpret_cast<const float*>(smem);
  constexpr int NTH = W * 32;
  for (int it = tid; it < G * D; it += NTH) {
    const int g = it / D;
    const int d = it % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < W; ++w) M = fmaxf(M, wall[w * Lyt::WST + g * (2 + NG + D)]);
    float L = 0.0f, acc = 0.0f;
#pragma unroll
    for (int w = 0; w < W; ++w) {
      const float* hs = wall + w * Lyt::WST + g * (2 + NG + D);
      const float e = (M == -INFINITY || hs[0] == -INFINITY) ? 0.0f : fast_exp2(hs[0] - M);
      L += e * hs[1];
      acc += e * (64.0f * hs[2 + NG + d] + hs[2 + d / 64]);
    }
    const int h = h0 + g;
    if (direct) {
      if (p.partial) {
        put_state(static_cast<long long>(h) * D + d, acc);
        if (d == 0)
          put_state2(static_cast<long long>(p.H) * D + 2 * h, L == 0.0f ? -INFINITY : M * kLn2, L);
      } else {
        store_from_float(p.out, (static_cast<long long>(b) * p.H + h) * D + d, p.out_dtype,
                         L == 0.0f ? 0.0f : acc / L);
      }
    } else {
      const long long base = (unit * p.splits + split) * G;
      p.ws_o[(base + g) * D + d] = acc;
      if (d == 0) {
        p.ws_ml[(base + g) * 2] = L == 0.0f ? -INFINITY : M;
        p.ws_ml[(base + g) * 2 + 1] = L;
      }
    }
  }
  if (direct) return;

  // ---- last CTA of this (b, head group) merges the splits -------------------
  // Release: the CTA barrier orders every thread's partial stores before
  // thread 0's acquire-release ticket; the CTA that draws the last ticket has
  // acquired every other CTA's partials, and its barrier passes that on.
  // Up to 2 * kMergeGroup splits one CTA merges them all. Beyond that (few
  // (sequence, KV head) units over a long context, so one wave holds
  // hundreds of splits per unit) the merge has two levels: the last CTA of
  // each group of kMergeGroup consecutive splits merges its group into the
  // group's first slot, then the last of those merges the groups -- a
  // single CTA streaming hundreds of partials from L2 took longer than the
  // attention itself.
  const int S_ = p.splits;
  const long long base = unit * S_ * G;
  auto ticket = [&](unsigned* counter, int expected) {
    consumers_sync<W>();
    if (tid == 0) {
      const unsigned prev = atomic_add_acq_rel(counter, 1u);
      s_flag[0] = (prev == static_cast<unsigned>(expected - 1)) ? 1 : 0;
    }
    consumers_sync<W>();
    return s_flag[0] != 0;
  };

  // float4 items (head, 4 dims); the slots first, first + stride, ... (count
  // of them) of an item are spread over R thread subsets, each running an
  // online log-sum-exp merge with kML slots' (m, l, o) loads in flight per
  // step (16 at G <= 2: one round of L2 loads for up to 32 slots; 8 above,
  // where 16 would spill), then the R states are combined: into the outputs
  // (to_out) or, as a partial state, into slot `first`.
  constexpr int NI = G * D / 4;
  constexpr int R = NI >= NTH ? 1 : NTH / NI;
  constexpr int kML = G <= 2 ? 16 : 8;
  float2* mst = reinterpret_cast<float2*>(smem);           // [R][NI] (M, L)
  float4* ost = reinterpret_cast<float4*>(smem + R * NI * 8);  // [R][NI] o
  auto merge = [&](int first, int count, int stride, bool to_out) {
    for (int it = tid; it < NI * R; it += NTH) {
      const int item = it % NI, sub = it / NI;
      const int g = item / (D / 4);
      const float* ow = p.ws_o + (base + g) * D + 4 * (item % (D / 4));
      const float* mw = p.ws_ml + (base + g) * 2;
      float M = -INFINITY, L = 0.0f;
      float4 a = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      for (int j0 = sub; j0 < count; j0 += kML * R) {
        float2 ml[kML];
        float4 v[kML];
#pragma unroll
        for (int j = 0; j < kML; ++j) {
          const int jj = j0 + j * R;
          const long long sl = first + static_cast<long long>(jj) * stride;
          if (jj < count) {
            ml[j] = __ldcg(reinterpret_cast<const float2*>(mw + sl * G * 2));
            v[j] = __ldcg(reinterpret_cast<const float4*>(ow + sl * G * D));
          } else {
            ml[j] = make_float2(-INFINITY, 0.0f);
            v[j] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
          }
        }
        float mb = M;
#pragma unroll
        for (int j = 0; j < kML; ++j) mb = fmaxf(mb, ml[j].x);
        const float sc = M == -INFINITY ? 0.0f : fast_exp2(M - mb);
        L *= sc;
        a.x *= sc;
        a.y *= sc;
        a.z *= sc;
        a.w *= sc;
#pragma unroll
        for (int j = 0; j < kML; ++j) {
          const float e = ml[j].x == -INFINITY ? 0.0f : fast_exp2(ml[j].x - mb);
          L = fmaf(e, ml[j].y, L);
          a.x = fmaf(e, v[j].x, a.x);
          a.y = fmaf(e, v[j].y, a.y);
          a.z = fmaf(e, v[j].z, a.z);
          a.w = fmaf(e, v[j].w, a.w);
        }
        M = mb;
      }
      mst[sub * NI + item] = make_float2(M, L);
      ost[sub * NI + item] = a;
    }
    consumers_sync<W>();  // (every slot is read before slot `first` is rewritten)
    for (int item = tid; item < NI; item += NTH) {
      float M = -INFINITY;
#pragma unroll
      for (int sub = 0; sub < R; ++sub) M = fmaxf(M, mst[sub * NI + item].x);
      float L = 0.0f;
      float4 a = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
      for (int sub = 0; sub < R; ++sub) {
        const float2 ml = mst[sub * NI + item];
        const float4 v = ost[sub * NI + item];
        const float e = ml.x == -INFINITY ? 0.0f : fast_exp2(ml.x - M);
        L = fmaf(e, ml.y, L);
        a.x = fmaf(e, v.x, a.x);
        a.y = fmaf(e, v.y, a.y);
        a.z = fmaf(e, v.z, a.z);
        a.w = fmaf(e, v.w, a.w);
      }
      const int g = item / (D / 4);
      const int d = 4 * (item % (D / 4));
      const int h = h0 + g;
      const float av[4] = {a.x, a.y, a.z, a.w};
      if (!to_out) {  // the group's state, in the layout of a split's partial
        const long long sb = base + static_cast<long long>(first) * G + g;
        *reinterpret_cast<float4*>(p.ws_o + sb * D + d) = a;
        if (d == 0) {
          p.ws_ml[sb * 2] = L == 0.0f ? -INFINITY : M;
          p.ws_ml[sb * 2 + 1] = L;
        }
      } else if (p.partial) {
        put_state2(static_cast<long long>(h) * D + d, av[0], av[1]);
        put_state2(static_cast<long long>(h) * D + d + 2, av[2], av[3]);
        if (d == 0)
          put_state2(static_cast<long long>(p.H) * D + 2 * h, L == 0.0f ? -INFINITY : M * kLn2, L);
      } else {
        const float inv = L == 0.0f ? 0.0f : 1.0f / L;
#pragma unroll
        for (int j = 0; j < 4; ++j)
          store_from_float(p.out, (static_cast<long long>(b) * p.H + h) * D + d + j, p.out_dtype,
                           av[j] * inv);
      }
    }
  };

  if (S_ <= 2 * kMergeGroup) {
    if (!ticket(&p.counters[unit], S_)) return;
    merge(0, S_, 1, true);
  } else {
    const int ng = (S_ + kMergeGroup - 1) / kMergeGroup;
    const int grp = split / kMergeGroup;
    const int gsz = min(kMergeGroup, S_ - grp * kMergeGroup);
    // group counters follow the units' counters: [units][ng]
    const long long units = static_cast<long long>(gridDim.z) * gridDim.y;
    unsigned* gc = p.counters + units + unit * ng + grp;
    if (!ticket(gc, gsz)) return;
    merge(grp * kMergeGroup, gsz, 1, false);
    if (tid == 0) *gc = 0u;
    if (!ticket(&p.counters[unit], ng)) return;
    merge(0, ng, kMergeGroup, true);
  }
  if (tid == 0) p.counters[unit] = 0u;
}

// ---- host side ----------------------------------------------------------------

using MKernelFn = void (*)(CUtensorMap, CUtensorMap, MParams);

struct MKernelInfo {
  MKernelFn fn = nullptr;
  int smem = 0;
  int threads = 0;
};

template <int D, int G, typename SB>
MKernelInfo mk(bool qsplit) {
  MKernelInfo k;
  k.fn = qsplit ? decode_mma_kernel<D, G, SB, true> : decode_mma_kernel<D, G, SB, false>;
  k.smem = MLayout<D, G, SB>::BYTES;
  k.threads = MCfg<D>::THREADS;
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
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k.fn, k.threads, k.smem) != cudaSuccess || n < 1)
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
  cuuint32_t box[2] = {static_cast<cuuint32_t>(D / 8), static_cast<cuuint32_t>(kChunk)};
  cuuint32_t estr[2] = {1, 1};
  const CUtensorMapSwizzle swz = D == 128 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B;
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<uint32_t*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

}  // namespace

std::string& launch_detail() {
  static thread_local std::string d;
  return d;
}

bool mma_supported(int D, int G) { return (D == 128 || D == 256) && G >= 1 && G <= 8 && (G & (G - 1)) == 0; }

int mma_tokens_per_tile() { return kChunk; }

int mma_occupancy(int device, int D, int gsub, bool qsplit) {
  MKernelInfo k = pick_mma(D, gsub, kF16, qsplit);
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
  if (rows >= (1LL << 31)) {
    launch_detail() = "batch * kv_heads * capacity must be below 2^31 tokens";
    return cudaErrorInvalidValue;
  }
  CUtensorMap tmk, tmv;
  if (!encode_codes_map(&tmk, a.kq, a.D, rows) || !encode_codes_map(&tmv, a.vq, a.D, rows)) {
    launch_detail() = "cuTensorMapEncodeTiled failed for the code tiles";
    return cudaErrorInvalidValue;
  }
  MParams p{};
  p.q = a.q;
  p.q_dtype = a.q_dtype;
  p.kq = a.kq;
  p.vq = a.vq;
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
  p.chunks_per_split = pl.tiles_per_split;  // the planner's tiles are 64-token chunks here
  p.k_new = a.k_new;
  p.v_new = a.v_new;
  p.new_dtype = a.new_dtype;
  p.new_slot = a.new_slot;
  p.new_slots = a.new_slots;
  if (pl.splits > 1) {
    unsigned char* ws = static_cast<unsigned char*>(a.workspace);
    p.ws_o = reinterpret_cast<float*>(ws + pl.ws_o_off);
    p.ws_ml = reinterpret_cast<float*>(ws + pl.ws_ml_off);
    p.counters = reinterpret_cast<unsigned*>(ws + pl.ws_cnt_off);
  }
  p.err = a.err;
  p.peer_bufs = a.peer_bufs;
  p.peer_world = a.peer_world;
  p.peer_rank = a.peer_rank;
  p.B = a.B;
  dim3 grid(pl.splits, a.Hkv * pl.nsub, a.B);
  return launch_pdl(k.fn, grid, dim3(k.threads), static_cast<size_t>(k.smem), stream, tmk, tmv, p);
}

}  // namespace tq
