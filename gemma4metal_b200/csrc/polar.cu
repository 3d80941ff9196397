// PolarQuant + QJL compressed keys on sm_100a: encode, decode, QJL signs, and
// compressed-key attention (scores only, or softmax . int4 V) with GQA and
// split-KV. Reference: lib/turboquant.metal:8-224 (encode, decode, sequential
// compressed SDPA), :424-499 (compressed scores), :501-704 (packed formats and
// cos/sin tables), generalised from 16-value blocks / 4 levels to blocks of
// 2^L values (16..128; 128 = the 7 levels of the task's config 3). QJL
// (residual sign sketch) follows its paper; the reference has no code for it.
//
// Numerics shared with the CPU oracle so that angle indices, radii and QJL
// sign bits are bit-identical: the polynomial atan2 below, IEEE sqrt and
// division, explicit fmaf in a fixed order for every quantity that feeds an
// index or a sign, and cos/sin tables of the codebook entries computed on the
// host in double and rounded to fp32.
#include <cmath>
#include <cstdio>

#include "../../include/turboquant_c.h"
#include "tq_common.cuh"
#include "tq_internal.h"

namespace tq {
namespace {

constexpr int kCB = 16;         // codebook entries per level (4-bit indices)
constexpr int kMaxLevels = 7;   // blocks of up to 128 values

struct PolarTables {
  float cb[kMaxLevels][kCB];        // angle codebooks, level 1 first
  float cs[kMaxLevels][kCB][2];     // (cos, sin) of the entries
  int n[kMaxLevels];                // entries used per level
};

__device__ __forceinline__ float polar_atan2(float y, float x) {
  // odd degree-17 polynomial for atan on [0, 1] (fit: least squares on
  // Chebyshev nodes, reweighted towards minimax; max error 9.6e-8 rad)
  const float ax = fabsf(x), ay = fabsf(y);
  const float mx = fmaxf(ax, ay), mn = fminf(ax, ay);
  if (mx == 0.0f) return 0.0f;
  const float t = __fdiv_rn(mn, mx);
  const float s = __fmul_rn(t, t);
  float p = 0.0024567244108766317f;
  p = fmaf(p, s, -0.014401360414922237f);
  p = fmaf(p, s, 0.03978123515844345f);
  p = fmaf(p, s, -0.07234859466552734f);
  p = fmaf(p, s, 0.10498947650194168f);
  p = fmaf(p, s, -0.14161230623722076f);
  p = fmaf(p, s, 0.19985906779766083f);
  p = fmaf(p, s, -0.33332598209381104f);
  p = fmaf(p, s, 0.9999998807907104f);
  float a = __fmul_rn(p, t);
  if (ay > ax) a = __fsub_rn(1.5707963705062866f, a);
  if (x < 0.0f) a = __fsub_rn(3.1415927410125732f, a);
  if (y < 0.0f) a = -a;
  return a;
}

__device__ __forceinline__ int nearest(float ang, const float* cb, int n) {
  float best = 1e10f;
  int id = 0;
  for (int c = 0; c < n; ++c) {
    const float d = fabsf(__fsub_rn(ang, cb[c]));
    if (d < best) {
      best = d;
      id = c;
    }
  }
  return id;
}

__host__ __device__ constexpr int level_off(int block, int L) {
  int off = 0;
  for (int l = 1; l < L; ++l) off += block >> l;
  return off;
}

// ---- encode: one warp per 128 consecutive values; lane l holds 4 values ------
// Levels 1 and 2 stay in the lane; level L >= 3 pairs lane l with lane
// l + 2^(L-3) inside the block (lanes l with l % 2^(L-2) == 0 compute).
__global__ void __launch_bounds__(128) polar_encode_kernel(const float* __restrict__ y,
                                                           long long groups, int block,
                                                           const __grid_constant__ PolarTables T,
                                                           uint8_t* angles,
                                                           uint8_t* packed, __half* radii) {
  __shared__ uint8_t s_idx[4][128];
  // the codebooks from shared memory (a dynamically indexed kernel parameter
  // would be copied to every thread's local memory)
  __shared__ float s_cb[kMaxLevels][kCB];
  __shared__ int s_n[kMaxLevels];
  for (int i = threadIdx.x; i < kMaxLevels * kCB; i += blockDim.x) (&s_cb[0][0])[i] = (&T.cb[0][0])[i];
  if (threadIdx.x < kMaxLevels) s_n[threadIdx.x] = T.n[threadIdx.x];
  __syncthreads();
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int levels = 31 - __clz(block);
  const int lpb = block / 4;            // lanes per block
  const int ll = lane % lpb;            // lane inside its block
  const int kb = lane / lpb;            // block inside the 128 values
  for (long long g = static_cast<long long>(blockIdx.x) * 4 + w; g < groups;
       g += static_cast<long long>(gridDim.x) * 4) {
    const float4 v = reinterpret_cast<const float4*>(y + g * 128)[lane];
    uint8_t* si = s_idx[w] + kb * block;  // this block's angles, level-major
    // level 1: pairs (v.x, v.y), (v.z, v.w) = level-1 nodes 2ll, 2ll + 1
    float r1a, r1b;
    {
      float a0 = polar_atan2(v.y, v.x);
      if (a0 < 0.0f) a0 = __fadd_rn(a0, 6.2831854820251465f);
      float a1 = polar_atan2(v.w, v.z);
      if (a1 < 0.0f) a1 = __fadd_rn(a1, 6.2831854820251465f);
      si[2 * ll] = static_cast<uint8_t>(nearest(a0, s_cb[0], s_n[0]));
      si[2 * ll + 1] = static_cast<uint8_t>(nearest(a1, s_cb[0], s_n[0]));
      r1a = __fsqrt_rn(fmaf(v.x, v.x, __fmul_rn(v.y, v.y)));
      r1b = __fsqrt_rn(fmaf(v.z, v.z, __fmul_rn(v.w, v.w)));
    }
    // level 2: node ll from (r1a, r1b)
    float r = r1a;
    if (levels >= 2) {
      const float a = polar_atan2(r1b, r1a);
      si[level_off(block, 2) + ll] = static_cast<uint8_t>(nearest(a, s_cb[1], s_n[1]));
      r = __fsqrt_rn(fmaf(r1a, r1a, __fmul_rn(r1b, r1b)));
    }
    for (int L = 3; L <= levels; ++L) {
      const int step = 1 << (L - 3);
      const float other = __shfl_down_sync(0xffffffffu, r, step);
      if ((ll & ((step << 1) - 1)) == 0) {
        const float a = polar_atan2(other, r);
        si[level_off(block, L) + (ll >> (L - 2))] =
            static_cast<uint8_t>(nearest(a, s_cb[L - 1], s_n[L - 1]));
        r = __fsqrt_rn(fmaf(r, r, __fmul_rn(other, other)));
      }
    }
    if (ll == 0) radii[g * (128 / block) + kb] = __float2half_rn(r);
    __syncwarp();
    const long long blk0 = g * (128 / block);
    if (angles) {
      for (int i = lane; i < 128; i += 32) {
        const int b = i / block, j = i % block;
        if (j < block - 1) angles[(blk0 + b) * (block - 1) + j] = s_idx[w][b * block + j];
      }
    }
    if (packed) {
      for (int i = lane; i < 64; i += 32) {
        const int b = (2 * i) / block, j = (2 * i) % block;  // angles j, j+1 of block b
        const int lo = s_idx[w][b * block + j];
        const int hi = (j + 1 < block - 1) ? s_idx[w][b * block + j + 1] : 0;
        packed[(blk0 + b) * (block / 2) + j / 2] = static_cast<uint8_t>((lo & 15) | ((hi & 15) << 4));
      }
    }
    __syncwarp();
  }
}

// Angle index i of a block from the packed bytes (4-bit, low nibble first).
__device__ __forceinline__ int packed_idx(const uint8_t* pk, int i) {
  return (pk[i >> 1] >> (4 * (i & 1))) & 15;
}

// Values 4ll .. 4ll+3 of a block of `block` values: top-down products
// radius * e_top * ... * e_1 in the same order as the oracle's decode.
template <typename IdxFn>
__device__ __forceinline__ float4 decode4(IdxFn idx, float radius, int block, int ll,
                                          const float (*cs)[kCB][2]) {
  const int levels = 31 - __clz(block);
  float x = radius;
  for (int L = levels; L >= 3; --L) {
    const int node = ll >> (L - 2);             // this lane's node at level L
    const int child = (ll >> (L - 3)) & 1;      // which child the lane descends into
    const int i = idx(level_off(block, L) + node);
    x = __fmul_rn(x, cs[L - 1][i][child]);
  }
  float xa = x, xb = 0.0f;
  if (levels >= 2) {
    const int i = idx(level_off(block, 2) + ll);
    xa = __fmul_rn(x, cs[1][i][0]);
    xb = __fmul_rn(x, cs[1][i][1]);
  }
  const int ia = idx(2 * ll), ib = idx(2 * ll + 1);
  return make_float4(__fmul_rn(xa, cs[0][ia][0]), __fmul_rn(xa, cs[0][ia][1]),
                     __fmul_rn(xb, cs[0][ib][0]), __fmul_rn(xb, cs[0][ib][1]));
}

__global__ void __launch_bounds__(128) polar_decode_kernel(const uint8_t* angles,
                                                           const uint8_t* packed,
                                                           const __half* radii, long long groups,
                                                           int block,
                                                           const __grid_constant__ PolarTables T,
                                                           float* y) {
  __shared__ float s_cs[kMaxLevels][kCB][2];
  for (int i = threadIdx.x; i < kMaxLevels * kCB * 2; i += blockDim.x)
    (&s_cs[0][0][0])[i] = (&T.cs[0][0][0])[i];
  __syncthreads();
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int lpb = block / 4, ll = lane % lpb, kb = lane / lpb;
  for (long long g = static_cast<long long>(blockIdx.x) * 4 + w; g < groups;
       g += static_cast<long long>(gridDim.x) * 4) {
    const long long b = g * (128 / block) + kb;
    const float rad = __half2float(radii[b]);
    float4 out;
    if (angles) {
      const uint8_t* a = angles + b * (block - 1);
      out = decode4([&](int i) { return static_cast<int>(a[i]); }, rad, block, ll, s_cs);
    } else {
      const uint8_t* pk = packed + b * (block / 2);
      out = decode4([&](int i) { return packed_idx(pk, i); }, rad, block, ll, s_cs);
    }
    reinterpret_cast<float4*>(y + g * 128)[lane] = out;
  }
}

// ---- QJL: r = y - yhat, signs of S r (m rows), |r| -------------------------------
// A CTA takes kQjlKeys keys at a time: their residuals go to shared memory
// dim-major, S streams through shared memory in chunks of kQjlDims dims
// (transposed, one padded row per dim), and thread i accumulates (S r)_i for
// all the keys with a sequential fmaf sum over j = 0..D-1 -- the oracle's
// order, so the sign bits are bit-identical. Warp ballots pack the bits; the
// norms |r| are sequential fmaf sums too (lanes of warp 0, one key each).
constexpr int kQjlKeys = 16;
constexpr int kQjlDims = 32;
constexpr int kQjlThreads = 256;

size_t qjl_smem_bytes(int D, int m) {
  return (static_cast<size_t>(D) * kQjlKeys + static_cast<size_t>(kQjlDims) * (m + 1)) * sizeof(float);
}

__global__ void __launch_bounds__(kQjlThreads) qjl_encode_kernel(const float* __restrict__ y,
                                                                 const float* __restrict__ yhat,
                                                                 long long rows, int D,
                                                                 const float* __restrict__ S, int m,
                                                                 uint32_t* signs, __half* rnorm) {
  extern __shared__ float smq[];
  float* s_r = smq;                                  // [D][kQjlKeys]
  float* s_S = smq + static_cast<size_t>(D) * kQjlKeys;  // [kQjlDims][m + 1]
  const int tid = threadIdx.x;
  const long long batches = (rows + kQjlKeys - 1) / kQjlKeys;
  for (long long bt = blockIdx.x; bt < batches; bt += gridDim.x) {
    const long long n0 = bt * kQjlKeys;
    const int nk = static_cast<int>(min(static_cast<long long>(kQjlKeys), rows - n0));
    for (int idx = tid; idx < D * kQjlKeys; idx += kQjlThreads) {
      const int k = idx / D, j = idx % D;
      s_r[j * kQjlKeys + k] =
          k < nk ? __fsub_rn(y[(n0 + k) * D + j], yhat[(n0 + k) * D + j]) : 0.0f;
    }
    float acc[kQjlKeys];
#pragma unroll
    for (int k = 0; k < kQjlKeys; ++k) acc[k] = 0.0f;
    for (int j0 = 0; j0 < D; j0 += kQjlDims) {
      const int nj = min(kQjlDims, D - j0);
      __syncthreads();  // residuals written / previous chunk consumed
      for (int idx = tid; idx < m * kQjlDims; idx += kQjlThreads) {
        const int i = idx / kQjlDims, jj = idx % kQjlDims;
        if (jj < nj) s_S[jj * (m + 1) + i] = S[static_cast<long long>(i) * D + j0 + jj];
      }
      __syncthreads();
      if (tid < m) {
        for (int jj = 0; jj < nj; ++jj) {
          const float sv = s_S[jj * (m + 1) + tid];
          const float4* r4 = reinterpret_cast<const float4*>(s_r + (j0 + jj) * kQjlKeys);
#pragma unroll
          for (int q = 0; q < kQjlKeys / 4; ++q) {
            const float4 r = r4[q];
            acc[4 * q] = fmaf(sv, r.x, acc[4 * q]);
            acc[4 * q + 1] = fmaf(sv, r.y, acc[4 * q + 1]);
            acc[4 * q + 2] = fmaf(sv, r.z, acc[4 * q + 2]);
            acc[4 * q + 3] = fmaf(sv, r.w, acc[4 * q + 3]);
          }
        }
      }
    }
    // signs: warp w holds rows 32w .. 32w + 31 of S r for every key
    for (int k = 0; k < nk; ++k) {
      const unsigned bits = __ballot_sync(0xffffffffu, tid < m && acc[k] >= 0.0f);
      if ((tid & 31) == 0 && tid < m) signs[(n0 + k) * (m / 32) + tid / 32] = bits;
    }
    if (tid < nk) {
      float nn = 0.0f;
      for (int j = 0; j < D; ++j) {
        const float r = s_r[j * kQjlKeys + tid];
        nn = fmaf(r, r, nn);
      }
      rnorm[n0 + tid] = __float2half_rn(__fsqrt_rn(nn));
    }
    __syncthreads();  // s_r is rewritten by the next batch
  }
}

// ---- compressed-key attention ----------------------------------------------------
// grid = (splits, Hkv), 128 threads; a split's keys go through shared memory
// 128 at a time (kCChunk). Per chunk:
//  * scores, one thread per key: the PolarQuant part is q . k without
//    rebuilding k -- the angle tree evaluated bottom-up, a level-1 node
//    (values 2j, 2j+1) giving q_2j cos + q_2j+1 sin of its angle and a node
//    at level L giving cos(theta) u_left + sin(theta) u_right of its
//    children (the decode's products, lib/turboquant.metal:100-224,
//    reassociated), times the block's radius; the QJL part sums a table of
//    the signed S q sums of every 4-bit sign pattern (one lookup per 4 sign
//    bits) times |r| sqrt(pi/2) / m;
//  * the chunk's max and sum per head over the CTA, then softmax . int4 V
//    with each thread on 8 consecutive dimensions (one V word) of every
//    KV_SUB-th key: exact fp32 codes times (p * scale), the bias term summed
//    once per key and group;
// then the per-thread states are summed, one partial per CTA goes to the
// workspace and the last CTA of the KV head merges the splits.
// S q (the QJL projection of the queries) comes from cattn_sq_kernel when the
// caller gives a workspace, else every CTA computes it.
struct CParams {
  const void* q;
  int q_dtype;
  const uint8_t* packed;  // (Hkv, N, D/block, block/2)
  const __half* radii;    // (Hkv, N, D/block)
  const uint32_t* signs;  // (Hkv, N, m/32) or null
  const __half* rnorm;    // (Hkv, N)
  const float* S;         // (m, D)
  const float* sq;        // (H, m) precomputed S q, or null
  int m;
  const uint32_t* vq;     // (Hkv, N, D/8) int4 V, or null when vdense is used
  const void* vdense;     // (Hkv, N, D) dense V in vdense_dtype (the reference's fp32 values)
  int vdense_dtype;
  int attend;             // 1: softmax . V into out; 0: scores only
  const void* vs;
  const void* vb;
  int sb_f32;
  int H, Hkv, N, block;
  float scale;            // natural-log scale of the scores
  int keys_per_split;
  float* scores;          // (H, N) when scores-only
  void* out;              // (H, D)
  int out_dtype;
  float* ws;              // split partials: (Hkv, splits, G, D + 2)
  unsigned* counters;     // Hkv tickets
  int splits;
};

constexpr int kCChunk = 128;  // keys per chunk: one per thread while scoring
#ifndef TQ_CATTN_SQ_KERNEL
#define TQ_CATTN_SQ_KERNEL 1
#endif
constexpr bool kCattnSqKernel = TQ_CATTN_SQ_KERNEL != 0;  // S q in its own kernel

// Shared-memory layout of compressed attention (32-bit words; rows padded so
// that 16-byte loads of consecutive keys' rows hit distinct banks).
template <int D, int G, int BLOCK>
struct CLay {
  static constexpr int PKW = D / 8;        // angle-nibble words per key
  static constexpr int PKS = PKW + 4;      // padded row
  static constexpr int SGS = 12;           // sign words per key (<= 8 used)
  static constexpr int VQW = D / 8;        // int4 V words per key
  static constexpr int NG = D / 64;        // V groups per key
  static constexpr int NBK = D / BLOCK;    // radii per key
  static constexpr int KSUB = 128 / (D / 8);  // keys in flight in the V phase
  static constexpr int PK = 0;
  static constexpr int SG = PK + kCChunk * PKS;
  static constexpr int VQ = SG + kCChunk * SGS;
  static constexpr int VSB = VQ + kCChunk * VQW;      // (scale, bias) pairs
  static constexpr int RAD = VSB + kCChunk * NG * 2;  // [kCChunk][NBK]
  static constexpr int RN = RAD + kCChunk * NBK;
  static constexpr int P = RN + kCChunk;              // [kCChunk][G] softmax weights
  static constexpr int QT = P + kCChunk * G;          // [64][16][G] QJL nibble table
  static constexpr int Q2 = QT + 64 * 16 * G;         // [D/2][G] float2 query pairs
  static constexpr int SQ = Q2 + D * G;               // [G][256] S q
  // level-1 table [D/2][16][G]: q_2j cos + q_2j+1 sin of every codebook
  // angle, when it fits in 16 KB
  static constexpr bool U1 = (D / 2) * 16 * G <= 4096;
  static constexpr int U1T = SQ + G * 256;
  static constexpr int WORDS = U1T + (U1 ? (D / 2) * 16 * G : 0);
  // reused after the last chunk: [KSUB][G][D] per-thread output sums
  static_assert(KSUB * G * D <= WORDS, "output sums must fit in the chunk buffers");
};

template <int D, int G, int BLOCK>
constexpr size_t cattn_smem_bytes() {
  return static_cast<size_t>(CLay<D, G, BLOCK>::WORDS) * 4;
}

constexpr int ilog2c(int x) { return x <= 1 ? 0 : 1 + ilog2c(x / 2); }

template <int I, int W>
__device__ __forceinline__ int nib(const uint32_t (&w)[W]) {
  return static_cast<int>((w[I >> 3] >> (4 * (I & 7))) & 15u);
}

// Angle I's entry of a 16-entry float2 table: its byte offset (index * 8)
// taken from the nibble with one shift and one mask.
template <int I, int W>
__device__ __forceinline__ const float2& cs_entry(const float2* row, const uint32_t (&w)[W]) {
  constexpr int sh = 4 * (I & 7);
  const uint32_t off = sh >= 3 ? (w[I >> 3] >> (sh - 3)) & 0x78u : (w[I >> 3] << (3 - sh)) & 0x78u;
  return *reinterpret_cast<const float2*>(reinterpret_cast<const char*>(row) + off);
}

// q . (unit vector of node N at level L of a BLOCK-value angle tree), for G
// query heads; q2 = this block's query pairs [BLOCK/2][G], u1 (when U1) =
// this block's level-1 table [BLOCK/2][16][G].
template <int BLOCK, int L, int N, int G, bool U1>
__device__ __forceinline__ void polar_node(const uint32_t (&pkw)[BLOCK / 8],
                                           const float2* __restrict__ q2,
                                           const float* __restrict__ u1,
                                           const float2 (*cs)[kCB], float (&out)[G]) {
  if constexpr (L == 1) {
    if constexpr (U1) {
      const float* t = u1 + (N * 16 + nib<N>(pkw)) * G;
      if constexpr (G == 1) {
        out[0] = t[0];
      } else if constexpr (G == 2) {
        const float2 v = *reinterpret_cast<const float2*>(t);
        out[0] = v.x;
        out[1] = v.y;
      } else {
#pragma unroll
        for (int g0 = 0; g0 < G; g0 += 4) {
          const float4 v = *reinterpret_cast<const float4*>(t + g0);
          out[g0] = v.x;
          out[g0 + 1] = v.y;
          out[g0 + 2] = v.z;
          out[g0 + 3] = v.w;
        }
      }
    } else {
      const float2 c = cs_entry<N>(cs[0], pkw);
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float2 qq = q2[N * G + g];
        out[g] = fmaf(qq.x, c.x, qq.y * c.y);
      }
    }
  } else {
    float a[G], b[G];
    polar_node<BLOCK, L - 1, 2 * N, G, U1>(pkw, q2, u1, cs, a);
    polar_node<BLOCK, L - 1, 2 * N + 1, G, U1>(pkw, q2, u1, cs, b);
    const float2 c = cs_entry<level_off(BLOCK, L) + N>(cs[L - 1], pkw);
#pragma unroll
    for (int g = 0; g < G; ++g) out[g] = fmaf(c.x, a[g], c.y * b[g]);
  }
}

__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// nrows rows of rw 32-bit words from contiguous global memory into shared
// rows of stride ds words: 16-byte copies when rows and source allow.
__device__ __forceinline__ void stage_rows(uint32_t* dst, int ds, const uint32_t* src, int rw,
                                           int nrows, int tid) {
  if ((rw & 3) == 0 && (reinterpret_cast<uintptr_t>(src) & 15u) == 0) {
    const int r4 = rw / 4;
    for (int i = tid; i < nrows * r4; i += 128)
      cp_async16(dst + (i / r4) * ds + 4 * (i % r4), src + 4 * i);
  } else {
    for (int i = tid; i < nrows * rw; i += 128) cp_async4(dst + (i / rw) * ds + i % rw, src + i);
  }
}

// S q for H heads: CTA (rb, hb) takes rows 8 rb .. 8 rb + 7 of S (a warp per
// row, lanes over the dimensions) and heads 8 hb .. 8 hb + 7 (queries staged
// in shared memory); shuffles sum each (row, head) dot product.
constexpr int kSqRows = 8, kSqHeads = 8;
template <int D>
__global__ void __launch_bounds__(256) cattn_sq_kernel(const void* q, int q_dtype, const float* S,
                                                       int m, int H, float* sq) {
  __shared__ __align__(16) float sQ[kSqHeads][D];
  pdl_wait();
  pdl_trigger();
  const int hq0 = blockIdx.y * kSqHeads;
  for (int i = threadIdx.x; i < kSqHeads * D; i += 256) {
    const int h = i / D, d = i % D;
    sQ[h][d] = hq0 + h < H ? load_as_float(q, static_cast<long long>(hq0 + h) * D + d, q_dtype) : 0.0f;
  }
  const int lane = threadIdx.x & 31, r = blockIdx.x * kSqRows + (threadIdx.x >> 5);
  float4 s4[D / 128];
#pragma unroll
  for (int c = 0; c < D / 128; ++c)
    s4[c] = r < m ? reinterpret_cast<const float4*>(S + static_cast<long long>(r) * D + c * 128)[lane]
                  : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  __syncthreads();
  float a[kSqHeads];
#pragma unroll
  for (int h = 0; h < kSqHeads; ++h) {
    a[h] = 0.0f;
#pragma unroll
    for (int c = 0; c < D / 128; ++c) {
      const float4 q4 = reinterpret_cast<const float4*>(&sQ[h][c * 128])[lane];
      a[h] = fmaf(s4[c].x, q4.x, fmaf(s4[c].y, q4.y, fmaf(s4[c].z, q4.z, fmaf(s4[c].w, q4.w, a[h]))));
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1)
#pragma unroll
    for (int h = 0; h < kSqHeads; ++h) a[h] += __shfl_xor_sync(0xffffffffu, a[h], off);
  if (lane < kSqHeads && r < m && hq0 + lane < H) {
    float v = a[0];
#pragma unroll
    for (int h = 1; h < kSqHeads; ++h) v = lane == h ? a[h] : v;
    sq[static_cast<long long>(hq0 + lane) * m + r] = v;
  }
}

template <int D, int G, int BLOCK>
__global__ void __launch_bounds__(128) compressed_attn_kernel(const CParams p,
                                                              const __grid_constant__ PolarTables T) {
  using Ly = CLay<D, G, BLOCK>;
  constexpr int LV = ilog2c(BLOCK);
  constexpr int NBK = D / BLOCK;
  constexpr int OCT = D / 8;  // V words per key
  __shared__ float2 s_cs[kMaxLevels][kCB];
  __shared__ float s_red[2][4][G];
  __shared__ float s_m[G], s_l[G], s_a[G];
  __shared__ int s_last;
  extern __shared__ __align__(16) uint32_t dsw[];
  uint32_t* s_pk = dsw + Ly::PK;
  uint32_t* s_sg = dsw + Ly::SG;
  uint32_t* s_vq = dsw + Ly::VQ;
  float2* s_vsb = reinterpret_cast<float2*>(dsw + Ly::VSB);
  float* s_rad = reinterpret_cast<float*>(dsw + Ly::RAD);
  float* s_rn = reinterpret_cast<float*>(dsw + Ly::RN);
  float* s_p = reinterpret_cast<float*>(dsw + Ly::P);
  float* s_qt = reinterpret_cast<float*>(dsw + Ly::QT);
  float2* s_q2 = reinterpret_cast<float2*>(dsw + Ly::Q2);
  float* s_sq = reinterpret_cast<float*>(dsw + Ly::SQ);
  float* s_u1 = reinterpret_cast<float*>(dsw + Ly::U1T);

  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int split = blockIdx.x, kv = blockIdx.y;
  const int h0 = kv * G;
  const bool qjl = p.signs != nullptr;
  const int mw = p.m / 32;  // sign words per key
  const int t_begin = split * p.keys_per_split;
  const int t_end = min(p.N, t_begin + p.keys_per_split);
  const bool stage_v = p.attend && !p.vdense;
  // a chunk of keys into shared memory: the word arrays by asynchronous
  // copies (waited for by the caller), the fp16 arrays by plain loads
  auto stage = [&](int c0) {
    const int nk = min(kCChunk, t_end - c0);
    const long long row0 = static_cast<long long>(kv) * p.N + c0;
    stage_rows(s_pk, Ly::PKS, reinterpret_cast<const uint32_t*>(p.packed) + row0 * Ly::PKW, Ly::PKW, nk, tid);
    if (qjl) stage_rows(s_sg, Ly::SGS, p.signs + row0 * mw, mw, nk, tid);
    if (stage_v) stage_rows(s_vq, Ly::VQW, p.vq + row0 * Ly::VQW, Ly::VQW, nk, tid);
    cp_async_commit();
    for (int i = tid; i < nk * NBK; i += 128) s_rad[i] = __half2float(p.radii[row0 * NBK + i]);
    if (qjl)
      for (int i = tid; i < nk; i += 128) s_rn[i] = __half2float(p.rnorm[row0 + i]);
    if (stage_v) {
      for (int i = tid; i < nk * Ly::NG; i += 128) {
        const long long gi = row0 * Ly::NG + i;
        s_vsb[i] = p.sb_f32 ? make_float2(reinterpret_cast<const float*>(p.vs)[gi],
                                          reinterpret_cast<const float*>(p.vb)[gi])
                            : make_float2(__half2float(reinterpret_cast<const __half*>(p.vs)[gi]),
                                          __half2float(reinterpret_cast<const __half*>(p.vb)[gi]));
      }
    }
  };
  // Dependencies: with p.sq the preceding kernel is cattn_sq_kernel, which
  // signals its dependents only after its own wait for the kernels before
  // it, so the keys, values and queries those wrote are visible here already
  // and the first chunk and the query set-up go ahead of this kernel's wait,
  // which then covers S q alone. Without it, everything waits.
  if (!p.sq) pdl_wait();
  pdl_trigger();
  if (t_begin < t_end) stage(t_begin);  // the first chunk's loads go out before the set-up's
  for (int i = tid; i < kMaxLevels * kCB; i += 128)
    s_cs[i / kCB][i % kCB] = make_float2(T.cs[i / kCB][i % kCB][0], T.cs[i / kCB][i % kCB][1]);
  for (int i = tid; i < G * D / 2; i += 128) {
    const int g = i / (D / 2), j = i % (D / 2);
    const long long qi = static_cast<long long>(h0 + g) * D + 2 * j;
    s_q2[j * G + g] = make_float2(load_as_float(p.q, qi, p.q_dtype), load_as_float(p.q, qi + 1, p.q_dtype));
  }
  if (tid < G) {
    s_m[tid] = -INFINITY;
    s_l[tid] = 0.0f;
  }
  __syncthreads();
  if constexpr (Ly::U1) {
    // level-1 table: entry (pair j, angle v, head g)
    for (int i = tid; i < (D / 2) * 16 * G; i += 128) {
      const int g = i % G, v = (i / G) % 16, j = i / (16 * G);
      const float2 qq = s_q2[j * G + g], c = s_cs[0][v];
      s_u1[i] = fmaf(qq.x, c.x, qq.y * c.y);
    }
  }

  if (qjl) {
    if (p.sq) {
      pdl_wait();  // S q
      for (int i = tid; i < G * p.m; i += 128)
        s_sq[(i / p.m) * 256 + i % p.m] = __ldcg(p.sq + static_cast<long long>(h0 + i / p.m) * p.m + i % p.m);
    } else {
      // a warp per row of S, lanes over 4 consecutive dims each, summed by shuffles
      for (int r = w; r < p.m; r += 4) {
        float a[G];
#pragma unroll
        for (int g = 0; g < G; ++g) a[g] = 0.0f;
#pragma unroll
        for (int c = 0; c < D / 128; ++c) {
          const float4 s4 = reinterpret_cast<const float4*>(p.S + static_cast<long long>(r) * D + c * 128)[lane];
          const int j = c * 64 + 2 * lane;
#pragma unroll
          for (int g = 0; g < G; ++g) {
            const float2 q0 = s_q2[j * G + g], q1 = s_q2[(j + 1) * G + g];
            a[g] = fmaf(s4.x, q0.x, fmaf(s4.y, q0.y, fmaf(s4.z, q1.x, fmaf(s4.w, q1.y, a[g]))));
          }
        }
#pragma unroll
        for (int g = 0; g < G; ++g) {
#pragma unroll
          for (int off = 16; off > 0; off >>= 1) a[g] += __shfl_xor_sync(0xffffffffu, a[g], off);
        }
        if (lane == 0)
#pragma unroll
          for (int g = 0; g < G; ++g) s_sq[g * 256 + r] = a[g];
      }
    }
    __syncthreads();
    // table [pos][pattern][g]: sum over the 4 bits of pattern of +-(S q)_(4 pos + b)
    for (int i = tid; i < (p.m / 4) * 16 * G; i += 128) {
      const int g = i % G, v = (i / G) % 16, pos = i / (16 * G);
      float t = 0.0f;
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const float x = s_sq[g * 256 + 4 * pos + b];
        t += ((v >> b) & 1) ? x : -x;
      }
      s_qt[i] = t;
    }
  }
  const float qjl_c = 1.2533141373155003f / static_cast<float>(p.m > 0 ? p.m : 1);  // sqrt(pi/2)/m

  // V-phase thread roles: 8 dimensions (one V word) of every KSUB-th key
  const int oct = tid % OCT, ksub = tid / OCT;
  float acc[G][8], bsum[G];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    bsum[g] = 0.0f;
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[g][e] = 0.0f;
  }

  for (int c0 = t_begin; c0 < t_end; c0 += kCChunk) {
    const int nk = min(kCChunk, t_end - c0);
    const long long row0 = static_cast<long long>(kv) * p.N + c0;
    if (c0 != t_begin) {
      __syncthreads();  // the previous chunk is consumed
      stage(c0);
    }
    cp_async_wait_all();
    __syncthreads();

    // ---- scores: thread tid scores key c0 + tid for the G heads
    float s[G];
    if (tid < nk) {
      float sc[G];
#pragma unroll
      for (int g = 0; g < G; ++g) sc[g] = 0.0f;
#pragma unroll
      for (int bk = 0; bk < NBK; ++bk) {
        uint32_t pkw[BLOCK / 8];
        const uint32_t* src = s_pk + tid * Ly::PKS + bk * (BLOCK / 8);
        if constexpr (BLOCK / 8 >= 4) {
#pragma unroll
          for (int i = 0; i < BLOCK / 32; ++i) {
            const uint4 v4 = reinterpret_cast<const uint4*>(src)[i];
            pkw[4 * i] = v4.x;
            pkw[4 * i + 1] = v4.y;
            pkw[4 * i + 2] = v4.z;
            pkw[4 * i + 3] = v4.w;
          }
        } else {
          const uint2 v2 = *reinterpret_cast<const uint2*>(src);
          pkw[0] = v2.x;
          pkw[1] = v2.y;
        }
        float u[G];
        polar_node<BLOCK, LV, 0, G, Ly::U1>(pkw, s_q2 + bk * (BLOCK / 2) * G,
                                            s_u1 + bk * (BLOCK / 2) * 16 * G, s_cs, u);
        const float r = s_rad[tid * NBK + bk];
#pragma unroll
        for (int g = 0; g < G; ++g) sc[g] = fmaf(r, u[g], sc[g]);
      }
      if (qjl) {
        float qs[G];
#pragma unroll
        for (int g = 0; g < G; ++g) qs[g] = 0.0f;
        const uint32_t* sgr = s_sg + tid * Ly::SGS;
#pragma unroll
        for (int wd = 0; wd < 8; ++wd) {
          if (wd < mw) {
            const uint32_t word = sgr[wd];
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              const float* tq = s_qt + ((wd * 8 + k) * 16 + ((word >> (4 * k)) & 15u)) * G;
#pragma unroll
              for (int g = 0; g < G; ++g) qs[g] += tq[g];
            }
          }
        }
        const float rn = s_rn[tid] * qjl_c;
#pragma unroll
        for (int g = 0; g < G; ++g) sc[g] = fmaf(rn, qs[g], sc[g]);
      }
#pragma unroll
      for (int g = 0; g < G; ++g) s[g] = sc[g] * p.scale;
      if (!p.attend) {
#pragma unroll
        for (int g = 0; g < G; ++g) p.scores[static_cast<long long>(h0 + g) * p.N + c0 + tid] = s[g];
      }
    } else {
#pragma unroll
      for (int g = 0; g < G; ++g) s[g] = -INFINITY;
    }
    if (!p.attend) continue;

    // ---- the chunk's max per head, the running max, the weights and their sum
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float mx = s[g];
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      if (lane == 0) s_red[0][w][g] = mx;
    }
    __syncthreads();
    if (tid < G) {
      const float cm = fmaxf(fmaxf(s_red[0][0][tid], s_red[0][1][tid]), fmaxf(s_red[0][2][tid], s_red[0][3][tid]));
      const float mo = s_m[tid], mn = fmaxf(mo, cm);
      s_a[tid] = mo == -INFINITY ? 0.0f : __expf(mo - mn);
      s_m[tid] = mn;
    }
    __syncthreads();
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float pe = s[g] == -INFINITY ? 0.0f : __expf(s[g] - s_m[g]);
      s_p[tid * G + g] = pe;
      float sm = pe;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) sm += __shfl_xor_sync(0xffffffffu, sm, off);
      if (lane == 0) s_red[1][w][g] = sm;
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float a = s_a[g];
      bsum[g] *= a;
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[g][e] *= a;
    }
    __syncthreads();
    if (tid < G)
      s_l[tid] = fmaf(s_l[tid], s_a[tid], (s_red[1][0][tid] + s_red[1][1][tid]) + (s_red[1][2][tid] + s_red[1][3][tid]));

    // ---- softmax . V: this thread's 8 dimensions of keys ksub, ksub + KSUB, ...
    for (int tk = ksub; tk < nk; tk += Ly::KSUB) {
      float pw[G];
#pragma unroll
      for (int g = 0; g < G; ++g) pw[g] = s_p[tk * G + g];
      if (stage_v) {
        const uint32_t word = s_vq[tk * Ly::VQW + oct];
        const float2 sb = s_vsb[tk * Ly::NG + oct / 8];
        float ps[G];
#pragma unroll
        for (int g = 0; g < G; ++g) {
          ps[g] = pw[g] * sb.x;
          bsum[g] = fmaf(pw[g], sb.y, bsum[g]);
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          // the code as an exact fp32: 2^23 + c read from its bits, minus 2^23
          const float c = __uint_as_float(0x4B000000u | ((word >> (4 * e)) & 15u)) - 8388608.0f;
#pragma unroll
          for (int g = 0; g < G; ++g) acc[g][e] = fmaf(ps[g], c, acc[g][e]);
        }
      } else {
        const long long vi = (row0 + tk) * D + 8 * oct;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float v = load_as_float(p.vdense, vi + e, p.vdense_dtype);
#pragma unroll
          for (int g = 0; g < G; ++g) acc[g][e] = fmaf(pw[g], v, acc[g][e]);
        }
      }
    }
  }
  if (!p.attend) return;

  // ---- this CTA's partial: the threads' sums over their key subsets, then
  // (o, m, l) to the workspace; the last CTA of the KV head merges the splits
  __syncthreads();  // the chunk buffers are free
  float* s_o = reinterpret_cast<float*>(dsw);  // [KSUB][G][D]
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int e = 0; e < 8; ++e) s_o[(ksub * G + g) * D + 8 * oct + e] = acc[g][e] + bsum[g];
  __syncthreads();
  float* wsp = p.ws + (static_cast<long long>(kv) * p.splits + split) * G * (D + 2);
  for (int i = tid; i < G * D; i += 128) {
    const int g = i / D, d = i % D;
    float o = 0.0f;
#pragma unroll
    for (int k = 0; k < Ly::KSUB; ++k) o += s_o[(k * G + g) * D + d];
    wsp[g * (D + 2) + d] = o;
    if (d == 0) {
      wsp[g * (D + 2) + D] = s_m[g];
      wsp[g * (D + 2) + D + 1] = s_l[g];
    }
  }
  __syncthreads();
  if (tid == 0) {
    const unsigned prev = atomic_add_acq_rel(&p.counters[kv], 1u);
    s_last = prev == static_cast<unsigned>(p.splits - 1);
  }
  __syncthreads();
  if (!s_last) return;
  const int S_ = p.splits;
  const float* base = p.ws + static_cast<long long>(kv) * S_ * G * (D + 2);
  for (int i = tid; i < G * D; i += 128) {
    const int g = i / D, d = i % D;
    float M = -INFINITY, L = 0.0f, o = 0.0f;
    for (int s0 = 0; s0 < S_; s0 += 16) {
      float ms[16], ls[16], os[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int sp = s0 + j;
        const float* ps = base + (static_cast<long long>(sp) * G + g) * (D + 2);
        ms[j] = sp < S_ ? __ldcg(ps + D) : -INFINITY;
        ls[j] = sp < S_ ? __ldcg(ps + D + 1) : 0.0f;
        os[j] = sp < S_ ? __ldcg(ps + d) : 0.0f;
      }
      float mb = M;
#pragma unroll
      for (int j = 0; j < 16; ++j) mb = fmaxf(mb, ms[j]);
      const float a = M == -INFINITY ? 0.0f : __expf(M - mb);
      L *= a;
      o *= a;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        // an empty state (m = -inf) weighs 0; a NaN state makes the head NaN
        const float e = ms[j] == -INFINITY ? 0.0f : __expf(ms[j] - mb);
        L = fmaf(e, ls[j], L);
        if (e != 0.0f) o = fmaf(e, os[j], o);
      }
      M = mb;
    }
    store_from_float(p.out, static_cast<long long>(h0 + g) * D + d, p.out_dtype,
                     L == 0.0f ? 0.0f : o / L);
  }
  if (tid == 0) p.counters[kv] = 0u;
}

template <int D, int G>
void* pick_cattn_g(int block, size_t* smem) {
  switch (block) {
    case 16: *smem = cattn_smem_bytes<D, G, 16>(); return reinterpret_cast<void*>(compressed_attn_kernel<D, G, 16>);
    case 32: *smem = cattn_smem_bytes<D, G, 32>(); return reinterpret_cast<void*>(compressed_attn_kernel<D, G, 32>);
    case 64: *smem = cattn_smem_bytes<D, G, 64>(); return reinterpret_cast<void*>(compressed_attn_kernel<D, G, 64>);
    case 128: *smem = cattn_smem_bytes<D, G, 128>(); return reinterpret_cast<void*>(compressed_attn_kernel<D, G, 128>);
  }
  return nullptr;
}

template <int D>
void* pick_cattn(int G, int block, size_t* smem) {
  switch (G) {
    case 1: return pick_cattn_g<D, 1>(block, smem);
    case 2: return pick_cattn_g<D, 2>(block, smem);
    case 4: return pick_cattn_g<D, 4>(block, smem);
    case 8: return pick_cattn_g<D, 8>(block, smem);
  }
  return nullptr;
}

bool make_tables(const float* codebooks, const int* cb_sizes, int levels, PolarTables* T) {
  *T = PolarTables{};
  for (int l = 0; l < levels; ++l) {
    const int n = cb_sizes ? cb_sizes[l] : kCB;
    if (n < 1 || n > kCB) return false;
    T->n[l] = n;
    for (int c = 0; c < kCB; ++c) {
      const float th = codebooks[l * kCB + c];
      T->cb[l][c] = th;
      T->cs[l][c][0] = static_cast<float>(std::cos(static_cast<double>(th)));
      T->cs[l][c][1] = static_cast<float>(std::sin(static_cast<double>(th)));
    }
  }
  return true;
}

int levels_of(int block) {
  int l = 0;
  while ((1 << l) < block) ++l;
  return l;
}

bool valid_block(int block, int D) {
  return (block == 16 || block == 32 || block == 64 || block == 128) && D % 128 == 0;
}

int grid_for(long long groups) {
  const long long ctas = (groups + 3) / 4;
  return static_cast<int>(ctas < 4096 ? (ctas > 0 ? ctas : 1) : 4096);
}

int err(int code, const char* msg) {
  set_last_error("%s", msg);
  return code;
}

int cuda_err(cudaError_t e, const char* where) {
  set_last_error("%s: %s", where, cudaGetErrorString(e));
  return TQ_ERR_CUDA;
}

constexpr int kCSplitsMax = 64;

int csplits(int Hkv, int N) {
  int dev = 0;
  cudaGetDevice(&dev);
  const int target = device_sm_count(dev) * 4;  // 4 CTAs of 128 threads per SM
  int s = target / (Hkv > 0 ? Hkv : 1);
  s = s < 1 ? 1 : (s > kCSplitsMax ? kCSplitsMax : s);
  const int per = (N + s - 1) / (s > 0 ? s : 1);
  return per > 0 ? (N + per - 1) / per : 1;
}

size_t cattn_partials_bytes(int H, int Hkv, int D, int splits) {
  return static_cast<size_t>(Hkv) * splits * (H / Hkv) * (D + 2) * sizeof(float);
}

// ---- the reference's packed format for 16-value blocks (lib/turboquant.metal:501-600)
// level 1: 8 x 4-bit in one uint32 (low nibble first); levels 2..4: 4, 2, 1 x
// 2-bit fields in one byte each.
__global__ void pack_ref_kernel(const uint8_t* angles, long long nblocks, uint32_t* p1, uint8_t* p2,
                                uint8_t* p3, uint8_t* p4) {
  for (long long b = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; b < nblocks;
       b += static_cast<long long>(gridDim.x) * blockDim.x) {
    const uint8_t* a = angles + b * 15;
    uint32_t w = 0;
    for (int j = 0; j < 8; ++j) w |= (static_cast<uint32_t>(a[j]) & 15u) << (4 * j);
    p1[b] = w;
    uint32_t x = 0;
    for (int j = 0; j < 4; ++j) x |= (a[8 + j] & 3u) << (2 * j);
    p2[b] = static_cast<uint8_t>(x);
    p3[b] = static_cast<uint8_t>((a[12] & 3u) | ((a[13] & 3u) << 2));
    p4[b] = static_cast<uint8_t>(a[14] & 3u);
  }
}

__global__ void unpack_ref_kernel(const uint32_t* p1, const uint8_t* p2, const uint8_t* p3,
                                  const uint8_t* p4, long long nblocks, uint8_t* angles) {
  for (long long b = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; b < nblocks;
       b += static_cast<long long>(gridDim.x) * blockDim.x) {
    uint8_t* a = angles + b * 15;
    for (int j = 0; j < 8; ++j) a[j] = static_cast<uint8_t>((p1[b] >> (4 * j)) & 15u);
    for (int j = 0; j < 4; ++j) a[8 + j] = static_cast<uint8_t>((p2[b] >> (2 * j)) & 3u);
    a[12] = static_cast<uint8_t>(p3[b] & 3u);
    a[13] = static_cast<uint8_t>((p3[b] >> 2) & 3u);
    a[14] = static_cast<uint8_t>(p4[b] & 3u);
  }
}

// level-major angle bytes (block-1 per block) -> 4-bit packed (block/2 per block)
__global__ void pack4_kernel(const uint8_t* angles, long long nblocks, int block, uint8_t* packed) {
  const long long total = nblocks * (block / 2);
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long b = i / (block / 2);
    const int j = static_cast<int>(i % (block / 2)) * 2;
    const uint8_t* a = angles + b * (block - 1);
    const int lo = a[j], hi = (j + 1 < block - 1) ? a[j + 1] : 0;
    packed[i] = static_cast<uint8_t>((lo & 15) | ((hi & 15) << 4));
  }
}

// y = x P^T (transpose_p = 0) or y = x P (transpose_p = 1), D x D fp32 P.
__global__ void __launch_bounds__(256) precondition_kernel(const void* x, int x_dtype, long long rows,
                                                           int D, const float* P, int transpose_p,
                                                           float* y) {
  extern __shared__ float s_x[];  // 8 rows
  for (long long r0 = static_cast<long long>(blockIdx.x) * 8; r0 < rows;
       r0 += static_cast<long long>(gridDim.x) * 8) {
    const int nr = static_cast<int>(rows - r0 < 8 ? rows - r0 : 8);
    for (int i = threadIdx.x; i < nr * D; i += blockDim.x)
      s_x[i] = load_as_float(x, r0 * D + i, x_dtype);
    __syncthreads();
    for (int i = threadIdx.x; i < nr * D; i += blockDim.x) {
      const int rr = i / D, c = i % D;
      float acc = 0.0f;
      for (int j = 0; j < D; ++j)
        acc = fmaf(s_x[rr * D + j], transpose_p ? P[static_cast<long long>(j) * D + c]
                                                : P[static_cast<long long>(c) * D + j], acc);
      y[(r0 + rr) * D + c] = acc;
    }
    __syncthreads();
  }
}

}  // namespace
}  // namespace tq

using namespace tq;

extern "C" {

TQ_API int tq_polar_encode(const float* y, int64_t rows, int head_dim, int block,
                           const float* codebooks, const int* cb_sizes, uint8_t* angles,
                           uint8_t* packed, void* radii, void* stream) {
  if (!valid_block(block, head_dim))
    return err(TQ_ERR_UNSUPPORTED, "tq_polar_encode: block must be 16/32/64/128 and head_dim a multiple of 128");
  if (rows < 0 || !y || !codebooks || !radii || (!angles && !packed))
    return err(TQ_ERR_INVALID, "tq_polar_encode: bad arguments");
  PolarTables T;
  if (!make_tables(codebooks, cb_sizes, levels_of(block), &T))
    return err(TQ_ERR_INVALID, "tq_polar_encode: codebook sizes must be 1..16");
  const long long groups = rows * (head_dim / 128);
  if (groups == 0) return TQ_OK;
  polar_encode_kernel<<<grid_for(groups), 128, 0, static_cast<cudaStream_t>(stream)>>>(
      y, groups, block, T, angles, packed, static_cast<__half*>(radii));
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? TQ_OK : cuda_err(e, "tq_polar_encode");
}

TQ_API int tq_polar_decode(const uint8_t* angles, const uint8_t* packed, const void* radii,
                           int64_t rows, int head_dim, int block, const float* codebooks,
                           float* y, void* stream) {
  if (!valid_block(block, head_dim))
    return err(TQ_ERR_UNSUPPORTED, "tq_polar_decode: block must be 16/32/64/128 and head_dim a multiple of 128");
  if (rows < 0 || !y || !codebooks || !radii || (!angles == !packed))
    return err(TQ_ERR_INVALID, "tq_polar_decode: give exactly one of angles / packed");
  PolarTables T;
  make_tables(codebooks, nullptr, levels_of(block), &T);
  const long long groups = rows * (head_dim / 128);
  if (groups == 0) return TQ_OK;
  polar_decode_kernel<<<grid_for(groups), 128, 0, static_cast<cudaStream_t>(stream)>>>(
      angles, packed, static_cast<const __half*>(radii), groups, block, T, y);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? TQ_OK : cuda_err(e, "tq_polar_decode");
}

TQ_API int tq_qjl_encode(const float* y, const float* y_hat, int64_t rows, int head_dim,
                         const float* S, int m, uint32_t* signs, void* rnorm, void* stream) {
  if (rows < 0 || !y || !y_hat || !S || !signs || !rnorm || head_dim < 1 || head_dim > 1024 ||
      m < 32 || m % 32 != 0 || m > 256)
    return err(TQ_ERR_INVALID, "tq_qjl_encode: bad arguments (m a multiple of 32 in [32, 256])");
  if (rows == 0) return TQ_OK;
  const size_t smem = qjl_smem_bytes(head_dim, m);
  cudaFuncSetAttribute(qjl_encode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       static_cast<int>(smem));
  int dev = 0;
  cudaGetDevice(&dev);
  const long long batches = (rows + kQjlKeys - 1) / kQjlKeys;
  const long long cap = 2LL * device_sm_count(dev);
  const int grid = static_cast<int>(batches < cap ? batches : cap);
  qjl_encode_kernel<<<grid, kQjlThreads, smem, static_cast<cudaStream_t>(stream)>>>(
      y, y_hat, rows, head_dim, S, m, signs, static_cast<__half*>(rnorm));
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? TQ_OK : cuda_err(e, "tq_qjl_encode");
}

TQ_API size_t tq_compressed_sdpa_workspace_size(int num_heads, int num_kv_heads, int head_dim,
                                                int n_keys) {
  if (num_kv_heads < 1 || num_heads < num_kv_heads || n_keys < 0) return 0;
  const int s = csplits(num_kv_heads, n_keys);
  // merge counters in the counter region every workspace of this library
  // starts with (so decode and compressed calls can share one workspace),
  // the split partials, then S q for every query head (m <= 256)
  return kCounterRegionBytes + cattn_partials_bytes(num_heads, num_kv_heads, head_dim, s) +
         static_cast<size_t>(num_heads) * 256 * sizeof(float);
}

static int compressed_common(const void* q, tq_dtype q_dtype, const uint8_t* packed,
                             const void* radii, const uint32_t* signs, const void* rnorm,
                             const float* S, int m, int num_heads, int num_kv_heads, int head_dim,
                             int n_keys, int block, const float* codebooks, float scale,
                             float* scores, const uint32_t* vq, const void* vs, const void* vb,
                             tq_dtype sb_dtype, void* out, tq_dtype out_dtype, void* workspace,
                             size_t workspace_bytes, void* stream, const char* fn,
                             const void* vdense = nullptr, tq_dtype vdense_dtype = TQ_F32) {
  // key and value buffers may be NULL only for an empty context
  if (!q || !codebooks || (n_keys > 0 && (!packed || !radii || (signs && (!rnorm || !S)))))
    return err(TQ_ERR_INVALID, "compressed attention: null pointer argument");
  if (head_dim != 128 && head_dim != 256)
    return err(TQ_ERR_UNSUPPORTED, "compressed attention: head_dim must be 128 or 256");
  if (block != 16 && block != 32 && block != 64 && block != 128)
    return err(TQ_ERR_UNSUPPORTED, "compressed attention: block must be 16, 32, 64 or 128");
  if (num_kv_heads < 1 || num_heads % num_kv_heads != 0 || n_keys < 0)
    return err(TQ_ERR_INVALID, "compressed attention: bad head counts");
  const int G = num_heads / num_kv_heads;
  if (G != 1 && G != 2 && G != 4 && G != 8)
    return err(TQ_ERR_UNSUPPORTED, "compressed attention: gqa factor must be 1, 2, 4 or 8");
  if (signs && (m % 32 != 0 || m < 32 || m > 256))
    return err(TQ_ERR_INVALID, "compressed attention: m must be a multiple of 32 in [32, 256]");
  PolarTables T;
  make_tables(codebooks, nullptr, levels_of(block), &T);
  CParams p{};
  p.q = q;
  p.q_dtype = q_dtype;
  p.packed = packed;
  p.radii = static_cast<const __half*>(radii);
  p.signs = signs;
  p.rnorm = static_cast<const __half*>(rnorm);
  p.S = S;
  p.m = signs ? m : 0;
  p.vq = vq;
  p.vdense = vdense;
  p.vdense_dtype = vdense_dtype;
  p.attend = out != nullptr;
  p.vs = vs;
  p.vb = vb;
  p.sb_f32 = sb_dtype == TQ_F32;
  p.H = num_heads;
  p.Hkv = num_kv_heads;
  p.N = n_keys;
  p.block = block;
  p.scale = scale;
  p.scores = scores;
  p.out = out;
  p.out_dtype = out_dtype;
  const bool attend = out != nullptr;
  const int splits = attend ? csplits(num_kv_heads, n_keys) : (n_keys + 127) / 128;
  p.splits = splits > 0 ? splits : 1;
  p.keys_per_split = (n_keys + p.splits - 1) / p.splits;
  if (attend) {
    const size_t need = tq_compressed_sdpa_workspace_size(num_heads, num_kv_heads, head_dim, n_keys);
    if (!workspace || workspace_bytes < need) {
      set_last_error("%s: workspace of %zu bytes needed", fn, need);
      return TQ_ERR_WORKSPACE;
    }
    p.counters = static_cast<unsigned*>(workspace);
    p.ws = reinterpret_cast<float*>(static_cast<unsigned char*>(workspace) + kCounterRegionBytes);
    if (num_kv_heads * sizeof(unsigned) > kCounterRegionBytes)
      return err(TQ_ERR_UNSUPPORTED, "compressed attention: too many KV heads");
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (attend && signs && n_keys > 0 && kCattnSqKernel) {
    // S q once per query head into the workspace (after the split partials)
    float* sq = reinterpret_cast<float*>(static_cast<unsigned char*>(workspace) + kCounterRegionBytes +
                                         cattn_partials_bytes(num_heads, num_kv_heads, head_dim,
                                                              p.splits));
    const dim3 sgrid((m + kSqRows - 1) / kSqRows, (num_heads + kSqHeads - 1) / kSqHeads);
    const cudaError_t e =
        head_dim == 128
            ? launch_pdl(cattn_sq_kernel<128>, sgrid, dim3(256), 0, st, q, static_cast<int>(q_dtype), S, m,
                         num_heads, sq)
            : launch_pdl(cattn_sq_kernel<256>, sgrid, dim3(256), 0, st, q, static_cast<int>(q_dtype), S, m,
                         num_heads, sq);
    if (e != cudaSuccess) return cuda_err(e, fn);
    p.sq = sq;
  }
  size_t dsmem = 0;
  void* fn_ptr = head_dim == 128 ? pick_cattn<128>(G, block, &dsmem) : pick_cattn<256>(G, block, &dsmem);
  cudaFuncSetAttribute(fn_ptr, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(dsmem));
  void* args[] = {&p, &T};
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.splits, num_kv_heads);
  cfg.blockDim = dim3(128);
  cfg.dynamicSmemBytes = dsmem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_launches() ? 1 : 0;
  const cudaError_t e = cudaLaunchKernelExC(&cfg, fn_ptr, args);
  return e == cudaSuccess ? TQ_OK : cuda_err(e, fn);
}

TQ_API int tq_compressed_score(const void* queries, tq_dtype q_dtype, const uint8_t* packed,
                               const void* radii, const uint32_t* signs, const void* rnorm,
                               const float* S, int m, int num_heads, int num_kv_heads,
                               int head_dim, int n_keys, int block, const float* codebooks,
                               float scale, float* scores, void* stream) {
  if (!scores) return err(TQ_ERR_INVALID, "tq_compressed_score: null scores");
  return compressed_common(queries, q_dtype, packed, radii, signs, rnorm, S, m, num_heads,
                           num_kv_heads, head_dim, n_keys, block, codebooks, scale, scores,
                           nullptr, nullptr, nullptr, TQ_F16, nullptr, TQ_F32, nullptr, 0, stream,
                           "tq_compressed_score");
}

TQ_API int tq_compressed_sdpa(const void* queries, tq_dtype q_dtype, const uint8_t* packed,
                              const void* radii, const uint32_t* signs, const void* rnorm,
                              const float* S, int m, int num_heads, int num_kv_heads,
                              int head_dim, int n_keys, int block, const float* codebooks,
                              float scale, const uint32_t* v_quant, const void* v_scales,
                              const void* v_biases, tq_dtype sb_dtype, void* out,
                              tq_dtype out_dtype, void* workspace, size_t workspace_bytes,
                              void* stream) {
  if (!out || (n_keys > 0 && (!v_quant || !v_scales || !v_biases)))
    return err(TQ_ERR_INVALID, "tq_compressed_sdpa: null V or out");
  return compressed_common(queries, q_dtype, packed, radii, signs, rnorm, S, m, num_heads,
                           num_kv_heads, head_dim, n_keys, block, codebooks, scale, nullptr,
                           v_quant, v_scales, v_biases, sb_dtype, out, out_dtype, workspace,
                           workspace_bytes, stream, "tq_compressed_sdpa");
}

TQ_API int tq_compressed_sdpa_dense_v(const void* queries, tq_dtype q_dtype, const uint8_t* packed,
                                      const void* radii, const uint32_t* signs, const void* rnorm,
                                      const float* S, int m, int num_heads, int num_kv_heads,
                                      int head_dim, int n_keys, int block, const float* codebooks,
                                      float scale, const void* values, tq_dtype v_dtype, void* out,
                                      tq_dtype out_dtype, void* workspace, size_t workspace_bytes,
                                      void* stream) {
  if (!out || (n_keys > 0 && !values))
    return err(TQ_ERR_INVALID, "tq_compressed_sdpa_dense_v: null values or out");
  return compressed_common(queries, q_dtype, packed, radii, signs, rnorm, S, m, num_heads,
                           num_kv_heads, head_dim, n_keys, block, codebooks, scale, nullptr,
                           nullptr, nullptr, nullptr, TQ_F16, out, out_dtype, workspace,
                           workspace_bytes, stream, "tq_compressed_sdpa_dense_v", values, v_dtype);
}

}  // extern "C"

extern "C" {

TQ_API int tq_polar_pack_ref(const uint8_t* angles, int64_t n_blocks, uint32_t* packed_l1,
                             uint8_t* packed_l2, uint8_t* packed_l3, uint8_t* packed_l4,
                             void* stream) {
  if (n_blocks < 0 || (n_blocks > 0 && (!angles || !packed_l1 || !packed_l2 || !packed_l3 || !packed_l4)))
    return err(TQ_ERR_INVALID, "tq_polar_pack_ref: bad arguments");
  if (n_blocks == 0) return TQ_OK;
  const int grid = static_cast<int>((n_blocks + 255) / 256 < 4096 ? (n_blocks + 255) / 256 : 4096);
  pack_ref_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(angles, n_blocks, packed_l1,
                                                                      packed_l2, packed_l3, packed_l4);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? TQ_OK : cuda_err(e, "tq_polar_pack_ref");
}

TQ_API int tq_polar_unpack_ref(const uint32_t* packed_l1, const uint8_t* packed_l2,
                               const uint8_t* packed_l3, const uint8_t* packed_l4, int64_t n_blocks,
                               uint8_t* angles, void* stream) {
  if (n_blocks < 0 || (n_blocks > 0 && (!angles || !packed_l1 || !packed_l2 || !packed_l3 || !packed_l4)))
    return err(TQ_ERR_INVALID, "tq_polar_unpack_ref: bad arguments");
  if (n_blocks == 0) return TQ_OK;
  const int grid = static_cast<int>((n_blocks + 255) / 256 < 4096 ? (n_blocks + 255) / 256 : 4096);
  unpack_ref_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(packed_l1, packed_l2,
                                                                        packed_l3, packed_l4, n_blocks,
                                                                        angles);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? TQ_OK : cuda_err(e, "tq_polar_unpack_ref");
}

}  // extern "C"

extern "C" {

TQ_API int tq_polar_pack4(const uint8_t* angles, int64_t n_blocks, int block, uint8_t* packed,
                          void* stream) {
  if (n_blocks < 0 || block < 2 || block > 128 || (n_blocks > 0 && (!angles || !packed)))
    return err(TQ_ERR_INVALID, "tq_polar_pack4: bad arguments");
  if (n_blocks == 0) return TQ_OK;
  const long long total = n_blocks * (block / 2);
  const int grid = static_cast<int>((total + 255) / 256 < 4096 ? (total + 255) / 256 : 4096);
  pack4_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(angles, n_blocks, block, packed);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? TQ_OK : cuda_err(e, "tq_polar_pack4");
}

TQ_API int tq_precondition(const void* x, tq_dtype x_dtype, int64_t rows, int head_dim,
                           const float* P, int transpose_p, float* y, void* stream) {
  if (rows < 0 || head_dim < 1 || head_dim > 1024 || (rows > 0 && (!x || !P || !y)))
    return err(TQ_ERR_INVALID, "tq_precondition: bad arguments");
  if (rows == 0) return TQ_OK;
  const long long ctas = (rows + 7) / 8;
  const int grid = static_cast<int>(ctas < 4096 ? ctas : 4096);
  precondition_kernel<<<grid, 256, 8 * head_dim * sizeof(float), static_cast<cudaStream_t>(stream)>>>(
      x, x_dtype, rows, head_dim, P, transpose_p, y);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? TQ_OK : cuda_err(e, "tq_precondition");
}

}  // extern "C"
