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
// grid = (splits, Hkv); 4 warps. Each warp takes keys of its split's range in
// turn; lane l decodes values 4l..4l+3 of each 128-value group (DPL = D/128
// groups), forms the partial dot products with the G query heads plus its 8
// QJL sign terms, a warp sum gives the scores; softmax . int4 V (lane l owns
// dims 4l..4l+3 of every group) or the scores themselves are the output.
struct CParams {
  const void* q;
  int q_dtype;
  const uint8_t* packed;  // (Hkv, N, D/block, block/2)
  const __half* radii;    // (Hkv, N, D/block)
  const uint32_t* signs;  // (Hkv, N, m/32) or null
  const __half* rnorm;    // (Hkv, N)
  const float* S;         // (m, D)
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

constexpr int kCKeys = 64;  // keys per shared-memory chunk of compressed attention

// Dynamic shared memory of compressed attention: one staged chunk of keys,
// reused at the end for the 4 warps' (o, m, l) states.
constexpr size_t cattn_smem_bytes(int D, int G) {
  const size_t chunk = static_cast<size_t>(kCKeys) * (D / 8 + 8 + D / 8 + 2 * (D / 64) + 16 + 1) * 4;
  const size_t states = static_cast<size_t>(4) * G * (D + 2) * 4;
  return chunk > states ? chunk : states;
}

__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

template <int D, int G>
__global__ void __launch_bounds__(128) compressed_attn_kernel(const CParams p,
                                                              const __grid_constant__ PolarTables T) {
  constexpr int DPL = D / 128;      // 128-value groups per key
  __shared__ float s_cs[kMaxLevels][kCB][2];
  __shared__ float s_sq[G][256];    // S q per head (m <= 256)
  __shared__ float s_q[G][D];
  __shared__ int s_last;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int split = blockIdx.x, kv = blockIdx.y;
  const int h0 = kv * G;
  pdl_wait();
  pdl_trigger();
  for (int i = tid; i < kMaxLevels * kCB * 2; i += 128) (&s_cs[0][0][0])[i] = (&T.cs[0][0][0])[i];
  for (int i = tid; i < G * D; i += 128) s_q[i / D][i % D] = load_as_float(p.q, static_cast<long long>(h0) * D + i, p.q_dtype);
  __syncthreads();
  const bool qjl = p.signs != nullptr;
  if (qjl) {
    // S q for the CTA's G heads: a warp per row of S, lanes over 4 consecutive
    // dims each (coalesced 512-byte row reads, RB rows' loads in flight),
    // summed by shuffles
    constexpr int RB = D == 128 ? 16 : 8;
    for (int r0 = w; r0 < p.m; r0 += 4 * RB) {
      float4 s4[RB][D / 128];
#pragma unroll
      for (int j = 0; j < RB; ++j) {
        const int r = r0 + 4 * j;
#pragma unroll
        for (int c = 0; c < D / 128; ++c)
          s4[j][c] = r < p.m ? reinterpret_cast<const float4*>(p.S + static_cast<long long>(r) * D + c * 128)[lane]
                             : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      }
#pragma unroll
      for (int j = 0; j < RB; ++j) {
        const int r = r0 + 4 * j;
        float a[G];
#pragma unroll
        for (int g = 0; g < G; ++g) {
          a[g] = 0.0f;
#pragma unroll
          for (int c = 0; c < D / 128; ++c) {
            const float* qq = &s_q[g][c * 128 + 4 * lane];
            a[g] = fmaf(s4[j][c].x, qq[0], fmaf(s4[j][c].y, qq[1], fmaf(s4[j][c].z, qq[2], fmaf(s4[j][c].w, qq[3], a[g]))));
          }
#pragma unroll
          for (int off = 16; off > 0; off >>= 1) a[g] += __shfl_xor_sync(0xffffffffu, a[g], off);
        }
        if (lane == 0 && r < p.m)
#pragma unroll
          for (int g = 0; g < G; ++g) s_sq[g][r] = a[g];
      }
    }
  }
  __syncthreads();
  const float qjl_c = 1.2533141373155003f / static_cast<float>(p.m > 0 ? p.m : 1);  // sqrt(pi/2)/m

  // this lane's query values and QJL terms
  float qv[G][DPL][4];
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int c = 0; c < DPL; ++c)
#pragma unroll
      for (int e = 0; e < 4; ++e) qv[g][c][e] = s_q[g][c * 128 + 4 * lane + e];
  const int block = p.block, lpb = block / 4, ll = lane % lpb, kb = lane / lpb;
  const int nbk = D / block;  // blocks per key

  float m_run[G], l_run[G], o[G][DPL][4];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m_run[g] = -INFINITY;
    l_run[g] = 0.0f;
#pragma unroll
    for (int c = 0; c < DPL; ++c)
#pragma unroll
      for (int e = 0; e < 4; ++e) o[g][c][e] = 0.0f;
  }

  const int t_begin = split * p.keys_per_split;
  const int t_end = min(p.N, t_begin + p.keys_per_split);
  // The split's keys go through shared memory kCKeys at a time: every array
  // of a chunk (angle nibbles, radii, QJL bits and norms, int4 V and its
  // scales) is one contiguous range, copied by all threads with asynchronous
  // 4-byte copies (2-byte loads for the fp16 radii and norms), so a key's
  // data costs the warps no dependent global round trips.
  extern __shared__ __align__(16) unsigned char dsm[];
  constexpr int PKW = D / 8;                    // 32-bit words of angle nibbles per key
  const int mw = p.m / 32;                      // QJL sign words per key
  uint32_t* s_pk = reinterpret_cast<uint32_t*>(dsm);                // [kCKeys][PKW]
  uint32_t* s_sg = s_pk + kCKeys * PKW;                             // [kCKeys][mw <= 8]
  uint32_t* s_vq = s_sg + kCKeys * 8;                               // [kCKeys][D/8]
  float* s_vs = reinterpret_cast<float*>(s_vq + kCKeys * (D / 8));  // [kCKeys][D/64]
  float* s_vb = s_vs + kCKeys * (D / 64);
  float* s_rad = s_vb + kCKeys * (D / 64);                          // [kCKeys][nbk <= 16]
  float* s_rn = s_rad + kCKeys * 16;                                // [kCKeys]
  const bool stage_v = p.attend && !p.vdense;
  for (int c0 = t_begin; c0 < t_end; c0 += kCKeys) {
    const int nk = min(kCKeys, t_end - c0);
    const long long row0 = static_cast<long long>(kv) * p.N + c0;
    __syncthreads();  // the previous chunk is consumed
    {
      const uint32_t* src = reinterpret_cast<const uint32_t*>(p.packed) + row0 * PKW;
      for (int i = tid; i < nk * PKW; i += 128) cp_async4(s_pk + i, src + i);
    }
    if (qjl) {
      const uint32_t* src = p.signs + row0 * mw;
      for (int i = tid; i < nk * mw; i += 128) cp_async4(s_sg + (i / mw) * 8 + i % mw, src + i);
    }
    if (stage_v) {
      const uint32_t* src = p.vq + row0 * (D / 8);
      for (int i = tid; i < nk * (D / 8); i += 128) cp_async4(s_vq + i, src + i);
      if (p.sb_f32) {
        const float* vs = reinterpret_cast<const float*>(p.vs) + row0 * (D / 64);
        const float* vb = reinterpret_cast<const float*>(p.vb) + row0 * (D / 64);
        for (int i = tid; i < nk * (D / 64); i += 128) {
          cp_async4(s_vs + i, vs + i);
          cp_async4(s_vb + i, vb + i);
        }
      }
    }
    cp_async_commit();
    // the fp16 arrays with plain loads (no 4-byte alignment), converted
    for (int i = tid; i < nk * nbk; i += 128)
      s_rad[(i / nbk) * 16 + i % nbk] = __half2float(p.radii[row0 * nbk + i]);
    if (qjl)
      for (int i = tid; i < nk; i += 128) s_rn[i] = __half2float(p.rnorm[row0 + i]);
    if (stage_v && !p.sb_f32) {
      const __half* vs = reinterpret_cast<const __half*>(p.vs) + row0 * (D / 64);
      const __half* vb = reinterpret_cast<const __half*>(p.vb) + row0 * (D / 64);
      for (int i = tid; i < nk * (D / 64); i += 128) {
        s_vs[i] = __half2float(vs[i]);
        s_vb[i] = __half2float(vb[i]);
      }
    }
    cp_async_wait_all();
    __syncthreads();

    for (int tl = w; tl < nk; tl += 4) {
      const int t = c0 + tl;
      const long long row = row0 + tl;
      const unsigned char* pkb = reinterpret_cast<const unsigned char*>(s_pk + tl * PKW);
      float part[G];
#pragma unroll
      for (int g = 0; g < G; ++g) part[g] = 0.0f;
#pragma unroll
      for (int c = 0; c < DPL; ++c) {
        const int bi = c * (128 / block) + kb;
        const unsigned char* pk = pkb + bi * (block / 2);
        const float4 kv4 = decode4([&](int i) { return packed_idx(pk, i); },
                                   s_rad[tl * 16 + bi], block, ll, s_cs);
#pragma unroll
        for (int g = 0; g < G; ++g)
          part[g] += qv[g][c][0] * kv4.x + qv[g][c][1] * kv4.y + qv[g][c][2] * kv4.z +
                     qv[g][c][3] * kv4.w;
      }
      if (qjl) {
        // lane l owns sign bits [l*m/32, (l+1)*m/32)
        const int per = p.m / 32;
        const float rn = s_rn[tl] * qjl_c;
        for (int i = lane * per; i < (lane + 1) * per; ++i) {
          const bool bit = (s_sg[tl * 8 + (i >> 5)] >> (i & 31)) & 1u;
#pragma unroll
          for (int g = 0; g < G; ++g) part[g] += rn * (bit ? s_sq[g][i] : -s_sq[g][i]);
        }
      }
#pragma unroll
      for (int g = 0; g < G; ++g) {
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) part[g] += __shfl_xor_sync(0xffffffffu, part[g], off);
        part[g] *= p.scale;
      }
      if (!p.attend) {  // scores only
        if (lane < G) {
          float v = part[0];
#pragma unroll
          for (int g = 1; g < G; ++g) v = (lane == g) ? part[g] : v;
          p.scores[static_cast<long long>(h0 + lane) * p.N + t] = v;
        }
        continue;
      }
      // online softmax (natural log) and V accumulation
#pragma unroll
      for (int c = 0; c < DPL; ++c) {
        const int d0 = c * 128 + 4 * lane;
        float vv[4];
        if (p.vdense) {
#pragma unroll
          for (int e = 0; e < 4; ++e) vv[e] = load_as_float(p.vdense, row * D + d0 + e, p.vdense_dtype);
        } else {
          const uint32_t word = s_vq[tl * (D / 8) + d0 / 8];
          const int sh = 4 * (d0 % 8);
          const float sc = s_vs[tl * (D / 64) + d0 / 64];
          const float bi = s_vb[tl * (D / 64) + d0 / 64];
#pragma unroll
          for (int e = 0; e < 4; ++e) vv[e] = fmaf(sc, static_cast<float>((word >> (sh + 4 * e)) & 15u), bi);
        }
#pragma unroll
        for (int g = 0; g < G; ++g) {
          if (c == 0) {
            const float mn = fmaxf(m_run[g], part[g]);
            const float a = (m_run[g] == -INFINITY) ? 0.0f : __expf(m_run[g] - mn);
            const float pe = __expf(part[g] - mn);
            l_run[g] = l_run[g] * a + pe;
            m_run[g] = mn;
#pragma unroll
            for (int cc = 0; cc < DPL; ++cc)
#pragma unroll
              for (int e = 0; e < 4; ++e) o[g][cc][e] *= a;
            part[g] = pe;  // reuse as this key's weight
          }
#pragma unroll
          for (int e = 0; e < 4; ++e) o[g][c][e] = fmaf(part[g], vv[e], o[g][c][e]);
        }
      }
    }
  }
  if (!p.attend) return;

  // ---- the 4 warps' states combined in shared memory (the chunk buffer is
  // free now), one partial per CTA to the workspace; the last CTA of the KV
  // head merges the splits' partials, 16 splits' loads in flight per thread
  __syncthreads();
  float* wst = reinterpret_cast<float*>(dsm);  // [4 warps][G][D + 2]
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float* ws_g = wst + (w * G + g) * (D + 2);
#pragma unroll
    for (int c = 0; c < DPL; ++c)
#pragma unroll
      for (int e = 0; e < 4; ++e) ws_g[c * 128 + 4 * lane + e] = o[g][c][e];
    if (lane == 0) {
      ws_g[D] = m_run[g];
      ws_g[D + 1] = l_run[g];
    }
  }
  __syncthreads();
  float* wsp = p.ws + (static_cast<long long>(kv) * p.splits + split) * G * (D + 2);
  for (int i = tid; i < G * D; i += 128) {
    const int g = i / D, d = i % D;
    float M = -INFINITY;
#pragma unroll
    for (int ww = 0; ww < 4; ++ww) M = fmaxf(M, wst[(ww * G + g) * (D + 2) + D]);
    float L = 0.0f, acc = 0.0f;
#pragma unroll
    for (int ww = 0; ww < 4; ++ww) {
      const float* st = wst + (ww * G + g) * (D + 2);
      const float e = st[D] == -INFINITY ? 0.0f : __expf(st[D] - M);
      L = fmaf(e, st[D + 1], L);
      if (e != 0.0f) acc = fmaf(e, st[d], acc);
    }
    wsp[g * (D + 2) + d] = acc;
    if (d == 0) {
      wsp[g * (D + 2) + D] = M;
      wsp[g * (D + 2) + D + 1] = L;
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
    float M = -INFINITY, L = 0.0f, acc = 0.0f;
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
      acc *= a;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        // an empty state (m = -inf) weighs 0; a NaN state makes the head NaN
        const float e = ms[j] == -INFINITY ? 0.0f : __expf(ms[j] - mb);
        L = fmaf(e, ls[j], L);
        if (e != 0.0f) acc = fmaf(e, os[j], acc);
      }
      M = mb;
    }
    store_from_float(p.out, static_cast<long long>(h0 + g) * D + d, p.out_dtype,
                     L == 0.0f ? 0.0f : acc / L);
  }
  if (tid == 0) p.counters[kv] = 0u;
}

template <int D>
void* pick_cattn(int G) {
  switch (G) {
    case 1: return reinterpret_cast<void*>(compressed_attn_kernel<D, 1>);
    case 2: return reinterpret_cast<void*>(compressed_attn_kernel<D, 2>);
    case 4: return reinterpret_cast<void*>(compressed_attn_kernel<D, 4>);
    case 8: return reinterpret_cast<void*>(compressed_attn_kernel<D, 8>);
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
  const int G = num_heads / num_kv_heads;
  const int s = csplits(num_kv_heads, n_keys);
  // merge counters in the counter region every workspace of this library
  // starts with (so decode and compressed calls can share one workspace)
  return kCounterRegionBytes +
         static_cast<size_t>(num_kv_heads) * s * G * (head_dim + 2) * sizeof(float);
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
  void* fn_ptr = head_dim == 128 ? pick_cattn<128>(G) : pick_cattn<256>(G);
  const size_t dsmem = cattn_smem_bytes(head_dim, G);
  cudaFuncSetAttribute(fn_ptr, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(dsmem));
  void* args[] = {&p, &T};
  const cudaError_t e = cudaLaunchKernel(fn_ptr, dim3(p.splits, num_kv_heads), dim3(128), args,
                                         dsmem,
                                         static_cast<cudaStream_t>(stream));
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
