// Affine group-64 4-bit quantization, dequantization and quantize-on-append.
//
// One thread produces one packed uint32 word (8 values); the 8 threads of a
// 64-value group exchange min/max with three xor-shuffles. All arithmetic is
// IEEE round-to-nearest (explicit __fsub_rn/__fdiv_rn, rintf = ties-to-even)
// so the packed cache is bit-identical to the CPU oracle.
#include "tq_common.cuh"
#include "tq_internal.h"

namespace tq {

namespace {

struct QuantRows {
  const void* x;       // rows of D values, row r at x + r*D
  int x_dtype;
  long long rows;
  int D;
  // destination: row r -> (b, h, i) with i fastest; slot = pos_b + i
  long long n_new;
  int Hkv, capacity;
  long long bstride_tok;  // tokens between consecutive sequences of the cache
  int pos;
  const int32_t* positions;  // nullable, per-sequence slot (+ pos_bias)
  int pos_bias;
  uint32_t* codes;
  void* scales;
  void* biases;
  int sb_dtype;
  // optional second tensor (V of a K/V append) handled by blockIdx.y == 1
  const void* x2;
  uint32_t* codes2;
  void* scales2;
  void* biases2;
};

__global__ void __launch_bounds__(256) quantize_rows_kernel(QuantRows p) {
  pdl_wait();
  pdl_trigger();
  if (blockIdx.y == 1) {  // second tensor: same geometry, other buffers
    p.x = p.x2;
    p.codes = p.codes2;
    p.scales = p.scales2;
    p.biases = p.biases2;
  }
  const int words_per_row = p.D / 8;
  const long long word = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long total = p.rows * words_per_row;
  // Threads past the end still take part in the group shuffles (full warps),
  // but neither load nor store.
  const bool live = word < total;
  const long long r = live ? word / words_per_row : 0;
  const int w = static_cast<int>(live ? word % words_per_row : 0);

  float v[8];
  if (live) {
    load8_aligned(p.x, r * p.D + w * 8, p.x_dtype, v);
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = 0.0f;
  }
  float mn, mx;
  group_minmax8(v, mn, mx);
  if (!live) return;

  // destination slot
  const long long i = r % p.n_new;
  const long long bh = r / p.n_new;
  const int h = static_cast<int>(bh % p.Hkv);
  const long long b = bh / p.Hkv;
  const int base = p.positions ? p.positions[b] + p.pos_bias : p.pos;
  // a device-provided position outside the cache writes nothing
  if (p.positions && (base < 0 || base + i >= p.capacity)) return;
  const long long tok = b * p.bstride_tok + static_cast<long long>(h) * p.capacity + base + i;

  const int g = w / 8;
  const long long sidx = tok * (p.D / 64) + g;
  const bool leader = (w % 8) == 0;
  p.codes[tok * words_per_row + w] =
      quantize_word8(v, mn, mx, p.sb_dtype, p.scales, p.biases, sidx, leader);
}

template <typename OUT>
__global__ void __launch_bounds__(256) dequantize_kernel(const uint32_t* codes, const void* scales,
                                                         const void* biases, int sb_dtype,
                                                         long long rows, int D, void* out,
                                                         int out_dtype) {
  const int words_per_row = D / 8;
  const long long word = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (word >= rows * words_per_row) return;
  const long long r = word / words_per_row;
  const int w = static_cast<int>(word % words_per_row);
  const long long sidx = r * (D / 64) + w / 8;
  const float s = load_as_float(scales, sidx, sb_dtype);
  const float b = load_as_float(biases, sidx, sb_dtype);
  const uint32_t c = codes[word];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float val = __fadd_rn(__fmul_rn(s, static_cast<float>((c >> (4 * j)) & 0xFu)), b);
    store_from_float(out, r * D + w * 8 + j, out_dtype, val);
  }
}

}  // namespace

cudaError_t launch_quantize_rows(const void* x, int x_dtype, long long rows, int D, long long n_new,
                                 int Hkv, int capacity, long long bstride_tok, int pos,
                                 const int32_t* positions, uint32_t* codes, void* scales,
                                 void* biases, int sb_dtype, cudaStream_t stream, const void* x2,
                                 uint32_t* codes2, void* scales2, void* biases2, int pos_bias) {
  QuantRows p;
  p.pos_bias = pos_bias;
  p.x2 = x2;
  p.codes2 = codes2;
  p.scales2 = scales2;
  p.biases2 = biases2;
  p.x = x;
  p.x_dtype = x_dtype;
  p.rows = rows;
  p.D = D;
  p.n_new = n_new;
  p.Hkv = Hkv;
  p.capacity = capacity;
  p.bstride_tok = bstride_tok;
  p.pos = pos;
  p.positions = positions;
  p.codes = codes;
  p.scales = scales;
  p.biases = biases;
  p.sb_dtype = sb_dtype;
  const long long words = rows * (D / 8);
  if (words == 0) return cudaSuccess;
  const unsigned blocks = static_cast<unsigned>((words + 255) / 256);
  return launch_pdl(quantize_rows_kernel, dim3(blocks, x2 ? 2 : 1), dim3(256), 0, stream, p);
}

cudaError_t launch_dequantize(const uint32_t* codes, const void* scales, const void* biases,
                              int sb_dtype, long long rows, int D, void* out, int out_dtype,
                              cudaStream_t stream) {
  const long long words = rows * (D / 8);
  if (words == 0) return cudaSuccess;
  const unsigned blocks = static_cast<unsigned>((words + 255) / 256);
  dequantize_kernel<float><<<blocks, 256, 0, stream>>>(codes, scales, biases, sb_dtype, rows, D,
                                                       out, out_dtype);
  return cudaGetLastError();
}

}  // namespace tq
