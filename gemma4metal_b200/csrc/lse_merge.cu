// Log-sum-exp merge of partial softmax states (m, l, o), one CTA per
// (head, sequence). Used after the NCCL all-gather of per-GPU shard partials.
// Partial layout per (part, sequence): o (H, D) unnormalised, then ml (H, 2)
// with m in natural-log units and l = sum exp(score - m).
#include "tq_common.cuh"
#include "tq_internal.h"

namespace tq {

namespace {

constexpr int kMergeThreads = 128;
constexpr int kMaxParts = 64;

__global__ void __launch_bounds__(kMergeThreads) lse_merge_kernel(const float* __restrict__ parts,
                                                                  int P, int B, int H, int D,
                                                                  void* out, int out_dtype) {
  __shared__ float e[kMaxParts];
  __shared__ float Ls;
  const int h = blockIdx.x;
  const int b = blockIdx.y;
  const long long blk = static_cast<long long>(H) * (D + 2);
  const long long stride_p = static_cast<long long>(B) * blk;
  const float* base = parts + static_cast<long long>(b) * blk;
  if (threadIdx.x == 0) {
    float M = -INFINITY;
    for (int p = 0; p < P; ++p) M = fmaxf(M, base[p * stride_p + static_cast<long long>(H) * D + 2 * h]);
    float L = 0.0f;
    for (int p = 0; p < P; ++p) {
      const float m = base[p * stride_p + static_cast<long long>(H) * D + 2 * h];
      const float l = base[p * stride_p + static_cast<long long>(H) * D + 2 * h + 1];
      // an empty state (m = -inf) weighs 0; a NaN state makes the result NaN
      const float w = m == -INFINITY ? 0.0f : __expf(m - M);
      e[p] = w;
      L += w * l;
    }
    Ls = L;
  }
  __syncthreads();
  const float L = Ls;
  for (int d = threadIdx.x; d < D; d += kMergeThreads) {
    float acc = 0.0f;
    for (int p = 0; p < P; ++p)  // an empty state's o is never read
      if (e[p] != 0.0f) acc += e[p] * base[p * stride_p + static_cast<long long>(h) * D + d];
    store_from_float(out, (static_cast<long long>(b) * H + h) * D + d, out_dtype,
                     L == 0.0f ? 0.0f : acc / L);
  }
}

}  // namespace

cudaError_t launch_lse_merge(const float* parts, int n_parts, int B, int H, int D, void* out,
                             int out_dtype, cudaStream_t stream) {
  if (n_parts > kMaxParts) return cudaErrorInvalidValue;
  dim3 grid(H, B);
  lse_merge_kernel<<<grid, kMergeThreads, 0, stream>>>(parts, n_parts, B, H, D, out, out_dtype);
  return cudaGetLastError();
}

}  // namespace tq
