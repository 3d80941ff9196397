/*
 * CPU oracle for the int4 KV-cache decode-attention path.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the checker that the CUDA library is
 * compared against (tests/, __graft_entry__.smoke(), bench.py's cpu_baseline and
 * `--impl reference` arm). Nothing in gemma4metal_b200/ links or calls it.
 *
 * PARITY UNPINNED against the reference's own outputs: the reference path is
 * Metal + MLX (lib/turboquant.metal, MLX quantize/dequantize/fast::sdpa), which
 * cannot be built or imported on Linux, and the reference ships no golden
 * vectors (tests/test_sdpa_int4.cpp:20-22 draws unseeded random inputs). This
 * restatement is pinned instead to the packing/quantization spec of the task
 * (affine group-64 4-bit, fp16 scale/bias, low nibble first) by the known-answer
 * tests in tests/test_oracle.py, and to the reference formulas cited below.
 *
 * Restated reference behaviour (file:line within svv232/gemma4metal):
 *   dequantize value = scale * nibble + bias            lib/turboquant.metal:718-720
 *   nibble j of a uint32 word sits at bits 4j..4j+3     lib/turboquant.metal:796-799, 823-826
 *   GQA map kv_head = head / gqa_factor                 lib/turboquant.metal:745
 *   sliding window: token t skipped if (N-1-t) >= W     lib/turboquant.metal:779
 *   scale multiplies q before the dot product           lib/turboquant.metal:762-765
 *   empty softmax (sum == 0) writes 0                   lib/turboquant.metal:886
 *   baseline path = dequantize then fp32 SDPA           engine/gemma4_multilayer.cpp:307-308,349
 *                                                       tests/test_sdpa_int4.cpp:31-41
 *
 * Build: see oracle/build_oracle.py (gcc -O3 -fopenmp -ffp-contract=off).
 * -ffp-contract=off keeps every a*b+c as two IEEE roundings, so the numpy
 * restatement in oracle/oracle.py reproduces the quantizer bit for bit.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

enum { TQO_F32 = 0, TQO_F16 = 1, TQO_BF16 = 2 };

/* ---- 16-bit float conversions (IEEE round-to-nearest-even) ---------------- */

uint16_t tqo_f32_to_f16(float x) {
  _Float16 h = (_Float16)x; /* gcc: IEEE RNE conversion */
  uint16_t u;
  memcpy(&u, &h, 2);
  return u;
}

float tqo_f16_to_f32(uint16_t u) {
  _Float16 h;
  memcpy(&h, &u, 2);
  return (float)h;
}

uint16_t tqo_f32_to_bf16(float x) {
  uint32_t u;
  memcpy(&u, &x, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u); /* quiet NaN */
  uint32_t lsb = (u >> 16) & 1u;
  u += 0x7fffu + lsb;
  return (uint16_t)(u >> 16);
}

float tqo_bf16_to_f32(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

static inline float load_elem(const void* p, int64_t i, int dtype) {
  switch (dtype) {
    case TQO_F16: return tqo_f16_to_f32(((const uint16_t*)p)[i]);
    case TQO_BF16: return tqo_bf16_to_f32(((const uint16_t*)p)[i]);
    default: return ((const float*)p)[i];
  }
}

/* Round x to the storage dtype and back (the value a kernel reads back). */
static inline float round_to(float x, int dtype, void* dst, int64_t i) {
  switch (dtype) {
    case TQO_F16: {
      uint16_t h = tqo_f32_to_f16(x);
      if (dst) ((uint16_t*)dst)[i] = h;
      return tqo_f16_to_f32(h);
    }
    case TQO_BF16: {
      uint16_t h = tqo_f32_to_bf16(x);
      if (dst) ((uint16_t*)dst)[i] = h;
      return tqo_bf16_to_f32(h);
    }
    default:
      if (dst) ((float*)dst)[i] = x;
      return x;
  }
}

/* ---- affine group-64 4-bit quantizer ----------------------------------------
 * Spec (task configs[0]): per group of 64 consecutive values along head_dim,
 *   scale = (max - min) / 15, bias = min, both rounded to the storage dtype;
 *   code  = clamp(rint((x - bias_s) / scale_s), 0, 15) using the ROUNDED
 *           scale_s / bias_s (what dequantize will see), ties to even;
 *   scale_s == 0 (constant group) -> every code 0.
 * Codes are packed 8 per uint32, element 8w+j of a row at bits 4j..4j+3 of
 * word w (lib/turboquant.metal:796-799).
 * Reference call sites: engine/gemma4_multilayer.cpp:228-229 (quantize on
 * append), tests/test_sdpa_int4.cpp:25-26.
 */
void tqo_quantize_rows(const void* x, int x_dtype, int64_t rows, int D, int sb_dtype,
                       uint32_t* codes, void* scales, void* biases) {
  const int ng = D / 64;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    for (int g = 0; g < ng; ++g) {
      float v[64];
      float mn = INFINITY, mx = -INFINITY;
      for (int j = 0; j < 64; ++j) {
        v[j] = load_elem(x, r * D + g * 64 + j, x_dtype);
        mn = v[j] < mn ? v[j] : mn;
        mx = v[j] > mx ? v[j] : mx;
      }
      const float scale_f = (mx - mn) / 15.0f;
      const int64_t si = r * ng + g;
      const float s = round_to(scale_f, sb_dtype, scales, si);
      const float b = round_to(mn, sb_dtype, biases, si);
      for (int w = 0; w < 8; ++w) {
        uint32_t word = 0;
        for (int j = 0; j < 8; ++j) {
          uint32_t c = 0;
          if (s != 0.0f) {
            float t = rintf((v[w * 8 + j] - b) / s);
            t = t < 0.0f ? 0.0f : (t > 15.0f ? 15.0f : t);
            c = (uint32_t)t;
          }
          word |= c << (4 * j);
        }
        codes[r * (D / 8) + g * 8 + w] = word;
      }
    }
  }
}

/* value = scale * code + bias (lib/turboquant.metal:718-720), fp32 */
void tqo_dequantize_rows(const uint32_t* codes, const void* scales, const void* biases,
                         int sb_dtype, int64_t rows, int D, float* out) {
  const int ng = D / 64;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    for (int d = 0; d < D; ++d) {
      const uint32_t c = (codes[r * (D / 8) + d / 8] >> (4 * (d % 8))) & 0xFu;
      const float s = load_elem(scales, r * ng + d / 64, sb_dtype);
      const float b = load_elem(biases, r * ng + d / 64, sb_dtype);
      out[r * D + d] = s * (float)c + b;
    }
  }
}

/* ---- single-query SDPA on dense fp32 K/V -------------------------------------
 * q: (B, H, D) fp32; k, v: (B, Hkv, cap, D) fp32 (only the first n_tokens[b]
 * rows of each head are read); out: (B, H, D) fp32.
 * Visible tokens: [max(0, N-W), N) when W > 0 else [0, N)
 * (lib/turboquant.metal:779). Scores s_t = sum_d (scale*q_d) * k_td
 * (lib/turboquant.metal:762), softmax with max subtraction, sum == 0 -> 0.
 * use_f64 != 0 accumulates everything in double (cross-check).
 */
void tqo_sdpa_dense(const float* q, const float* k, const float* v, int B, int H, int Hkv,
                    int cap, int D, const int* n_tokens, float scale, int window, int use_f64,
                    float* out) {
  const int G = H / Hkv;
#pragma omp parallel for collapse(2) schedule(dynamic, 1)
  for (int b = 0; b < B; ++b) {
    for (int h = 0; h < H; ++h) {
      const int N = n_tokens[b];
      const int kv = h / G;
      const int t0 = (window > 0 && N - window > 0) ? N - window : 0;
      const float* qh = q + ((int64_t)b * H + h) * D;
      const float* kb = k + ((int64_t)b * Hkv + kv) * cap * D;
      const float* vb = v + ((int64_t)b * Hkv + kv) * cap * D;
      float* oh = out + ((int64_t)b * H + h) * D;
      const int n = N - t0;
      if (n <= 0) {
        for (int d = 0; d < D; ++d) oh[d] = 0.0f;
        continue;
      }
      if (use_f64) {
        double* sc = (double*)malloc(sizeof(double) * n);
        double* acc = (double*)calloc(D, sizeof(double));
        double m = -INFINITY, l = 0.0;
        for (int i = 0; i < n; ++i) {
          const float* kt = kb + (int64_t)(t0 + i) * D;
          double s = 0.0;
          for (int d = 0; d < D; ++d) s += (double)scale * (double)qh[d] * (double)kt[d];
          sc[i] = s;
          m = s > m ? s : m;
        }
        for (int i = 0; i < n; ++i) {
          const double p = exp(sc[i] - m);
          l += p;
          const float* vt = vb + (int64_t)(t0 + i) * D;
          for (int d = 0; d < D; ++d) acc[d] += p * (double)vt[d];
        }
        for (int d = 0; d < D; ++d) oh[d] = l == 0.0 ? 0.0f : (float)(acc[d] / l);
        free(sc);
        free(acc);
      } else {
        float* sc = (float*)malloc(sizeof(float) * n);
        float* acc = (float*)calloc(D, sizeof(float));
        float* qs = (float*)malloc(sizeof(float) * D);
        float m = -INFINITY, l = 0.0f;
        for (int d = 0; d < D; ++d) qs[d] = scale * qh[d];
        for (int i = 0; i < n; ++i) {
          const float* kt = kb + (int64_t)(t0 + i) * D;
          float s = 0.0f;
          for (int d = 0; d < D; ++d) s += qs[d] * kt[d];
          sc[i] = s;
          m = s > m ? s : m;
        }
        for (int i = 0; i < n; ++i) {
          const float p = expf(sc[i] - m);
          l += p;
          const float* vt = vb + (int64_t)(t0 + i) * D;
          for (int d = 0; d < D; ++d) acc[d] += p * vt[d];
        }
        for (int d = 0; d < D; ++d) oh[d] = l == 0.0f ? 0.0f : acc[d] / l;
        free(sc);
        free(acc);
        free(qs);
      }
    }
  }
}

/* ---- the reference's baseline path: dequantize the int4 cache, then SDPA ----
 * engine/gemma4_multilayer.cpp:307-308 (dequantize K and V to fp32) followed by
 * engine/gemma4_multilayer.cpp:349 (fast::scaled_dot_product_attention).
 * q: (B, H, D) in q_dtype; cache arrays (B, Hkv, cap, D/8) / (B, Hkv, cap, D/64);
 * scratch_k/scratch_v: caller buffers of B*Hkv*cap*D floats (the dequantized
 * temporaries the fused kernel avoids, README.md:15-20).
 */
void tqo_sdpa_int4(const void* q, int q_dtype, const uint32_t* kq, const void* ks, const void* kb,
                   const uint32_t* vq, const void* vs, const void* vb, int sb_dtype, int B, int H,
                   int Hkv, int cap, int D, const int* n_tokens, float scale, int window,
                   int use_f64, float* scratch_k, float* scratch_v, float* out) {
  const int64_t rows = (int64_t)B * Hkv * cap;
  const int ng = D / 64;
  /* dequantize only the visible rows of each head (the baseline dequantizes
     the whole live cache; rows past n_tokens are not part of the cache) */
#pragma omp parallel for collapse(2) schedule(static)
  for (int64_t bh = 0; bh < (int64_t)B * Hkv; ++bh) {
    for (int t = 0; t < cap; ++t) {
      const int b = (int)(bh / Hkv);
      if (t >= n_tokens[b]) continue;
      const int64_t r = bh * cap + t;
      for (int d = 0; d < D; ++d) {
        const uint32_t c = (kq[r * (D / 8) + d / 8] >> (4 * (d % 8))) & 0xFu;
        const uint32_t cv = (vq[r * (D / 8) + d / 8] >> (4 * (d % 8))) & 0xFu;
        scratch_k[r * D + d] =
            load_elem(ks, r * ng + d / 64, sb_dtype) * (float)c + load_elem(kb, r * ng + d / 64, sb_dtype);
        scratch_v[r * D + d] =
            load_elem(vs, r * ng + d / 64, sb_dtype) * (float)cv + load_elem(vb, r * ng + d / 64, sb_dtype);
      }
    }
  }
  (void)rows;
  float* qf = (float*)malloc(sizeof(float) * (size_t)B * H * D);
  for (int64_t i = 0; i < (int64_t)B * H * D; ++i) qf[i] = load_elem(q, i, q_dtype);
  tqo_sdpa_dense(qf, scratch_k, scratch_v, B, H, Hkv, cap, D, n_tokens, scale, window, use_f64, out);
  free(qf);
}

/* ---- "oracle B": the reference kernel's own arithmetic order ---------------
 * Plain-C restatement of sdpa_int4_vector<D,BN> (lib/turboquant.metal:723-889)
 * for one query head: 32 lanes each own D/32 contiguous dims (:742,757); the
 * query is pre-scaled and pre-divided by {1,16,256,4096} (:759-770); K is read
 * as uint16 words and masked without shifting (:787-803); simdgroup g strides
 * over tokens ki = g, g+BN, ... (:778) with an online softmax (:807-812);
 * V is unpacked to s*code+b (:814-831); the BN partials are merged through
 * a max/sum exchange and a serial BN-pass accumulation (:838-888).
 * fast::exp is replaced by expf. Scales/biases are read as fp32 (:725-731).
 * Generalised to any D that is a multiple of 128 (the reference dispatches
 * only 256 and 512: lib/turboquant.cpp:378). BN = 32 for D <= 256, else 16
 * (lib/turboquant.cpp:398-399).
 */
void tqo_reference_kernel(const float* q, const uint32_t* kq, const float* ks, const float* kb,
                          const uint32_t* vq, const float* vs, const float* vb, int H, int gqa,
                          int N, int D, float scale, int window, float* out) {
  const int BN = D <= 256 ? 32 : 16;
  const int epl = D / 32;
  const int kpd = D / 8, ksd = D / 64;
#pragma omp parallel for schedule(dynamic, 1)
  for (int h = 0; h < H; ++h) {
    const int kvh = h / gqa;
    const uint16_t* kw16 = (const uint16_t*)(kq + (int64_t)kvh * N * kpd);
    const uint16_t* vw16 = (const uint16_t*)(vq + (int64_t)kvh * N * kpd);
    const float* ksb = ks + (int64_t)kvh * N * ksd;
    const float* kbb = kb + (int64_t)kvh * N * ksd;
    const float* vsb = vs + (int64_t)kvh * N * ksd;
    const float* vbb = vb + (int64_t)kvh * N * ksd;
    float* mxs = (float*)malloc(sizeof(float) * BN);
    float* sms = (float*)malloc(sizeof(float) * BN);
    float* o = (float*)calloc((size_t)BN * D, sizeof(float)); /* o[sg][lane*epl+i] */
    for (int sg = 0; sg < BN; ++sg) {
      float max_score = -1e30f, sum_exp = 0.0f;
      float* osg = o + (int64_t)sg * D;
      for (int ki = sg; ki < N; ki += BN) {
        if (window > 0 && (N - 1 - ki) >= window) continue;
        float lane_scores[32];
        for (int lane = 0; lane < 32; ++lane) {
          const int ls = lane * epl;
          float score = 0.0f;
          for (int i = 0; i < epl; i += 4) {
            const float q0 = scale * q[h * D + ls + i];
            const float q1 = scale * q[h * D + ls + i + 1] / 16.0f;
            const float q2 = scale * q[h * D + ls + i + 2] / 256.0f;
            const float q3 = scale * q[h * D + ls + i + 3] / 4096.0f;
            const int gi = (ls + i) / 64;
            const float s = ksb[ki * ksd + gi], b = kbb[ki * ksd + gi];
            const uint16_t w = kw16[(int64_t)ki * (kpd * 2) + (ls + i) / 4];
            const float accum = q0 * (float)(w & 0x000Fu) + q1 * (float)(w & 0x00F0u) +
                                q2 * (float)(w & 0x0F00u) + q3 * (float)(w & 0xF000u);
            const float qsum = q0 + q1 * 16.0f + q2 * 256.0f + q3 * 4096.0f;
            score += s * accum + b * qsum;
          }
          lane_scores[lane] = score;
        }
        float score = 0.0f; /* simd_sum */
        for (int lane = 0; lane < 32; ++lane) score += lane_scores[lane];
        const float new_max = max_score > score ? max_score : score;
        const float factor = expf(max_score - new_max);
        const float exp_score = expf(score - new_max);
        max_score = new_max;
        sum_exp = sum_exp * factor + exp_score;
        for (int d = 0; d < D; d += 4) {
          const int gi = d / 64;
          const float s = vsb[ki * ksd + gi], b = vbb[ki * ksd + gi];
          const uint16_t w = vw16[(int64_t)ki * (kpd * 2) + d / 4];
          for (int j = 0; j < 4; ++j) {
            const float vj = s * (float)((w >> (4 * j)) & 0xFu) + b;
            osg[d + j] = osg[d + j] * factor + exp_score * vj;
          }
        }
      }
      mxs[sg] = max_score;
      sms[sg] = sum_exp;
    }
    float new_max = -1e30f;
    for (int sg = 0; sg < BN; ++sg) new_max = mxs[sg] > new_max ? mxs[sg] : new_max;
    float global_sum = 0.0f;
    for (int sg = 0; sg < BN; ++sg) global_sum += sms[sg] * expf(mxs[sg] - new_max);
    for (int d = 0; d < D; ++d) {
      float acc = 0.0f;
      for (int sg = 0; sg < BN; ++sg) acc += o[(int64_t)sg * D + d] * expf(mxs[sg] - new_max);
      out[h * D + d] = global_sum == 0.0f ? 0.0f : acc / global_sum;
    }
    free(mxs);
    free(sms);
    free(o);
  }
}

/* ---- log-sum-exp merge of split partials ---------------------------------
 * Partials p = 0..P-1, each with per-head (m, l, o[D]): m = max score
 * (natural-log units), l = sum exp(s - m), o = sum exp(s - m) v (unnormalised).
 * Merged: M = max m_p; L = sum e^(m_p - M) l_p; out = sum e^(m_p - M) o_p / L,
 * L == 0 -> 0 (lib/turboquant.metal:838-888 is the in-threadgroup version).
 * Layout of one partial block: o (H, D) floats, then ml (H, 2) floats.
 */
void tqo_lse_merge(const float* parts, int P, int H, int D, float* out) {
  const int64_t blk = (int64_t)H * (D + 2);
  for (int h = 0; h < H; ++h) {
    double M = -INFINITY;
    for (int p = 0; p < P; ++p) {
      const double m = parts[p * blk + (int64_t)H * D + 2 * h];
      M = m > M ? m : M;
    }
    double L = 0.0;
    double* acc = (double*)calloc(D, sizeof(double));
    for (int p = 0; p < P; ++p) {
      const double m = parts[p * blk + (int64_t)H * D + 2 * h];
      const double l = parts[p * blk + (int64_t)H * D + 2 * h + 1];
      if (m == -INFINITY) continue; /* an empty state (its o is never read) */
      const double e = exp(m - M);  /* a NaN state makes L and the head NaN */
      L += e * l;
      for (int d = 0; d < D; ++d) acc[d] += e * parts[p * blk + (int64_t)h * D + d];
    }
    for (int d = 0; d < D; ++d) out[h * D + d] = L == 0.0 ? 0.0f : (float)(acc[d] / L);
    free(acc);
  }
}

int tqo_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

void tqo_set_num_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}
