/*
 * CPU oracle for the PolarQuant + QJL compressed-key path.
 *
 * TEST INFRASTRUCTURE ONLY: the checker the CUDA kernels are compared against
 * (tests/ and bench.py). Nothing in gemma4metal_b200/ links or calls it.
 *
 * PARITY UNPINNED against the reference's own outputs: the reference's
 * PolarQuant kernels are Metal (lib/turboquant.metal) and cannot run here, it
 * ships no golden vectors, and it has no QJL code at all. This restates the
 * reference's formulas (file:line within svv232/gemma4metal):
 *   encode, per pair (a, b) of a level: angle = atan2(b, a), level 1 wrapped
 *   to [0, 2pi) by +2pi; index = first codebook entry with the smallest
 *   |angle - cb[c]| (linear scan, strict <); parent radius = sqrt(a*a + b*b);
 *   the last radius is stored as fp16                lib/turboquant.metal:30-97
 *   decode: children = (r cos(cb[idx]), r sin(cb[idx])) top-down
 *                                                    lib/turboquant.metal:113-163
 *   cos/sin of codebook entries from tables          lib/turboquant.metal:655-704
 *   score = scale * <P q, decode(key)>               lib/turboquant.metal:424-499
 *   compressed attention: softmax(score) . V         lib/turboquant.metal:166-224
 * generalised from 16-value blocks (4 levels) to blocks of 2^L values (L
 * levels; 128 values = 7 levels for the task's config 3), and QJL as
 * published (Zandieh et al., "QJL: 1-Bit Quantized JL Transform for KV Cache
 * Quantization", arXiv 2406.03482): residual r = y - decode(key), stored as
 * sign bits of S r (S: m x D Gaussian) and |r|; the inner-product estimate is
 * <q, r> ~= sqrt(pi/2) / m * |r| * <S q, sign(S r)>.
 *
 * Determinism shared with the CUDA kernels (so angle indices, radii and sign
 * bits match bit for bit): tqo_atan2 is this file's own polynomial atan2 (an
 * odd degree-17 polynomial in t = min/max fitted to atan on [0, 1] by
 * iteratively reweighted least squares on Chebyshev nodes; max error 9.6e-8
 * rad), every multiply-add that feeds an index or a sign is an explicit fmaf in
 * a fixed order, and cos/sin tables are cos/sin of the fp32 codebook entries
 * evaluated in double and rounded to fp32.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

uint16_t tqo_f32_to_f16(float x);
float tqo_f16_to_f32(uint16_t u);
float tqo_bf16_to_f32(uint16_t b);

#define TQO_MAX_LEVELS 7
#define TQO_CB 16

static const float kAtanC[9] = {0.9999998807907104f,   -0.33332598209381104f, 0.19985906779766083f,
                                -0.14161230623722076f, 0.10498947650194168f,  -0.07234859466552734f,
                                0.03978123515844345f,  -0.014401360414922237f, 0.0024567244108766317f};
static const float kHalfPi = 1.5707963705062866f;
static const float kPi = 3.1415927410125732f;
static const float kTwoPi = 6.2831854820251465f;

float tqo_atan2(float y, float x) {
  const float ax = fabsf(x), ay = fabsf(y);
  const float mx = ax > ay ? ax : ay, mn = ax > ay ? ay : ax;
  if (mx == 0.0f) return 0.0f;
  const float t = mn / mx;
  const float s = t * t;
  float p = kAtanC[8];
  for (int k = 7; k >= 0; --k) p = fmaf(p, s, kAtanC[k]);
  float a = p * t;
  if (ay > ax) a = kHalfPi - a;
  if (x < 0.0f) a = kPi - a;
  if (y < 0.0f) a = -a;
  return a;
}

static int levels_of(int block) {
  int l = 0;
  while ((1 << l) < block) ++l;
  return l;
}

/* angle offset of level L (1-based) inside a block, level-major */
static int level_off(int block, int L) {
  int off = 0;
  for (int l = 1; l < L; ++l) off += block >> l;
  return off;
}

static void cs_tables(const float* codebooks, int levels, float* cs /* levels*16*2 */) {
  for (int l = 0; l < levels; ++l)
    for (int c = 0; c < TQO_CB; ++c) {
      const double th = (double)codebooks[l * TQO_CB + c];
      cs[(l * TQO_CB + c) * 2] = (float)cos(th);
      cs[(l * TQO_CB + c) * 2 + 1] = (float)sin(th);
    }
}

/* y: rows x D (f32); angles: rows x nb x (block-1) uint8 or NULL; packed:
 * rows x nb x block/2 bytes (4-bit, low nibble first) or NULL; radii fp16. */
void tqo_polar_encode(const float* y, int64_t rows, int D, int block, const float* codebooks,
                      const int* cb_sizes, uint8_t* angles, uint8_t* packed, uint16_t* radii) {
  const int levels = levels_of(block), nb = D / block;
#pragma omp parallel for schedule(static)
  for (int64_t bi = 0; bi < rows * nb; ++bi) {
    float r[256];
    uint8_t idx[256];
    memcpy(r, y + bi * block, sizeof(float) * block);
    for (int L = 1; L <= levels; ++L) {
      const int cnt = block >> L, off = level_off(block, L);
      const float* cb = codebooks + (L - 1) * TQO_CB;
      for (int j = 0; j < cnt; ++j) {
        const float a = r[2 * j], b = r[2 * j + 1];
        float ang = tqo_atan2(b, a);
        if (L == 1 && ang < 0.0f) ang += kTwoPi;
        float best = 1e10f;
        int id = 0;
        for (int c = 0; c < cb_sizes[L - 1]; ++c) {
          const float d = fabsf(ang - cb[c]);
          if (d < best) {
            best = d;
            id = c;
          }
        }
        idx[off + j] = (uint8_t)id;
        r[j] = sqrtf(fmaf(a, a, b * b));
      }
    }
    radii[bi] = tqo_f32_to_f16(r[0]);
    if (angles) memcpy(angles + bi * (block - 1), idx, block - 1);
    if (packed) {
      uint8_t* pk = packed + bi * (block / 2);
      for (int i = 0; i < block / 2; ++i) {
        const int lo = idx[2 * i];
        const int hi = (2 * i + 1 < block - 1) ? idx[2 * i + 1] : 0;
        pk[i] = (uint8_t)((lo & 15) | ((hi & 15) << 4));
      }
    }
  }
}

static void decode_block(const uint8_t* idx, float radius, int block, const float* cs, float* out) {
  const int levels = levels_of(block);
  out[0] = radius;
  for (int L = levels; L >= 1; --L) {
    const int cnt = block >> L, off = level_off(block, L);
    for (int n = cnt - 1; n >= 0; --n) {
      const float v = out[n];
      const float* e = cs + ((L - 1) * TQO_CB + idx[off + n]) * 2;
      out[2 * n] = v * e[0];
      out[2 * n + 1] = v * e[1];
    }
  }
}

static void unpack_block(const uint8_t* pk, int block, uint8_t* idx) {
  for (int i = 0; i < block - 1; ++i) idx[i] = (pk[i / 2] >> (4 * (i & 1))) & 15;
}

/* exactly one of angles / packed is non-NULL */
void tqo_polar_decode(const uint8_t* angles, const uint8_t* packed, const uint16_t* radii,
                      int64_t rows, int D, int block, const float* codebooks, float* y) {
  const int levels = levels_of(block), nb = D / block;
  float cs[TQO_MAX_LEVELS * TQO_CB * 2];
  cs_tables(codebooks, levels, cs);
#pragma omp parallel for schedule(static)
  for (int64_t bi = 0; bi < rows * nb; ++bi) {
    uint8_t idx[256];
    if (angles) memcpy(idx, angles + bi * (block - 1), block - 1);
    else unpack_block(packed + bi * (block / 2), block, idx);
    decode_block(idx, tqo_f16_to_f32(radii[bi]), block, cs, y + bi * block);
  }
}

/* r = y - yhat; signs: rows x m/32 words, bit i = (S r)_i >= 0; rnorm fp16 = |r|.
 * (S r)_i and |r|^2 are sequential fmaf sums over j = 0..D-1 from 0. */
void tqo_qjl_encode(const float* y, const float* yhat, int64_t rows, int D, const float* S, int m,
                    uint32_t* signs, uint16_t* rnorm) {
#pragma omp parallel for schedule(static)
  for (int64_t n = 0; n < rows; ++n) {
    float r[1024];
    float nn = 0.0f;
    for (int j = 0; j < D; ++j) {
      r[j] = y[n * D + j] - yhat[n * D + j];
      nn = fmaf(r[j], r[j], nn);
    }
    rnorm[n] = tqo_f32_to_f16(sqrtf(nn));
    uint32_t* sg = signs + n * (m / 32);
    for (int w = 0; w < m / 32; ++w) sg[w] = 0;
    for (int i = 0; i < m; ++i) {
      float acc = 0.0f;
      for (int j = 0; j < D; ++j) acc = fmaf(S[(int64_t)i * D + j], r[j], acc);
      if (acc >= 0.0f) sg[i / 32] |= 1u << (i % 32);
    }
  }
}

static float load_q(const void* q, int64_t i, int dtype) {
  if (dtype == 1) return tqo_f16_to_f32(((const uint16_t*)q)[i]);
  if (dtype == 2) return tqo_bf16_to_f32(((const uint16_t*)q)[i]);
  return ((const float*)q)[i];
}

/* score[h][n] = scale * (<q_h, decode(key n of kv h/G)> + qjl term), fp64 sums.
 * q: H x D (already preconditioned); keys: Hkv x N rows of D; signs/rnorm may
 * be NULL (no QJL term). */
static void scores_one_head(const void* q, int q_dtype, int h, int G, int D, int N, int block,
                            const uint8_t* packed, const uint16_t* radii, const float* cs,
                            const uint32_t* signs, const uint16_t* rnorm, const float* S, int m,
                            float scale, double* out) {
  const int kv = h / G, nb = D / block;
  double qd[1024], sq[4096];
  for (int d = 0; d < D; ++d) qd[d] = load_q(q, (int64_t)h * D + d, q_dtype);
  if (signs)
    for (int i = 0; i < m; ++i) {
      double a = 0;
      for (int j = 0; j < D; ++j) a += (double)S[(int64_t)i * D + j] * qd[j];
      sq[i] = a;
    }
  for (int n = 0; n < N; ++n) {
    const int64_t row = (int64_t)kv * N + n;
    double acc = 0;
    for (int b = 0; b < nb; ++b) {
      uint8_t idx[256];
      float k[256];
      unpack_block(packed + (row * nb + b) * (block / 2), block, idx);
      decode_block(idx, tqo_f16_to_f32(radii[row * nb + b]), block, cs, k);
      for (int j = 0; j < block; ++j) acc += qd[b * block + j] * k[j];
    }
    if (signs) {
      double e = 0;
      const uint32_t* sg = signs + row * (m / 32);
      for (int i = 0; i < m; ++i) e += ((sg[i / 32] >> (i % 32)) & 1u) ? sq[i] : -sq[i];
      acc += sqrt(M_PI / 2.0) / m * tqo_f16_to_f32(rnorm[row]) * e;
    }
    out[n] = acc * scale;
  }
}

void tqo_compressed_score(const void* q, int q_dtype, int H, int Hkv, int D, int N, int block,
                          const uint8_t* packed, const uint16_t* radii, const float* codebooks,
                          const uint32_t* signs, const uint16_t* rnorm, const float* S, int m,
                          float scale, float* scores) {
  const int levels = levels_of(block), G = H / Hkv;
  float cs[TQO_MAX_LEVELS * TQO_CB * 2];
  cs_tables(codebooks, levels, cs);
#pragma omp parallel for schedule(dynamic)
  for (int h = 0; h < H; ++h) {
    double* s = (double*)malloc(sizeof(double) * N);
    scores_one_head(q, q_dtype, h, G, D, N, block, packed, radii, cs, signs, rnorm, S, m, scale, s);
    for (int n = 0; n < N; ++n) scores[(int64_t)h * N + n] = (float)s[n];
    free(s);
  }
}

/* out[h] = softmax(score[h]) . V, V = int4 affine group-64 (codes (Hkv, N, D/8),
 * scales/biases (Hkv, N, D/64) fp16 or fp32 (sb_f32)); fp64 throughout. An
 * empty context writes 0. */
void tqo_compressed_sdpa(const void* q, int q_dtype, int H, int Hkv, int D, int N, int block,
                         const uint8_t* packed, const uint16_t* radii, const float* codebooks,
                         const uint32_t* signs, const uint16_t* rnorm, const float* S, int m,
                         float scale, const uint32_t* vq, const void* vs, const void* vb, int sb_f32,
                         float* out) {
  const int levels = levels_of(block), G = H / Hkv;
  float cs[TQO_MAX_LEVELS * TQO_CB * 2];
  cs_tables(codebooks, levels, cs);
#pragma omp parallel for schedule(dynamic)
  for (int h = 0; h < H; ++h) {
    const int kv = h / G;
    double* s = (double*)malloc(sizeof(double) * (N > 0 ? N : 1));
    scores_one_head(q, q_dtype, h, G, D, N, block, packed, radii, cs, signs, rnorm, S, m, scale, s);
    double mx = -INFINITY, l = 0;
    for (int n = 0; n < N; ++n) mx = s[n] > mx ? s[n] : mx;
    double o[1024];
    for (int d = 0; d < D; ++d) o[d] = 0;
    for (int n = 0; n < N; ++n) {
      const double p = exp(s[n] - mx);
      l += p;
      const int64_t row = (int64_t)kv * N + n;
      for (int d = 0; d < D; ++d) {
        const uint32_t w = vq[row * (D / 8) + d / 8];
        const int c = (w >> (4 * (d % 8))) & 15;
        const int64_t gi = row * (D / 64) + d / 64;
        const double sc = sb_f32 ? ((const float*)vs)[gi] : tqo_f16_to_f32(((const uint16_t*)vs)[gi]);
        const double bi = sb_f32 ? ((const float*)vb)[gi] : tqo_f16_to_f32(((const uint16_t*)vb)[gi]);
        o[d] += p * (sc * c + bi);
      }
    }
    for (int d = 0; d < D; ++d) out[(int64_t)h * D + d] = l == 0 ? 0.0f : (float)(o[d] / l);
    free(s);
  }
}
