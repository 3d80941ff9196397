// C++ checks of the reference's PolarQuant entry points (lib/turboquant.h:52-165)
// on the turboquant.hpp API: 16-value blocks with four level codebooks, the
// per-level index arrays, the 2-bit packed format and the compressed scores /
// attention, each compared with a host computation from the decoded keys.
// Exit code 0 = pass.
#include <cmath>
#include <cstdio>
#include <random>
#include <vector>

#include "turboquant.hpp"

using turboquant::array;
using turboquant::Dtype;

namespace {

array codebook(int n, double lo, double hi) {
  std::vector<float> c(n);
  for (int i = 0; i < n; ++i) c[i] = static_cast<float>(lo + (hi - lo) * (i + 0.5) / n);
  return array::from_host(c.data(), {n}, Dtype::float32);
}

bool report(const char* name, double err, double tol) {
  const bool ok = err <= tol;
  printf("%-40s err=%.3e tol=%.1e %s\n", name, err, tol, ok ? "PASS" : "FAIL");
  return ok;
}

}  // namespace

int main() {
  const int N = 96, D = 128, Nq = 4, Nk = N / Nq;
  std::mt19937 rng(7);
  std::normal_distribution<float> nd;
  std::vector<float> x(static_cast<size_t>(N) * D), I(static_cast<size_t>(D) * D, 0.0f);
  for (auto& v : x) v = nd(rng);
  for (int i = 0; i < D; ++i) I[static_cast<size_t>(i) * D + i] = 1.0f;
  auto X = array::from_host(x.data(), {N, D}, Dtype::float32);
  auto P = array::from_host(I.data(), {D, D}, Dtype::float32);
  const double kPi = 3.14159265358979323846;
  auto c1 = codebook(16, 0, 2 * kPi), c2 = codebook(4, 0, kPi / 2), c3 = codebook(4, 0, kPi / 2),
       c4 = codebook(4, 0, kPi / 2);
  bool ok = true;

  auto q = turboquant::polar_quantize(X, P, c1, c2, c3, c4, 16);
  const int nb = N * D / 16;
  ok &= q.size() == 5 && q[0].size() == static_cast<size_t>(nb) * 8 && q[1].size() == static_cast<size_t>(nb) * 4 &&
        q[2].size() == static_cast<size_t>(nb) * 2 && q[3].size() == static_cast<size_t>(nb) && q[4].size() == static_cast<size_t>(nb);
  auto y = turboquant::polar_dequantize(q[0], q[1], q[2], q[3], q[4], P, c1, c2, c3, c4, 16).to_vector<float>();
  auto yf = turboquant::polar_dequantize_fast(q[0], q[1], q[2], q[3], q[4], c1, c2, c3, c4, D, 16).to_vector<float>();
  double e_same = 0, num = 0, den = 0;
  for (size_t i = 0; i < y.size(); ++i) {
    e_same = std::max(e_same, static_cast<double>(std::fabs(y[i] - yf[i])));
    num += (y[i] - x[i]) * (y[i] - x[i]);
    den += x[i] * x[i];
  }
  ok &= report("dequantize == dequantize_fast (P = I)", e_same, 1e-5);
  ok &= report("round-trip relative error (coarse codes)", std::sqrt(num / den), 0.35);

  auto pk = turboquant::polar_quantize_packed(X, P, c1, c2, c3, c4, 16);
  auto yp = turboquant::polar_dequantize_packed(pk[0], pk[1], pk[2], pk[3], pk[4], c1, c2, c3, c4, D, 16).to_vector<float>();
  double e_pk = 0;
  for (size_t i = 0; i < y.size(); ++i) e_pk = std::max(e_pk, static_cast<double>(std::fabs(yp[i] - yf[i])));
  ok &= report("packed round trip == unpacked", e_pk, 0.0);
  // cos/sin tables of the same codebooks
  std::vector<array> cs;
  for (const array* c : {&c1, &c2, &c3, &c4}) {
    auto v = c->to_vector<float>();
    std::vector<float> t;
    for (float a : v) {
      t.push_back(static_cast<float>(std::cos(static_cast<double>(a))));
      t.push_back(static_cast<float>(std::sin(static_cast<double>(a))));
    }
    cs.push_back(array::from_host(t.data(), {static_cast<int>(v.size()), 2}, Dtype::float32));
  }
  auto ypf = turboquant::polar_dequantize_packed_fast(pk[0], pk[1], pk[2], pk[3], pk[4], cs[0], cs[1], cs[2], cs[3], D, 16).to_vector<float>();
  double e_fast = 0;
  for (size_t i = 0; i < y.size(); ++i) e_fast = std::max(e_fast, static_cast<double>(std::fabs(ypf[i] - yp[i])));
  ok &= report("packed_fast (cos/sin tables) == packed", e_fast, 1e-5);

  // compressed scores / attention: query i against keys [i*Nk, (i+1)*Nk)
  std::vector<float> qh(static_cast<size_t>(Nq) * D), vh(static_cast<size_t>(N) * D);
  for (auto& v : qh) v = nd(rng);
  for (auto& v : vh) v = nd(rng);
  auto Q = array::from_host(qh.data(), {Nq, D}, Dtype::float32);
  auto V = array::from_host(vh.data(), {N, D}, Dtype::float32);
  const float scale = 0.0884f;
  auto sc = turboquant::compressed_score(Q, q[0], q[1], q[2], q[3], q[4], c1, c2, c3, c4, Nk, 16, scale).to_vector<float>();
  auto at = turboquant::compressed_sdpa(Q, q[0], q[1], q[2], q[3], q[4], c1, c2, c3, c4, V, 16, scale).to_vector<float>();
  double e_sc = 0, e_at = 0;
  for (int h = 0; h < Nq; ++h) {
    std::vector<double> s(Nk);
    double m = -1e300, l = 0;
    for (int n = 0; n < Nk; ++n) {
      double a = 0;
      for (int d = 0; d < D; ++d) a += static_cast<double>(qh[h * D + d]) * yf[(static_cast<size_t>(h) * Nk + n) * D + d];
      s[n] = a * scale;
      e_sc = std::max(e_sc, std::fabs(s[n] - sc[static_cast<size_t>(h) * Nk + n]));
      m = std::max(m, s[n]);
    }
    std::vector<double> o(D, 0.0);
    for (int n = 0; n < Nk; ++n) {
      const double p = std::exp(s[n] - m);
      l += p;
      for (int d = 0; d < D; ++d) o[d] += p * vh[(static_cast<size_t>(h) * Nk + n) * D + d];
    }
    for (int d = 0; d < D; ++d) e_at = std::max(e_at, std::fabs(o[d] / l - at[static_cast<size_t>(h) * D + d]));
  }
  ok &= report("compressed_score vs decoded dot", e_sc, 2e-4);
  ok &= report("compressed_sdpa vs softmax . values", e_at, 2e-3);
  printf("\n%s\n", ok ? "PASS" : "FAIL");
  return ok ? 0 : 1;
}
