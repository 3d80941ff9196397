// The engine's kv_cache.safetensors through the C++ API: loads the file named
// by argv[1] (layer 0 a global cache, layer 3 a sliding layer with window
// 950), checks a decode over each loaded cache against one over a copy made
// on the host, writes the caches back to argv[2] and reloads that file,
// which must hold the same bytes. Prints PASS at the end.
#include <cstdio>
#include <cstring>
#include <map>
#include <vector>

#include "turboquant.hpp"

using turboquant::array;
using turboquant::Dtype;

namespace {

bool same(const array& a, const array& b, int rows_a, int rows_b) {
  // (1, Hkv, cap, w): compare the first min(rows) rows of every head
  const int hkv = a.shape(1), w = a.shape(3), ca = a.shape(2), cb = b.shape(2);
  const int n = rows_a < rows_b ? rows_a : rows_b;
  const size_t es = turboquant::itemsize(a.dtype());
  std::vector<unsigned char> ha(a.nbytes()), hb(b.nbytes());
  a.to_host(ha.data());
  b.to_host(hb.data());
  for (int h = 0; h < hkv; ++h)
    if (std::memcmp(ha.data() + (size_t)h * ca * w * es, hb.data() + (size_t)h * cb * w * es,
                    (size_t)n * w * es) != 0)
      return false;
  return a.dtype() == b.dtype();
}

bool same_cache(const turboquant::KVCache& a, const turboquant::KVCache& b) {
  return a.length() == b.length() && same(a.k_quant, b.k_quant, a.length(), b.length()) &&
         same(a.k_scales, b.k_scales, a.length(), b.length()) &&
         same(a.k_biases, b.k_biases, a.length(), b.length()) &&
         same(a.v_quant, b.v_quant, a.length(), b.length()) &&
         same(a.v_scales, b.v_scales, a.length(), b.length()) &&
         same(a.v_biases, b.v_biases, a.length(), b.length());
}

}  // namespace

int main(int argc, char** argv) {
  if (argc != 3) {
    printf("usage: test_kvstore <engine file> <output file>\n");
    return 2;
  }
  bool ok = true;
  auto L = turboquant::load_kv_cache(argv[1], 0, {{3, 950}});
  printf("cache_offset %d, global layers %zu, sliding layers %zu\n", L.cache_offset,
         L.caches.size(), L.rings.size());
  if (!L.caches.count(0) || !L.rings.count(3)) {
    printf("FAIL: expected layers 0 (global) and 3 (sliding)\n");
    return 1;
  }
  auto& g = *L.caches[0];
  auto& r = *L.rings[3];
  printf("layer 0: %d tokens (capacity %d), scales %s; layer 3: %d of window %d (capacity %d)\n",
         g.length(), g.capacity(), g.k_scales.dtype() == Dtype::float16 ? "f16" : "f32",
         r.n_valid(), r.window(), r.cache.capacity());
  ok &= r.cache.capacity() % 4 == 0 && r.cache.capacity() >= 950;

  // a decode over each loaded cache runs (16 KV heads, GQA 2)
  const int hkv = g.k_quant.shape(1), D = g.k_quant.shape(3) * 8;
  std::vector<float> qh(static_cast<size_t>(2 * hkv) * D);
  for (size_t i = 0; i < qh.size(); ++i) qh[i] = 0.01f * static_cast<float>((i * 37) % 101) - 0.5f;
  auto q = array::from_host(qh.data(), {2 * hkv, D}, Dtype::float32);
  auto o1 = g.sdpa(q, 2).to_vector<float>();
  auto o2 = r.decode(q, 2).to_vector<float>();
  for (float v : o1) ok &= v == v;
  for (float v : o2) ok &= v == v;

  turboquant::save_kv_cache(argv[2], L.cache_offset, {{0, &g}}, {{3, &r}});
  auto L2 = turboquant::load_kv_cache(argv[2], 0, {{3, 950}});
  ok &= L2.cache_offset == L.cache_offset;
  ok &= same_cache(*L2.caches[0], g);
  ok &= same_cache(L2.rings[3]->cache, r.cache);
  auto o3 = L2.caches[0]->sdpa(q, 2).to_vector<float>();
  ok &= std::memcmp(o1.data(), o3.data(), o1.size() * 4) == 0;
  printf("round trip through %s: %s\n", argv[2], ok ? "same bytes, same decode" : "MISMATCH");
  printf(ok ? "PASS\n" : "FAIL\n");
  return ok ? 0 : 1;
}
