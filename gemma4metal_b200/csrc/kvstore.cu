// The engine's on-disk int4 KV cache for the C++ API: save_kv_cache /
// load_kv_cache over KVCache and RingKVCache, the file format of
// engine/gemma4_multilayer.cpp:113-144 (one safetensors file: cache_offset
// int32 [1] and l{L}.kq/ks/kb/vq/vs/vb per cached layer, codes uint32
// (1, Hkv, T, D/8), scales/biases (1, Hkv, T, D/64), T tokens oldest first).
//
// safetensors, written and read here without a dependency: an 8-byte
// little-endian header length, a JSON object {name: {"dtype", "shape",
// "data_offsets": [begin, end)}} (plus an optional "__metadata__" object)
// padded with spaces to a multiple of 8 bytes, then the tensors' bytes.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <fstream>
#include <map>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/turboquant.hpp"

namespace turboquant {
namespace {

[[noreturn]] void fail(const std::string& what) {
  throw std::runtime_error("turboquant::kv_cache file: " + what);
}

void cuda_ok(cudaError_t e, const char* where) {
  if (e != cudaSuccess) fail(std::string(where) + ": " + cudaGetErrorString(e));
}

// ---- a JSON reader for the safetensors header (objects, arrays, strings,
// integers; anything else is rejected) ------------------------------------------
struct Json {
  enum Kind { Null, Num, Str, Arr, Obj } kind = Null;
  long long num = 0;
  std::string str;
  std::vector<Json> arr;
  std::map<std::string, Json> obj;
};

class Parser {
 public:
  explicit Parser(const std::string& s) : s_(s) {}
  Json parse() {
    Json v = value();
    ws();
    if (i_ != s_.size()) fail("trailing bytes in the header");
    return v;
  }

 private:
  void ws() {
    while (i_ < s_.size() && (s_[i_] == ' ' || s_[i_] == '\n' || s_[i_] == '\t' || s_[i_] == '\r')) ++i_;
  }
  char peek() {
    ws();
    if (i_ >= s_.size()) fail("header ends early");
    return s_[i_];
  }
  void expect(char c) {
    if (peek() != c) fail(std::string("header: expected '") + c + "'");
    ++i_;
  }
  std::string string() {
    expect('"');
    std::string out;
    while (i_ < s_.size() && s_[i_] != '"') {
      if (s_[i_] == '\\') {
        if (++i_ >= s_.size()) break;
        const char e = s_[i_];
        out.push_back(e == 'n' ? '\n' : e == 't' ? '\t' : e);  // names here are plain ASCII
      } else {
        out.push_back(s_[i_]);
      }
      ++i_;
    }
    if (i_ >= s_.size()) fail("header: unterminated string");
    ++i_;
    return out;
  }
  Json value() {
    Json v;
    const char c = peek();
    if (c == '{') {
      ++i_;
      v.kind = Json::Obj;
      if (peek() == '}') {
        ++i_;
        return v;
      }
      while (true) {
        std::string k = string();
        expect(':');
        v.obj[k] = value();
        if (peek() == ',') {
          ++i_;
          continue;
        }
        expect('}');
        return v;
      }
    }
    if (c == '[') {
      ++i_;
      v.kind = Json::Arr;
      if (peek() == ']') {
        ++i_;
        return v;
      }
      while (true) {
        v.arr.push_back(value());
        if (peek() == ',') {
          ++i_;
          continue;
        }
        expect(']');
        return v;
      }
    }
    if (c == '"') {
      v.kind = Json::Str;
      v.str = string();
      return v;
    }
    if (c == '-' || (c >= '0' && c <= '9')) {
      v.kind = Json::Num;
      size_t used = 0;
      v.num = std::stoll(s_.substr(i_), &used);
      i_ += used;
      return v;
    }
    fail("header: unsupported JSON value");
  }
  const std::string& s_;
  size_t i_ = 0;
};

struct Tensor {
  std::string dtype;
  std::vector<long long> shape;
  size_t begin = 0, end = 0;
};

const char* st_name(Dtype d) {
  switch (d) {
    case Dtype::float32: return "F32";
    case Dtype::float16: return "F16";
    case Dtype::bfloat16: return "BF16";
    case Dtype::uint32: return "U32";
    case Dtype::int32: return "I32";
    case Dtype::uint8: return "U8";
  }
  return "U8";
}

// Rows [first, first + n) of every KV head of a (1, Hkv, cap, w) device array,
// appended to `out` in (Hkv, n, w) order.
void gather_rows(const array& a, int first, int n, std::vector<unsigned char>& out,
                 cudaStream_t s) {
  const int hkv = a.shape(1), cap = a.shape(2), w = a.shape(3);
  const size_t row = static_cast<size_t>(w) * itemsize(a.dtype());
  const size_t at = out.size();
  out.resize(at + static_cast<size_t>(hkv) * n * row);
  if (n == 0) return;
  cuda_ok(cudaMemcpy2DAsync(out.data() + at, n * row,
                            static_cast<const unsigned char*>(a.data()) + first * row, cap * row,
                            n * row, hkv, cudaMemcpyDeviceToHost, s),
          "save_kv_cache");
}

struct Blob {
  std::string dtype;
  std::vector<long long> shape;
  std::vector<unsigned char> bytes;
};

void write_file(const std::string& path, const std::map<std::string, Blob>& blobs) {
  std::string h = "{";
  size_t off = 0;
  bool first = true;
  for (const auto& [name, b] : blobs) {  // std::map: names sorted, as the Python writer does
    if (!first) h += ",";
    first = false;
    h += "\"" + name + "\":{\"dtype\":\"" + b.dtype + "\",\"shape\":[";
    for (size_t i = 0; i < b.shape.size(); ++i) h += (i ? "," : "") + std::to_string(b.shape[i]);
    h += "],\"data_offsets\":[" + std::to_string(off) + "," + std::to_string(off + b.bytes.size()) + "]}";
    off += b.bytes.size();
  }
  h += "}";
  while (h.size() % 8) h += ' ';
  std::ofstream f(path, std::ios::binary);
  if (!f) fail("cannot open " + path + " for writing");
  const uint64_t n = h.size();
  unsigned char len[8];
  for (int i = 0; i < 8; ++i) len[i] = static_cast<unsigned char>(n >> (8 * i));
  f.write(reinterpret_cast<const char*>(len), 8);
  f.write(h.data(), static_cast<std::streamsize>(h.size()));
  for (const auto& [name, b] : blobs)
    f.write(reinterpret_cast<const char*>(b.bytes.data()), static_cast<std::streamsize>(b.bytes.size()));
  if (!f) fail("write to " + path + " failed");
}

const char* kNames[6] = {"kq", "ks", "kb", "vq", "vs", "vb"};

void add_layer(std::map<std::string, Blob>& blobs, int layer, const KVCache& c,
               const std::vector<std::pair<int, int>>& ranges, cudaStream_t s) {
  if (c.k_quant.shape(0) != 1) fail("the engine's cache format has batch 1");
  const array* arrs[6] = {&c.k_quant, &c.k_scales, &c.k_biases, &c.v_quant, &c.v_scales, &c.v_biases};
  int T = 0;
  for (const auto& r : ranges) T += r.second;
  for (int i = 0; i < 6; ++i) {
    Blob b;
    b.dtype = st_name(arrs[i]->dtype());
    b.shape = {1, arrs[i]->shape(1), T, arrs[i]->shape(3)};
    std::vector<std::vector<unsigned char>> parts(ranges.size());
    for (size_t k = 0; k < ranges.size(); ++k) gather_rows(*arrs[i], ranges[k].first, ranges[k].second, parts[k], s);
    cuda_ok(cudaStreamSynchronize(s), "save_kv_cache");
    // (Hkv, n_k, w) pieces -> (Hkv, T, w): interleave per head
    const int hkv = arrs[i]->shape(1);
    const size_t row = static_cast<size_t>(arrs[i]->shape(3)) * itemsize(arrs[i]->dtype());
    b.bytes.resize(static_cast<size_t>(hkv) * T * row);
    size_t col = 0;
    for (size_t k = 0; k < ranges.size(); ++k) {
      const size_t n = ranges[k].second;
      for (int h = 0; h < hkv; ++h)
        if (n) std::memcpy(b.bytes.data() + (static_cast<size_t>(h) * T + col) * row,
                           parts[k].data() + static_cast<size_t>(h) * n * row, n * row);
      col += n;
    }
    blobs["l" + std::to_string(layer) + "." + kNames[i]] = std::move(b);
  }
}

}  // namespace

void save_kv_cache(const std::string& path, int cache_offset,
                   const std::map<int, const KVCache*>& caches,
                   const std::map<int, const RingKVCache*>& rings, cudaStream_t s) {
  std::map<std::string, Blob> blobs;
  Blob off;
  off.dtype = "I32";
  off.shape = {1};
  off.bytes.resize(4);
  std::memcpy(off.bytes.data(), &cache_offset, 4);
  blobs["cache_offset"] = std::move(off);
  for (const auto& [layer, c] : caches) {
    if (rings.count(layer)) fail("layer " + std::to_string(layer) + " given twice");
    add_layer(blobs, layer, *c, {{0, c->length()}}, s);
  }
  for (const auto& [layer, r] : rings) {
    // oldest first: slot total % window onwards, then the slots before it
    const int n = r->n_valid(), W = r->window();
    const int start = r->total() > W ? static_cast<int>(r->total() % W) : 0;
    const int first = std::min(n, W - start);
    add_layer(blobs, layer, r->cache, {{start, first}, {0, n - first}}, s);
  }
  write_file(path, blobs);
}

LoadedKVCache load_kv_cache(const std::string& path, int capacity, const std::map<int, int>& windows,
                            cudaStream_t s) {
  std::ifstream f(path, std::ios::binary);
  if (!f) fail("cannot open " + path);
  unsigned char len[8];
  if (!f.read(reinterpret_cast<char*>(len), 8)) fail(path + ": no header length");
  uint64_t n = 0;
  for (int i = 0; i < 8; ++i) n |= static_cast<uint64_t>(len[i]) << (8 * i);
  if (n > (64u << 20)) fail(path + ": header length " + std::to_string(n) + " is not plausible");
  std::string header(n, '\0');
  if (!f.read(&header[0], static_cast<std::streamsize>(n))) fail(path + ": header cut short");
  std::vector<unsigned char> data((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
  const Json root = Parser(header).parse();
  if (root.kind != Json::Obj) fail(path + ": header is not a JSON object");
  std::map<std::string, Tensor> ts;
  for (const auto& [name, e] : root.obj) {
    if (name == "__metadata__") continue;
    if (e.kind != Json::Obj || !e.obj.count("dtype") || !e.obj.count("shape") || !e.obj.count("data_offsets"))
      fail(path + ": tensor " + name + " lacks dtype/shape/data_offsets");
    Tensor t;
    t.dtype = e.obj.at("dtype").str;
    for (const auto& d : e.obj.at("shape").arr) t.shape.push_back(d.num);
    const auto& o = e.obj.at("data_offsets").arr;
    if (o.size() != 2 || o[0].num < 0 || o[1].num < o[0].num || static_cast<size_t>(o[1].num) > data.size())
      fail(path + ": tensor " + name + " has bad data_offsets");
    t.begin = static_cast<size_t>(o[0].num);
    t.end = static_cast<size_t>(o[1].num);
    ts[name] = t;
  }
  LoadedKVCache out;
  auto off = ts.find("cache_offset");
  if (off == ts.end() || off->second.end - off->second.begin < 4) fail(path + ": no cache_offset");
  std::memcpy(&out.cache_offset, data.data() + off->second.begin, 4);

  for (const auto& [name, t] : ts) {
    if (name.size() < 5 || name[0] != 'l' || name.compare(name.size() - 3, 3, ".kq") != 0) continue;
    const int layer = std::stoi(name.substr(1, name.size() - 4));
    const std::string p = "l" + std::to_string(layer) + ".";
    const Tensor* a[6];
    for (int i = 0; i < 6; ++i) {
      auto it = ts.find(p + kNames[i]);
      if (it == ts.end()) fail(path + ": layer " + std::to_string(layer) + " lacks " + kNames[i]);
      a[i] = &it->second;
      if (a[i]->shape.size() != 4 || a[i]->shape[0] != 1)
        fail(path + ": " + p + kNames[i] + " is not (1, Hkv, T, .)");
    }
    const int hkv = static_cast<int>(a[0]->shape[1]), T = static_cast<int>(a[0]->shape[2]);
    const int D = static_cast<int>(a[0]->shape[3]) * 8;
    const std::string sd = a[1]->dtype;
    if (a[0]->dtype != "U32" && a[0]->dtype != "I32") fail(p + "kq must be U32");
    if (sd != "F16" && sd != "F32" && sd != "BF16") fail(p + "ks must be F16, F32 or BF16");
    const Dtype sdt = sd == "F16" ? Dtype::float16 : Dtype::float32;  // bf16 widens to fp32
    KVCache* cache = nullptr;
    auto w = windows.find(layer);
    if (w != windows.end()) {
      if (T > w->second) fail(p + ": " + std::to_string(T) + " tokens do not fit the window");
      out.rings[layer] = std::make_unique<RingKVCache>(hkv, D, w->second, sdt, s);
      cache = &out.rings[layer]->cache;
    } else {
      const int cap = std::max({capacity, (T + 3) / 4 * 4, 4});
      out.caches[layer] = std::make_unique<KVCache>(1, hkv, D, cap, sdt, s);
      cache = out.caches[layer].get();
    }
    array* dst[6] = {&cache->k_quant, &cache->k_scales, &cache->k_biases,
                     &cache->v_quant, &cache->v_scales, &cache->v_biases};
    for (int i = 0; i < 6; ++i) {
      const int wdt = dst[i]->shape(3);
      if (a[i]->shape[1] != hkv || a[i]->shape[2] != T || a[i]->shape[3] != wdt ||
          (i % 3 && a[i]->dtype != sd))
        fail(p + kNames[i] + " does not match the layer's other arrays");
      const size_t src_es = (a[i]->dtype == "F32" || a[i]->dtype == "U32" || a[i]->dtype == "I32") ? 4 : 2;
      const size_t rows = static_cast<size_t>(hkv) * T;
      if (a[i]->end - a[i]->begin != rows * wdt * src_es) fail(p + kNames[i] + ": byte count does not match its shape");
      const unsigned char* src = data.data() + a[i]->begin;
      std::vector<unsigned char> widened;
      if (a[i]->dtype == "BF16") {  // exact: bf16 is the top half of an fp32
        widened.resize(rows * wdt * 4);
        for (size_t k = 0; k < rows * wdt; ++k) {
          uint32_t u = static_cast<uint32_t>(src[2 * k] | (src[2 * k + 1] << 8)) << 16;
          std::memcpy(widened.data() + 4 * k, &u, 4);
        }
        src = widened.data();
      }
      const size_t row = static_cast<size_t>(wdt) * itemsize(dst[i]->dtype());
      if (T > 0)
        cuda_ok(cudaMemcpy2DAsync(dst[i]->data(), static_cast<size_t>(dst[i]->shape(2)) * row, src,
                                  static_cast<size_t>(T) * row, static_cast<size_t>(T) * row, hkv,
                                  cudaMemcpyHostToDevice, s),
                "load_kv_cache");
      cuda_ok(cudaStreamSynchronize(s), "load_kv_cache");  // `widened` is released below
    }
    if (w != windows.end()) out.rings[layer]->set_total(T);
    else cache->set_length(T);
  }
  return out;
}

}  // namespace turboquant
