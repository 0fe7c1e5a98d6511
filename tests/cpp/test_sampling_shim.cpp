// test_sampling_shim -- the reference's tests/test_sampling.cpp check, run
// against the B200 drop-in (include/c4s_t2s_sampling.h) instead of the
// reference's host code: the same golden files (tools/dump_golden.py
// sampling), the same processor calls and parameters (test_sampling.cpp:48-51)
// and the same pass criterion (-inf masks equal and max_err < 1e-5,
// test_sampling.cpp:24-38), plus bit equality.
//
// usage: test_sampling_shim <golden dir containing logits.npy ids.npy ...>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <string>
#include <vector>

#include "c4s_t2s_sampling.h"

namespace {

// Minimal .npy reader for little-endian float32 / int64 C-order arrays.
bool load_npy(const std::string& path, std::vector<float>* f32, std::vector<int64_t>* i64) {
  std::ifstream in(path, std::ios::binary);
  if (!in) return false;
  char magic[6];
  in.read(magic, 6);
  if (std::memcmp(magic, "\x93NUMPY", 6) != 0) return false;
  unsigned char ver[2];
  in.read(reinterpret_cast<char*>(ver), 2);
  uint32_t hlen = 0;
  if (ver[0] == 1) {
    uint16_t h16;
    in.read(reinterpret_cast<char*>(&h16), 2);
    hlen = h16;
  } else {
    in.read(reinterpret_cast<char*>(&hlen), 4);
  }
  std::string header(hlen, ' ');
  in.read(&header[0], hlen);
  size_t n = 1;
  const size_t sp = header.find("'shape': (");
  if (sp == std::string::npos) return false;
  for (size_t p = sp + 10; header[p] != ')';) {
    if (header[p] >= '0' && header[p] <= '9') {
      size_t q = p;
      while (header[q] >= '0' && header[q] <= '9') ++q;
      n *= std::stoul(header.substr(p, q - p));
      p = q;
    } else {
      ++p;
    }
  }
  if (header.find("'<f4'") != std::string::npos && f32) {
    f32->resize(n);
    in.read(reinterpret_cast<char*>(f32->data()), n * 4);
    return bool(in);
  }
  if (header.find("'<i8'") != std::string::npos && i64) {
    i64->resize(n);
    in.read(reinterpret_cast<char*>(i64->data()), n * 8);
    return bool(in);
  }
  return false;
}

int failures = 0;

void check(const char* name, const std::vector<float>& got, const std::vector<float>& ref) {
  double max_err = 0;
  bool ok = got.size() == ref.size();
  bool bit_equal = ok;
  for (size_t i = 0; ok && i < got.size(); ++i) {
    const bool gi = std::isinf(got[i]) && got[i] < 0;
    const bool ri = std::isinf(ref[i]) && ref[i] < 0;
    if (gi != ri) { ok = false; break; }
    if (!gi) max_err = std::max(max_err, (double)std::abs(got[i] - ref[i]));
    if (std::memcmp(&got[i], &ref[i], 4) != 0) bit_equal = false;
  }
  const bool pass = ok && max_err < 1e-5 && bit_equal;
  std::printf("  [%s] max_err=%.3e bit_equal=%d %s\n", name, max_err, (int)bit_equal, pass ? "" : "<-- FAIL");
  if (!pass) ++failures;
}

}  // namespace

int main(int argc, char** argv) {
  if (argc < 2) { std::fprintf(stderr, "usage: %s <golden dir>\n", argv[0]); return 2; }
  const std::string G = std::string(argv[1]) + "/";
  std::printf("test_sampling_shim:\n");
  std::vector<float> base, temp, rep, topk, topp;
  std::vector<int64_t> ids64;
  if (!load_npy(G + "logits.npy", &base, nullptr) || !load_npy(G + "ids.npy", nullptr, &ids64) ||
      !load_npy(G + "temp.npy", &temp, nullptr) || !load_npy(G + "rep.npy", &rep, nullptr) ||
      !load_npy(G + "topk.npy", &topk, nullptr) || !load_npy(G + "topp.npy", &topp, nullptr)) {
    std::fprintf(stderr, "cannot read goldens from %s\n", G.c_str());
    return 2;
  }
  std::vector<int> ids(ids64.begin(), ids64.end());
  namespace sp = c4::t2s::sampling;
  try {
    { auto v = base; sp::temperature(v, 0.8f); check("temperature", v, temp); }
    { auto v = base; sp::repetition_penalty(v, ids, 1.3f); check("repetition_penalty", v, rep); }
    { auto v = base; sp::top_k(v, 10); check("top_k", v, topk); }
    { auto v = base; sp::top_p(v, 0.9f); check("top_p", v, topp); }
    {
      int am = sp::argmax(base);
      int want = 0;
      for (size_t i = 1; i < base.size(); ++i) if (base[want] < base[i]) want = (int)i;
      std::printf("  [argmax] %d vs %d %s\n", am, want, am == want ? "" : "<-- FAIL");
      if (am != want) ++failures;
    }
  } catch (const std::exception& e) {
    std::printf("  exception: %s <-- FAIL\n", e.what());
    ++failures;
  }
  std::printf("test_sampling_shim: %s\n", failures == 0 ? "ALL PASSED" : "FAILED");
  return failures == 0 ? 0 : 1;
}
