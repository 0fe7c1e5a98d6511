// c4s_shim.cpp -- c4::t2s::sampling (host std::vector in/out) on top of the
// C ABI. Mirrors include/c4tts/t2s.h:82-89 of the reference; each call is
// upload -> one kernel -> download on a per-thread stream.
#include "../../include/c4s_t2s_sampling.h"

#include <cuda_runtime.h>

#include <cstdint>
#include <stdexcept>
#include <string>

#include "../../include/c4s_sampling.h"

namespace {

struct ShimState {
  c4s_ctx* ctx = nullptr;
  int device = -1;
  int max_vocab = 0;
  cudaStream_t stream = nullptr;
  float* d_logits = nullptr;
  int32_t* d_hist = nullptr;
  size_t hist_cap = 0;
  int64_t* d_off = nullptr;
  c4s_row_params* d_params = nullptr;
  int32_t* d_id = nullptr;

  void release() {
    if (ctx) c4s_destroy(ctx);
    ctx = nullptr;
    if (stream) cudaStreamDestroy(stream);
    stream = nullptr;
    cudaFree(d_logits); d_logits = nullptr;
    cudaFree(d_hist); d_hist = nullptr; hist_cap = 0;
    cudaFree(d_off); d_off = nullptr;
    cudaFree(d_params); d_params = nullptr;
    cudaFree(d_id); d_id = nullptr;
    max_vocab = 0;
  }
  ~ShimState() { release(); }
};

thread_local ShimState g;

[[noreturn]] void fail(const std::string& what) {
  throw std::runtime_error("c4s sampling: " + what);
}

void cu(cudaError_t e, const char* what) {
  if (e != cudaSuccess) fail(std::string(what) + ": " + cudaGetErrorString(e));
}

void rc(int status, const char* what) {
  if (status != C4S_OK)
    fail(std::string(what) + ": " + c4s_status_string(status) + " (" + c4s_last_error(g.ctx) + ")");
}

// Context + buffers on the calling thread's current device, for rows up to V.
void ensure(int V, size_t H) {
  int dev = 0;
  cu(cudaGetDevice(&dev), "cudaGetDevice");
  if (g.ctx && (g.device != dev || g.max_vocab < V)) g.release();
  if (!g.ctx) {
    int mv = V < 8194 ? 8194 : V;
    rc(c4s_create_sized(&g.ctx, mv, 1, dev), "c4s_create_sized");   // one row per call
    g.device = dev;
    g.max_vocab = mv;
    cu(cudaStreamCreateWithFlags(&g.stream, cudaStreamNonBlocking), "cudaStreamCreate");
    cu(cudaMalloc(&g.d_logits, sizeof(float) * (size_t)mv), "cudaMalloc");
    cu(cudaMalloc(&g.d_off, sizeof(int64_t) * 2), "cudaMalloc");
    cu(cudaMalloc(&g.d_params, sizeof(c4s_row_params)), "cudaMalloc");
    cu(cudaMalloc(&g.d_id, sizeof(int32_t)), "cudaMalloc");
  }
  if (H > g.hist_cap) {
    cudaFree(g.d_hist);
    g.d_hist = nullptr;
    size_t cap = 1024;
    while (cap < H) cap <<= 1;
    cu(cudaMalloc(&g.d_hist, sizeof(int32_t) * cap), "cudaMalloc");
    g.hist_cap = cap;
  }
}

void process(std::vector<float>& logits, const std::vector<int>* hist, const c4s_row_params& P, int stages) {
  const int V = static_cast<int>(logits.size());
  if (V == 0) return;
  if (V > 32768) fail("vocabulary above the kernel's shared-memory limit (32768)");
  const size_t H = hist ? hist->size() : 0;
  ensure(V, H);
  cu(cudaMemcpyAsync(g.d_logits, logits.data(), sizeof(float) * V, cudaMemcpyHostToDevice, g.stream), "upload");
  cu(cudaMemcpyAsync(g.d_params, &P, sizeof(P), cudaMemcpyHostToDevice, g.stream), "upload");
  const int64_t off[2] = {0, static_cast<int64_t>(H)};
  if (hist) {
    cu(cudaMemcpyAsync(g.d_off, off, sizeof(off), cudaMemcpyHostToDevice, g.stream), "upload");
    if (H) cu(cudaMemcpyAsync(g.d_hist, hist->data(), sizeof(int32_t) * H, cudaMemcpyHostToDevice, g.stream), "upload");
  }
  rc(c4s_process(g.ctx, g.d_logits, 1, V, V, hist ? g.d_hist : nullptr, hist ? g.d_off : nullptr,
                 static_cast<int64_t>(H), g.d_params, 0, stages, g.stream),
     "c4s_process");
  cu(cudaMemcpyAsync(logits.data(), g.d_logits, sizeof(float) * V, cudaMemcpyDeviceToHost, g.stream), "download");
  cu(cudaStreamSynchronize(g.stream), "synchronize");
}

c4s_row_params defaults() {
  c4s_row_params P{};
  P.temperature = 1.0f;
  P.top_k = 0;
  P.top_p = 1.0f;
  P.repetition_penalty = 1.0f;
  P.greedy = 0;
  P.min_tokens_to_keep = 1;
  return P;
}

}  // namespace

namespace c4 {
namespace t2s {
namespace sampling {

// sampling.cpp:14-17
void temperature(std::vector<float>& logits, float temp) {
  if (temp == 1.0f || temp <= 0.0f) return;
  c4s_row_params P = defaults();
  P.temperature = temp;
  process(logits, nullptr, P, C4S_STAGE_TEMPERATURE);
}

// sampling.cpp:19-28 (static_assert: the reference's ids are int)
void repetition_penalty(std::vector<float>& logits, const std::vector<int>& prev_tokens, float penalty) {
  static_assert(sizeof(int) == sizeof(int32_t), "history ids are int32 on the device");
  if (penalty == 1.0f) return;
  c4s_row_params P = defaults();
  P.repetition_penalty = penalty;
  process(logits, &prev_tokens, P, C4S_STAGE_PENALTY);
}

// sampling.cpp:30-40
void top_k(std::vector<float>& logits, int k) {
  const int n = static_cast<int>(logits.size());
  if (k <= 0 || k >= n) return;
  c4s_row_params P = defaults();
  P.top_k = k;
  process(logits, nullptr, P, C4S_STAGE_TOP_K);
}

// sampling.cpp:42-71
void top_p(std::vector<float>& logits, float p, int min_tokens_to_keep) {
  c4s_row_params P = defaults();
  P.top_p = p;
  P.min_tokens_to_keep = min_tokens_to_keep;
  process(logits, nullptr, P, C4S_STAGE_TOP_P);
}

// sampling.cpp:73-76
int argmax(const std::vector<float>& logits) {
  const int V = static_cast<int>(logits.size());
  if (V == 0) return 0;
  if (V > 32768) fail("vocabulary above the kernel's shared-memory limit (32768)");
  ensure(V, 0);
  cu(cudaMemcpyAsync(g.d_logits, logits.data(), sizeof(float) * V, cudaMemcpyHostToDevice, g.stream), "upload");
  rc(c4s_argmax(g.ctx, g.d_logits, 1, V, V, g.d_id, g.stream), "c4s_argmax");
  int32_t id = 0;
  cu(cudaMemcpyAsync(&id, g.d_id, sizeof(id), cudaMemcpyDeviceToHost, g.stream), "download");
  cu(cudaStreamSynchronize(g.stream), "synchronize");
  return id;
}

}  // namespace sampling
}  // namespace t2s
}  // namespace c4
