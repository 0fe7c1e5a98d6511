// c4s_t2s_sampling.h -- drop-in C++ replacement for the reference's sampling
// processors, with the exact signatures of include/c4tts/t2s.h:82-89 of
// raoqu/mlx-confucius4-tts:
//
//   namespace c4::t2s::sampling {
//     void temperature(std::vector<float>&, float);
//     void repetition_penalty(std::vector<float>&, const std::vector<int>&, float);
//     void top_k(std::vector<float>&, int);
//     void top_p(std::vector<float>&, float, int min_tokens_to_keep = 1);
//     int  argmax(const std::vector<float>&);
//   }
//
// Each call uploads the host vector to the current CUDA device, runs the
// sm_100a kernel through the C ABI (c4s_process / c4s_argmax) and copies the
// result back in place, so the reference's call sites
// (text2semantic.cpp:142-149, :307-314) and its tests/test_sampling.cpp build
// against it unchanged. Results are bit-identical to the reference's host code
// (see c4s_sampling.h for the one tie-order note on top_p).
//
// Unlike the reference these functions can fail (no device, CUDA error); they
// then throw std::runtime_error instead of returning silently. Each host thread
// uses its own device context and stream.
//
// For the device-resident decode loop use the batched C ABI in c4s_sampling.h.
#ifndef C4S_T2S_SAMPLING_H_
#define C4S_T2S_SAMPLING_H_

#include <vector>

namespace c4 {
namespace t2s {
namespace sampling {
void temperature(std::vector<float>& logits, float temp);
void repetition_penalty(std::vector<float>& logits,
                        const std::vector<int>& prev_tokens, float penalty);
void top_k(std::vector<float>& logits, int k);
void top_p(std::vector<float>& logits, float p, int min_tokens_to_keep = 1);
int argmax(const std::vector<float>& logits);
}  // namespace sampling
}  // namespace t2s
}  // namespace c4

#endif  // C4S_T2S_SAMPLING_H_
