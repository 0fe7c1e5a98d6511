// Stand-in for the reference's include/c4tts/t2s.h, used only to compile the
// reference's own src/t2s/sampling.cpp (unmodified) into the CPU checker
// without MLX. It declares nothing but the five sampling processors, with the
// exact signatures of include/c4tts/t2s.h:82-89 (the interface the compiled
// definitions must match).
#ifndef C4S_ORACLE_STUB_T2S_H_
#define C4S_ORACLE_STUB_T2S_H_

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

#endif  // C4S_ORACLE_STUB_T2S_H_
