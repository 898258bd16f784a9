// sfk_sample.cuh -- device token sampling (sfk_sample.cu).
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

namespace sfk {

struct SampleArgs {
  float temperature;  // > 0 (greedy decoding does not launch the sampler)
  float top_p;        // >= 1: no nucleus filter
  int top_k;          // <= 0: no top-k filter
  uint64_t seed;
};

// Sample one token from logits [V] (device): writes the token to *tok_out and
// the greedy-loop key form of it (the next step's input) to *key_out.
// scratch: V floats.  One CTA.
cudaError_t launch_sample(const float* logits, int V, const SampleArgs& a, int step, float* scratch,
                          unsigned long long* key_out, int* tok_out, cudaStream_t st);

}  // namespace sfk
