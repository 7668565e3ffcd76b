// On-device sampler over the step's logits (see sampler.cu).
#pragma once

#include "common.cuh"

namespace yb {

// Written by the sampler kernel into host-mapped memory.
struct SampleResult {
  int token;        // argmax / sampled id
  float prob;       // probability of the target (op 2)
  unsigned epoch;   // step epoch the result belongs to
  int pad;
};

// Sampler op and parameters when they are not read from the step state.
struct SampleParams {
  int op;  // 0 argmax, 1 temperature sample, 2 probability of target
  int target;
  float temperature;
  float coin;
  unsigned epoch;
};

constexpr int kSampleThreads = 1024;

// One CTA: reads the vocab_size logits; the op and its parameters come from the step state when
// `step` is non-null (CUDA-graph steps), else from `direct`.
__global__ void sample_kernel(const float* logits, int vocab_size, const StepState* step, SampleParams direct,
                              SampleResult* out);

}  // namespace yb
