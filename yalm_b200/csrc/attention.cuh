// Split-K GQA decode attention (see attention.cu).
#pragma once

#include <cuda_runtime.h>
#include <cstddef>

#include "common.cuh"

namespace yb {

constexpr int kAttnCapacity = 128;  // cache slots one CTA covers (two staged sub-chunks of 64)

struct AttnArgs {
  const float* q;         // [n_heads][head_dim]
  const __half* k_cache;  // [n_kv_heads][max_seq_len][head_dim]
  const __half* v_cache;  // [n_kv_heads][max_seq_len][head_dim]
  float* out;             // [n_heads][head_dim]
  float* part;            // [n_heads][s_max][head_dim + 2] slice partials (o, m, l)
  unsigned* counters;     // [n_kv_heads], zero between launches
  const StepState* step;  // kv_len is read from here when non-null ...
  int kv_len;             // ... else from here
  int max_seq_len;
  unsigned* status;
};

struct AttnPlan {
  bool ok;
  const void* fn;
  dim3 grid;
  int s_max;
  size_t smem;
  size_t part_floats;
};

AttnPlan attn_plan(int n_heads, int n_kv_heads, int head_dim, int max_seq_len);
cudaError_t attn_prepare(const AttnPlan& p);  // once per plan, outside stream capture
cudaError_t attn_launch(const AttnPlan& p, AttnArgs a, cudaStream_t stream, bool pdl);

}  // namespace yb
