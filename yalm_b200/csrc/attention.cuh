// Split-K GQA decode attention (see attention.cu).
#pragma once

#include <cuda_runtime.h>
#include <cstddef>

#include "common.cuh"

namespace yb {

constexpr int kAttnCapacity = 128;  // cache slots one CTA covers (8 warps x 16)

struct AttnArgs {
  const float* q;         // [n_heads][head_dim]
  const __half* k_cache;  // [n_kv_heads][max_seq_len][head_dim]
  const __half* v_cache;  // [n_kv_heads][max_seq_len][head_dim]
  float* out;             // [n_heads][head_dim]
  float* part;            // [n_heads][s_max][head_dim + 4] slice partials (o, m, l, padding)
  unsigned* counters;     // [n_kv_heads], zero between launches
  const StepState* step;  // kv_len is read from here when non-null ...
  int kv_len;             // ... else from here
  int max_seq_len;
  unsigned* status;
  // optional timeline (null = off): per CTA c = blockIdx.y * gridDim.x + blockIdx.x,
  // trace[c * trace_stride + j] = %globaltimer at j = 0 entry, 1 inputs ready, 2 K/V rows staged,
  // 5 slot groups done (thread 0), 3 slice partial written, 4 exit (inactive slices stamp only 0
  // and 1)
  unsigned long long* trace;
  int trace_stride;
};

struct AttnPlan {
  bool ok;
  const void* fn;
  dim3 grid;
  int s_max;
  size_t smem;
  size_t part_floats;
};

// Shared memory of one attention CTA: a region holding the staged K/V rows, or, when larger and
// below kAttnMergeSmemMax, the slice partials of one kv head (merged in shared memory); then the
// warp-combine buffer and the barriers.
constexpr size_t kAttnMergeSmemMax = 96 * 1024;
// Shared-memory row of a staged cache slot: head_dim fp16 padded by 16 bytes (an odd multiple of 16).
__host__ __device__ constexpr int attn_row_bytes(int hd) { return hd * 2 + 16; }
__host__ __device__ constexpr size_t attn_stage_bytes(int hd) { return (size_t)2 * kAttnCapacity * attn_row_bytes(hd); }
__host__ __device__ constexpr size_t attn_merge_bytes(int hd, int gq, int s_max) {
  return (size_t)gq * s_max * (hd + 4) * 4 + (size_t)2 * gq * s_max * 4;
}
__host__ __device__ constexpr bool attn_merge_in_smem(int hd, int gq, int s_max) {
  return attn_merge_bytes(hd, gq, s_max) <= kAttnMergeSmemMax;
}
__host__ __device__ constexpr size_t attn_region_bytes(int hd, int gq, int s_max) {
  return attn_merge_in_smem(hd, gq, s_max) && attn_merge_bytes(hd, gq, s_max) > attn_stage_bytes(hd)
             ? (attn_merge_bytes(hd, gq, s_max) + 127) / 128 * 128
             : attn_stage_bytes(hd);
}

// Warp-combine buffer: per warp and head the output row (head_dim + 4 floats), max and sum, the
// warp weights, then per head the CTA max and sum.
__host__ __device__ constexpr size_t attn_red_bytes(int hd, int gq) {
  return ((size_t)8 * gq * (hd + 4) + (size_t)8 * gq * 3 + (size_t)2 * gq) * 4;
}

AttnPlan attn_plan(int n_heads, int n_kv_heads, int head_dim, int max_seq_len);
cudaError_t attn_prepare(const AttnPlan& p);  // once per plan, outside stream capture
cudaError_t attn_launch(const AttnPlan& p, AttnArgs a, cudaStream_t stream, bool pdl);

// The plan of a standalone launch, built and prepared (attn_prepare) on the first call for each
// (device, shape) and looked up afterwards, so only that first call does host work and it must come
// before any stream capture.  Returns 0 or a YB_E* code (message via yb_last_error).  capi.cu.
int cached_attn_plan(int n_heads, int n_kv_heads, int head_dim, int max_seq_len, AttnPlan* out);

}  // namespace yb
