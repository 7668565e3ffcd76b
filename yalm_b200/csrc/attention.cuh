// GQA decode attention, one thread-block cluster per kv head (see attention.cu).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cstddef>

#include "common.cuh"

namespace yb {

struct AttnArgs {
  const float* q;         // [n_heads][head_dim]
  const __half* k_cache;  // [n_kv_heads][max_seq_len][head_dim]
  const __half* v_cache;  // [n_kv_heads][max_seq_len][head_dim]
  float* out;             // [n_heads][head_dim]
  float* part;            // [n_kv_heads][clusters][GQ][head_dim + 2] cluster records (o, m, l) of the
                          // merge over clusters (AttnPlan::part_floats; unused with one cluster)
  unsigned* counters;     // [n_kv_heads], zero between launches
  const StepState* step;  // kv_len is read from here when non-null ...
  int kv_len;             // ... else from here
  int max_seq_len;
  int cta_slots;          // slots per CTA before a kv head's cache splits over more CTAs (0: 128)
  int cluster_slots;      // slots per CTA of one cluster before the cache takes more clusters of the
                          // kv head, where the grid has them (0: 1024)
  unsigned* status;
  // optional timeline (null = off): per CTA c = blockIdx.y * gridDim.x + blockIdx.x,
  // trace[c * trace_stride + j] = %globaltimer at j = 0 entry, 7 early copies issued, 1 inputs
  // ready, 2 first stage landed, 5 slots folded, 6 warp weights formed, 3 record written, 4 exit
  // (CTAs without slots stamp only 0, 7 and 1)
  unsigned long long* trace;
  int trace_stride;
};

struct AttnPlan {
  bool ok;
  const void* fn;
  dim3 grid;           // (cluster * clusters per kv head, n_kv_heads)
  int cluster;         // CTAs per cluster
  int s_max;           // bound on the clusters per kv head (sizes the scratch)
  int max_seq_len;
  size_t smem;
  size_t part_floats;  // scratch floats for the merge over clusters, valid for any device
  int max_active[16];  // attn_prepare: clusters of 1..16 CTAs the device holds at once
};

// TMA tensor maps of one layer's K and V caches: [n_kv_heads * max_seq_len][head_dim] fp16 read in
// 64-slot x 64-dim boxes with the 128-byte swizzle.
struct AttnMaps {
  CUtensorMap k, v;
};
bool attn_maps(AttnMaps* m, const __half* k_cache, const __half* v_cache, int n_kv_heads, int max_seq_len,
               int head_dim);

// The shape's kernel, shared memory and a device-independent scratch bound (host arithmetic only).
AttnPlan attn_plan(int n_heads, int n_kv_heads, int head_dim, int max_seq_len);
// Once per plan and device, outside stream capture: kernel attributes, and the cluster size and
// clusters per kv head from the device's cluster occupancy (sets p.cluster and p.grid).
cudaError_t attn_prepare(AttnPlan& p);
cudaError_t attn_launch(const AttnPlan& p, AttnArgs a, const AttnMaps& m, cudaStream_t stream, bool pdl);

// The plan of a standalone launch, built and prepared (attn_prepare) on the first call for each
// (device, shape) and looked up afterwards, so only that first call does host work and it must come
// before any stream capture.  Returns 0 or a YB_E* code (message via yb_last_error).  capi.cu.
int cached_attn_plan(int n_heads, int n_kv_heads, int head_dim, int max_seq_len, AttnPlan* out);

}  // namespace yb
