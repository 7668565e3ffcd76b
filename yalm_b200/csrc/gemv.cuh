// Weight-streaming fp16 matrix-vector kernels for batch-1 decode.
//
// y = W x with W fp16 [rows, cols] row-major (row stride ldw elements), x fp32, fp32 accumulation.
// Each CTA owns a contiguous range of rows, so the weight bytes it reads form one contiguous range
// of HBM.  A producer warp streams that range through a ring of shared-memory stages with 1-D TMA
// (cp.async.bulk, evict-first L2 policy); each stage holds RT whole rows.  Eight consumer warps hold
// their slice of x in registers (thread t owns the 16-byte column chunks t, t+256, ...), so each
// stage byte is read from shared memory exactly once.  Per stage, a warp reduce-scatter folds the
// RT partial sums; the cross-warp sums and the fused epilogue run once at the end of the CTA.
//
// Kernel boundaries are hidden with programmatic dependent launch: a kernel triggers its
// dependents on entry, its producer fills the ring (and optionally prefetches further into L2)
// before griddepcontrol.wait, and only the consumers — which read activations written by the
// previous kernel — wait.
#pragma once

#include "common.cuh"

namespace yb {

enum GemvEpilogue : int {
  kEpiStore = 0,   // y[r] = sum                                   (classifier, plain matvec)
  kEpiResid = 1,   // y[r] += sum                                  (wo, w2: residual into x)
  kEpiGateUp = 2,  // rows interleaved gate/up: y[r/2] = act(gate) * up   (fused w1/w3 + SwiGLU)
  kEpiQKV = 3,     // [q; k; v] rows: clip, RoPE, q -> fp32, k/v -> fp16 KV cache (+ sink rotation)
  kEpiResidTP = 4, // partial sums pushed to every tensor-parallel peer's exchange slot
  kEpiStoreTP = 5, // row sums stored at row_offset + r in every tensor-parallel peer's buffer
};

constexpr int kGemvWarps = 8;  // consumer warps; one more warp is the TMA producer

struct GemvArgs {
  const __half* w;
  long long ldw;        // row stride of W in elements
  int rows;
  int cols;             // multiple of 8
  const float* x;       // [cols]
  const float* norm_w;  // non-null: x is RMS-normalised with this weight first (cols == dim)
  float eps;
  float* y;
  unsigned* status;
  const StepState* step;
  // shared-memory plan (host computed)
  unsigned stage_bytes;  // slot stride (>= RT * cols * 2, multiple of 128)
  int n_slots;
  int red_floats;        // rows-per-CTA upper bound * kGemvWarps
  int l2_prefetch_stages;
  // kEpiGateUp
  int act_silu;
  // kEpiQKV
  int q_rows, kv_rows, head_dim, rotary_dim, max_seq_len;
  float qkv_clip;
  const float* inv_freq;  // [head_dim / 2]
  int pos, kv_pos, kv_sink;  // used when step == nullptr (standalone launches)
  __half* k_cache;        // [kv_heads][max_seq_len][head_dim] for this layer
  __half* v_cache;
  // kEpiResidTP: per rank p, where this rank's partial rows go in p's exchange region, written as
  // 8-byte words {fp32 bits, step epoch} (no fence and no counter: the reader checks the epoch half
  // of every word).  kEpiStoreTP: per rank p, p's fp32 logits buffer and p's arrival counter for this
  // rank, bumped with a system-scope release once the CTA's rows are written.
  unsigned long long* const* peer_ll;
  float* const* peer_slots;
  unsigned* const* peer_counters;
  int tp_size;
  int row_offset;
  // tensor-parallel input: x_in = x + sum over ranks r (in rank order) of the fp32 halves of
  // tp_ll[r * cols ..], each word read once its epoch half equals the step's epoch.  Each CTA forms
  // its share of x_in into x_out (required), bumps tp_bar (zeroed by the step kernel) and, once all
  // gridDim.x CTAs have, reads x_in back from x_out.
  const unsigned long long* tp_ll;
  float* x_out;
  unsigned* tp_bar;
  // optional L2 warm-up of another matrix (the next small matvec's weights), split across CTAs and
  // issued once after this CTA's ring fill
  const unsigned char* pf_src;
  long long pf_bytes;
  // kEpiQKV: non-zero = also warm L2 with this layer's K/V cache slots [0, kv_len) (kv_len as the
  // step state shows it when the producer starts), split across CTAs, for the attention kernel
  int kv_prefetch;
  // optional timeline (null = off): per CTA, trace[cta * trace_stride + j] = %globaltimer at
  // j = 0 entry, 1 input vector loaded, 2 tensor-parallel all-reduce done (before 1), 3 last stage
  // consumed, 4 epilogue done
  unsigned long long* trace;
  int trace_stride;
};

}  // namespace yb
