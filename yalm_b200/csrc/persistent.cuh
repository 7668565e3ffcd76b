// Persistent decode step: one cooperative launch runs a whole token (see persistent.cu).
#pragma once

#include <cuda_runtime.h>
#include <cstddef>

#include "common.cuh"

namespace yb {

constexpr int kPWarps = 16;                   // consumer warps per CTA (one CTA per SM)
constexpr int kPThreads = (kPWarps + 1) * 32; // + one TMA producer warp
constexpr int kPSlotBytes = 32768;            // ring slot: whole weight rows or one K/V sub-chunk
constexpr int kPSlots = 6;
constexpr int kPAttnSub = 64;                 // cache slots per attention stage
constexpr int kPMaxSplits = 8;                // attention slices per kv head (merge cost bound)

struct PLayer {
  const __half* wqkv;  // [q_rows + 2 kv_rows, dim]
  const __half* wo;    // [dim, q_rows]
  const __half* w13;   // [2 hid, dim] (W1 / W3 rows interleaved)
  const __half* w2;    // [dim, hid]
  const float* rms_att;
  const float* rms_ffn;
  __half* k_cache;     // [n_kv][max_seq_len][head_dim]
  __half* v_cache;
};

struct PArgs {
  const PLayer* layers;
  int n_layers;
  int dim, q_rows, kv_rows, hid, vocab_rows, head_dim, rotary_dim, max_seq_len, n_kv;
  float eps, qkv_clip;
  int act_silu;
  const __half* emb;
  const __half* wcls;
  const float* rms_final;
  const float* inv_freq;
  float* x;      // residual stream (two ping-pong copies under tensor parallelism)
  float* x2;
  float* q;
  float* att;
  float* hb;
  float* logits;
  float* attn_part;             // [n_heads_l][kPMaxSplits][head_dim + 2]
  unsigned* attn_cnt;           // [n_kv]
  unsigned long long* bar;      // [0] grid barrier counter, [1] low word failure flag, then the
                                // per-phase stage-claim counters (u32); all zeroed before each launch
  unsigned* fail;               // nonzero once any CTA gave up a bounded wait (all others stop)
  unsigned* status;
  int token, pos, kv_sink, kv_pos, kv_len, mode;
  unsigned epoch, lepoch;
  // tensor parallelism (tp_size 1: unused)
  int tp_size, tp_rank;
  float* const* peer_slots;       // [(2 L + 1) * tp] destinations in peers' exchange regions
  unsigned* const* peer_counters; // [(2 L + 1) * tp]
  const float* tp_slots;          // local exchange slots [2 L][tp][dim]
  const unsigned* tp_counters;    // local counters [2 L + 1][tp]
  float* gathered_logits;         // local [vocab]
  int red_floats;                 // shared-memory row-partial buffer size (host computed)
  int max_local;                  // per-phase bound on the stages one CTA processes (host computed)
  int static_pct;                 // share of each matvec phase split statically, in percent
  int claim_ctrs;                 // counters the dynamic remainder is spread over (per phase)
  // optional timeline: per CTA kTraceEvents %globaltimer stamps (ns); null = off
  unsigned long long* trace;
};

// Timeline events per CTA: [0] consumer start, then per grid barrier j: [1 + 2j] arrive,
// [2 + 2j] release; after the last barrier: [kTraceEvents - 2] consumer end,
// [kTraceEvents - 1] producer end.
constexpr int kTraceMaxBarriers = 5 * 128;
constexpr int kTraceEvents = 2 * kTraceMaxBarriers + 3;

struct PersistPlan {
  bool ok;
  const void* fn;
  int grid;
  size_t smem;
  int kd, rd, ko, ro, kh, rh;  // per-phase chunks per thread / rows per stage (dim, wo input, hidden)
};

// Chooses the instantiation for a model shape; ok = false when none fits (use the graph executor).
PersistPlan persist_plan(int dim, int q_rows, int hid, int head_dim, int gq, int n_sms);
int persist_max_local(int rows, int rt, int grid, int static_pct);
size_t persist_smem_bytes(int red_floats, int max_local);
cudaError_t persist_prepare(const PersistPlan& p);
cudaError_t persist_launch(const PersistPlan& p, const PArgs& a, cudaStream_t stream);

}  // namespace yb
