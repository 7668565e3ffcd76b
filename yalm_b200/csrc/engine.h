// Host-side decode engine: weight upload/packing, device buffers, per-step CUDA graphs.
#pragma once

#include <cuda_runtime.h>

#include <string>
#include <vector>

#include "../../include/yalm_b200.h"
#include "attention.cuh"
#include "sampler.cuh"
#include "common.cuh"
#include "gemv.cuh"
#include "launch.h"
#include "persistent.cuh"

namespace yb {

int set_error(int code, const std::string& msg);
const std::string& last_error();

#define YB_CK(x)                                                                                    \
  do {                                                                                              \
    cudaError_t _e = (x);                                                                           \
    if (_e != cudaSuccess)                                                                          \
      return ::yb::set_error(YB_E_CUDA, std::string(#x) + " failed: " + cudaGetErrorString(_e));    \
  } while (0)

// Element ranges [begin, end) of the tensor-parallel slices one rank holds (engine.cu shard_table).
struct ShardTable {
  long long q0, q1;    // rows of Wq, columns of Wo
  long long kv0, kv1;  // rows of Wk, Wv
  long long h0, h1;    // rows of W1 / W3, columns of W2
  long long v0, v1;    // classifier rows
};

struct LayerBuffers {
  __half* wqkv = nullptr;   // [q_rows + 2 kv_rows, dim]: this rank's Wq, Wk, Wv rows
  __half* wo = nullptr;     // [dim, q_rows]: this rank's Wo columns
  __half* w13 = nullptr;    // [2 hidden_l, dim]: W1 / W3 rows interleaved
  __half* w2 = nullptr;     // [dim, hidden_l]: this rank's W2 columns
  float* rms_att = nullptr;
  float* rms_ffn = nullptr;
  __half* k_cache = nullptr;  // [kv_heads_l][max_seq_len][head_dim]
  __half* v_cache = nullptr;
  yb::AttnMaps attn_maps{};   // TMA maps of k_cache / v_cache for the decode attention
};

// Tensor-parallel exchange region (one device allocation per rank, mapped by every peer).
struct TpRegion {
  void* base = nullptr;          // local allocation
  size_t bytes = 0;
  size_t x_off = 0;              // [2*n_layers][tp][dim] exchange words {fp32 partial, epoch}
  size_t logit_off = 0;          // [vocab] fp32 gathered logits
  size_t cnt_off = 0;            // [tp] u32 logits arrival counters
  std::vector<void*> peer_base;  // per rank (own rank: base)
  // device arrays of pointers used by kernels: [2*n_layers][tp] exchange destinations, [tp]
  // logits destinations and counters
  unsigned long long** d_peer_ll = nullptr;
  unsigned* d_bar = nullptr;  // [2*n_layers] arrival counters of the in-kernel barrier, zeroed per step
  float** d_peer_slots = nullptr;
  unsigned** d_peer_counters = nullptr;
  bool joined = false;
};

struct StepArgs {
  StepState* step;
  float* x;
  const __half* emb;
  int dim;
  int token;
  int pos;
  int max_seq_len;
  unsigned epoch;
  unsigned lepoch;
  int sample_op;
  int sample_target;
  float temperature;
  float coin;
  unsigned* bar;  // counters the step kernel zeroes (tensor-parallel barriers), n_bar of them
  int n_bar;
  int esz;  // bytes per weight: 2 fp16, 1 fp8 E5M2
};

// Graph / launch variants of a step: the two InferenceModes, and logits followed by the sampler.
constexpr int kStepHydrate = 0, kStepLogits = 1, kStepSample = 2, kStepVariants = 3;

}  // namespace yb

struct yb_engine {
  int device = 0;
  int n_sms = 148;
  cudaStream_t stream = nullptr;
  yb_config cfg{};
  int tp_rank = 0, tp_size = 1;
  int esz = 2;  // bytes per weight: 2 fp16, 1 fp8 E5M2 (device matrices hold that many bytes per element)
  bool fp8_grouped = false;  // fp8 matrices (not the embedding) in the tensor-core matvec's grouped layout
  // local (this rank's) shapes
  int nh = 0, nkv = 0, q_rows = 0, kv_rows = 0, hid = 0, vocab_l = 0;

  std::vector<yb::LayerBuffers> layers;
  __half* emb = nullptr;
  __half* wcls = nullptr;
  float* rms_final = nullptr;
  float* inv_freq = nullptr;
  float* x = nullptr;       // residual stream [dim] (TP: two ping-pong copies)
  float* x2 = nullptr;
  float* q = nullptr;       // [q_rows]
  float* att = nullptr;     // [q_rows]
  float* hb = nullptr;      // [hidden_l]
  float* logits = nullptr;  // [vocab] (TP: full gathered vector)
  float* attn_part = nullptr;
  unsigned* attn_cnt = nullptr;
  yb::StepState* step = nullptr;
  unsigned* status_h = nullptr;  // host-mapped status word
  unsigned* status_d = nullptr;
  std::vector<void*> allocs;
  size_t upload_bytes = 0;  // host bytes uploaded by yb_create

  yb::LaunchTuning tune;
  yb::GemvPlan plan_qkv{}, plan_wo{}, plan_gu{}, plan_w2{}, plan_cls{};
  yb::GemvPlan plan_qkv_tp{};  // tensor parallel: QKV of layers >= 1 (adds the previous w2 partials)
  int w2_panels = 1;
  yb::ShardTable shard{};
  yb::AttnPlan plan_attn{};

  // executor: per-step CUDA graph of kernels (false) or one persistent cooperative kernel (true)
  bool persistent = false;
  yb::PersistPlan plan_persist{};
  yb::PLayer* d_players = nullptr;
  unsigned long long* persist_sync = nullptr;  // [0] grid barrier counter, [1] failure flag
  int persist_red_floats = 0;
  int persist_max_local = 0;
  size_t persist_sync_bytes = 0;
  unsigned long long* trace = nullptr;  // YB_TRACE=1: persistent-kernel timeline of the last step
  // YB_TRACE=1 with the graph executor: per kernel of the step (in launch order: per layer qkv,
  // attention, wo, gate/up, w2 panels; then the classifier) 8 stamps per CTA, [cta][kernel * 8 + j]
  unsigned long long* gtrace = nullptr;
  int gtrace_rows = 0, gtrace_events = 0;
  cudaGraph_t graph[yb::kStepVariants] = {};
  cudaGraphExec_t exec[yb::kStepVariants] = {};
  cudaGraphNode_t step_node[yb::kStepVariants] = {};
  yb::SampleResult* sample_h = nullptr;  // host-mapped result of the on-device sampler
  yb::SampleResult* sample_d = nullptr;
  unsigned epoch = 0;
  unsigned lepoch = 0;
  yb::TpRegion tp;
  // batched prefill work buffers (allocated on first use, grown to the largest prompt)
  struct Prefill {
    int cap = 0;
    float* x = nullptr;       // [cap][dim] residual stream
    __half* xn = nullptr;     // [cap][dim] normalised, fp16 GEMM operand
    float* qkv = nullptr;     // [cap][q + 2 kv]
    float* q = nullptr;       // [cap][q_rows] after RoPE
    __half* att = nullptr;    // [cap][q_rows]
    __half* h = nullptr;      // [cap][hidden_l]
    int* tokens = nullptr;    // [cap]
  } pf;
};

namespace yb {
// Records one decode step (mode 0 hydrate / 1 logits) on e->stream.  Used for graph capture.
int record_step(yb_engine* e, int mode, const StepArgs& sa);
}  // namespace yb
