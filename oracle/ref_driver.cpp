// TEST INFRASTRUCTURE ONLY — never linked into, loaded by, or called from the product library.
//
// Drives yalm's own decode path (`Model::forward`, src/model.cpp:479-494: `_forward_cpu`,
// src/infer.cpp:483-528, or on a device the CUDA backends of src/infer.cu / src/coop.cu) so that
// tests and the bench's reference arm can compare against, and time, the reference itself.  The
// reference sources are compiled where they lie (see oracle/Makefile); this file only adds a flat
// extern "C" surface for ctypes and the drivers (open a .yalm file, move it to a device, step the
// model, read logits / KV).  Linked either with ref_cuda_stubs.cpp (the CPU-only build) or with the
// reference's own CUDA objects (the GPU build).
#include "model.h"

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <omp.h>
#include <string>

// ---- flat surface for ctypes ----
struct RefHandle {
  YALMData data;
  std::unique_ptr<Model> model;
  std::unique_ptr<InferenceState> state;
};

extern "C" {

// Opens a .yalm checkpoint with the reference loader (src/codec.cpp:97-156) and builds
// Model + InferenceState on the CPU (src/model.cpp:392-435, 291-307).  NULL on failure.
void* ref_open(const char* path, int context) {
  auto* h = new RefHandle();
  if (h->data.from_file(path) != 0) {
    delete h;
    return nullptr;
  }
  h->model = std::make_unique<Model>(h->data, context);
  h->state = std::make_unique<InferenceState>(h->model->config);
  return h;
}

// Config fields in a fixed order: dim, hidden_dim, head_dim, n_layers, n_heads, n_kv_heads,
// vocab_size, max_seq_len, rotary_dim, act (0 gelu / 1 silu), n_experts, n_experts_active.
void ref_config(void* hp, int* out12, float* out3) {
  const Config& c = *static_cast<RefHandle*>(hp)->model->config;
  int v[12] = {c.dim, c.hidden_dim, c.head_dim, c.n_layers, c.n_heads, c.n_kv_heads,
               c.vocab_size, c.max_seq_len, c.rotary_dim, c.act == ActivationType::SILU ? 1 : 0,
               c.n_experts, c.n_experts_active};
  std::memcpy(out12, v, sizeof(v));
  out3[0] = c.rope_theta;
  out3[1] = c.norm_eps;
  out3[2] = c.qkv_clip;
}

// One call of Model::forward (src/model.cpp:479-494) on the CPU.  mode 0 = HYDRATE_KV_CACHE,
// 1 = OUTPUT_LOGITS.  When logits_out is non-null and mode is 1, copies InferenceState::logits().
void ref_forward(void* hp, int token, int pos, int mode, float* logits_out) {
  auto* h = static_cast<RefHandle*>(hp);
  h->model->forward(*h->state, token, pos,
                    mode ? InferenceMode::OUTPUT_LOGITS : InferenceMode::HYDRATE_KV_CACHE);
  if (mode && logits_out) {
    std::memcpy(logits_out, h->state->logits(), sizeof(float) * h->model->config->vocab_size);
  }
}

// Reads n cache slots starting at slot pos0 of one layer / kv head, in canonical [slot][head_dim]
// order.  K is stored 16-tiled (k_cache_idx, src/model.h:14-17) and V as [head_dim][max_seq_len]
// (src/infer.cpp:300-305); both are decoded here.  fp16 bit patterns are returned unchanged.
void ref_read_kv(void* hp, int layer, int kvh, int pos0, int n, uint16_t* k_out, uint16_t* v_out) {
  auto* h = static_cast<RefHandle*>(hp);
  const Config& c = *h->model->config;
  const Block& b = *h->model->blocks[layer];
  const f16_t* kb = b.key_cache() + (size_t)kvh * c.head_dim * c.max_seq_len;
  const f16_t* vb = b.value_cache() + (size_t)kvh * c.head_dim * c.max_seq_len;
  for (int t = 0; t < n; ++t) {
    for (int j = 0; j < c.head_dim; ++j) {
      k_out[(size_t)t * c.head_dim + j] = kb[k_cache_idx(j, pos0 + t, c.max_seq_len)];
      v_out[(size_t)t * c.head_dim + j] = vb[(size_t)j * c.max_seq_len + pos0 + t];
    }
  }
}

void ref_close(void* hp) { delete static_cast<RefHandle*>(hp); }

// Moves the model and state to a device the way run_completion's setup_cuda does
// (src/main.cpp:57-86): "cuda" = Model::cuda() + InferenceState::cuda() (the CUDA-graph backend),
// "cuda-coop" = the cooperative backend.  Returns 0, or -1 for an unknown device name.  In the
// CPU-only build the CUDA symbols are stubs that abort.
int ref_to_device(void* hp, const char* device) {
  auto* h = static_cast<RefHandle*>(hp);
  const std::string d = device;
  if (d == "cpu") return 0;
  if (d == "cuda") {
    h->model->cuda();
    h->state->cuda();
    return 0;
  }
  if (d == "cuda-coop") {
    h->model->cuda_coop();
    h->state->cuda_coop();
    return 0;
  }
  return -1;
}

// Kernel-level hooks: the reference's own CPU test entry points (src/model.h:340-367).
void ref_matmul_f16(float* xout, float* x, uint16_t* w, int n, int d) { matmul_cpu(xout, x, w, n, d); }
void ref_matmul_f32(float* xout, float* x, float* w, int n, int d) { matmul_cpu(xout, x, w, n, d); }
void ref_mha(float* xout, float* att, uint16_t* kb, uint16_t* vb, float* q, int head_dim, int kv_len,
             int max_seq_len, int n_heads, int n_kv_heads) {
  mha_cpu(xout, att, kb, vb, q, head_dim, kv_len, max_seq_len, n_heads, n_kv_heads);
}
void ref_attn(float* xout, float* atth, float* qh, uint16_t* kh, uint16_t* vh, int head_dim, int n_kv_heads,
              int max_seq_len, int kv_len) {
  attn(xout, atth, qh, kh, vh, head_dim, n_kv_heads, max_seq_len, kv_len);
}
void ref_ffn_f32(float* xout, float* x, float* w1, float* w2, float* w3, int hidden_dim, int dim, int act_silu) {
  ffn_cpu(xout, x, w1, w2, w3, hidden_dim, dim, act_silu ? ActivationType::SILU : ActivationType::GELU);
}

void ref_set_threads(int n) { omp_set_num_threads(n); }
int ref_max_threads(void) { return omp_get_max_threads(); }

}  // extern "C"
