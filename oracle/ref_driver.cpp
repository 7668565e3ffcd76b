// TEST INFRASTRUCTURE ONLY — never linked into, loaded by, or called from the product library.
//
// Drives yalm's own CPU decode path (`Model::forward` -> `_forward_cpu`, src/infer.cpp:483-528) so
// that tests and the bench's reference arm can compare against, and time, the reference itself.
// The reference sources are compiled where they lie (see oracle/Makefile); this file only adds:
//   * a flat extern "C" surface for ctypes (open a .yalm file, step the model, read logits / KV);
//   * definitions for the CUDA-side symbols that src/model.cpp references but that the CPU path
//     never calls (upload_cuda & co from src/infer.cu:60-91, the coop entry points from
//     src/coop.h:5-6, libgemm_init from src/libgemm.h:12, and the `_block_cuda*` /
//     `_forward_cuda*` members).  Each aborts: reaching one means the CPU path was not taken.
#include "model.h"
#include "coop.h"
#include "libgemm.h"

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <omp.h>
#include <string>

[[noreturn]] static void not_cpu(const char* what) {
  std::fprintf(stderr, "oracle/ref_driver: CUDA symbol %s reached on the CPU path\n", what);
  std::abort();
}

// ---- CUDA-side symbols referenced from src/model.cpp, unused on the CPU path ----
extern "C" void* upload_cuda(void*, size_t) { not_cpu("upload_cuda"); }
extern "C" void* download_cuda(void*, size_t, std::string) { not_cpu("download_cuda"); }
extern "C" void register_cuda_host(void*, size_t) { not_cpu("register_cuda_host"); }
extern "C" void free_cuda(void*) { not_cpu("free_cuda"); }
extern "C" void unregister_cuda_host(void*) { not_cpu("unregister_cuda_host"); }
extern "C" void set_cuda_device(int) { not_cpu("set_cuda_device"); }
extern "C" void init_cuda_stream(cudaStream_t*) { not_cpu("init_cuda_stream"); }
void yalm_coop_prepare(Model&) { not_cpu("yalm_coop_prepare"); }
void yalm_coop_forward(Model&, InferenceState&, int, int, InferenceMode) { not_cpu("yalm_coop_forward"); }
void libgemm_init(cudaStream_t, LibGemmBackend) { not_cpu("libgemm_init"); }
template <typename T>
void Block::_block_cuda(InferenceState&, int, int, int, int) const { not_cpu("Block::_block_cuda"); }
template <typename T>
void Block::_block_cuda_lib(InferenceState&, int, int, int, int) const { not_cpu("Block::_block_cuda_lib"); }
template void Block::_block_cuda<float>(InferenceState&, int, int, int, int) const;
template void Block::_block_cuda<f16_t>(InferenceState&, int, int, int, int) const;
template void Block::_block_cuda_lib<f16_t>(InferenceState&, int, int, int, int) const;
void Model::_forward_cuda(InferenceState&, int, int, InferenceMode) { not_cpu("Model::_forward_cuda"); }
void Model::_forward_cuda_lib(InferenceState&, int, int, InferenceMode) { not_cpu("Model::_forward_cuda_lib"); }

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
