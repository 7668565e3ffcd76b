// yb_prefill: a prompt through the model in one batched pass (tensor-core GEMMs for every matrix,
// causal attention over the new and the cached slots), replacing the token-by-token prompt loop of
// yalm's run_completion (src/main.cpp:171-177).  The KV cache ends up as the per-token steps would
// leave it: every fp16 activation entering a GEMM goes in as two planes, the fp16 value and its fp16
// remainder, so the products keep about 22 bits as the per-token path's fp32 dot products do.  The
// last token runs as one decode step (yb_forward), whose logits the caller receives.
#include "engine.h"
#include "prefill.cuh"
#include "prefill_gemm.cuh"

#include <algorithm>
#include <cstring>

using namespace yb;

namespace {

__global__ void prefill_embed_kernel(const __half* emb, const int* tokens, float* x, int dim) {
  const __half* row = emb + (size_t)tokens[blockIdx.x] * dim;
  float* xr = x + (size_t)blockIdx.x * dim;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) xr[i] = __half2float(row[i]);
}

int ensure_buffers(yb_engine* e, int T) {
  auto& p = e->pf;
  if (p.cap >= T) return 0;
  const yb_config& c = e->cfg;
  void* old[] = {p.x, p.xn, p.qkv, p.q, p.att, p.h, p.tokens};
  for (void* v : old) if (v) cudaFree(v);
  p = yb_engine::Prefill{};
  const size_t cap = (size_t)((T + 127) / 128 * 128);
  const size_t qkv_rows = (size_t)e->q_rows + 2 * e->kv_rows;
  // the GEMMs' fp16 inputs hold two planes each: values and their fp16 remainders
  YB_CK(cudaMalloc(&p.x, cap * c.dim * 4));
  YB_CK(cudaMalloc(&p.xn, 2 * cap * c.dim * 2));
  YB_CK(cudaMalloc(&p.qkv, cap * qkv_rows * 4));
  YB_CK(cudaMalloc(&p.q, cap * e->q_rows * 4));
  YB_CK(cudaMalloc(&p.att, 2 * cap * e->q_rows * 2));
  YB_CK(cudaMalloc(&p.h, 2 * cap * e->hid * 2));
  YB_CK(cudaMalloc(&p.tokens, cap * 4));
  p.cap = (int)cap;
  return 0;
}

// planes: 2 = A as values + remainders ([2][M][K]), 1 = values only; lo_out: fp16 outputs also
// write their remainder plane (for a two-plane GEMM after this one)
int gemm(const __half* A, const __half* B, int M, int N, int K, int epi, float* of, __half* oh, int ldo, int planes,
         bool lo_out, cudaStream_t s) {
  PrefillGemmArgs g{};
  g.M = M;
  g.N = N;
  g.K = K;
  g.epi = epi;
  g.ldo = ldo;
  g.out_f32 = of;
  g.out_f16 = oh;
  g.status = nullptr;
  g.a_planes = planes;
  g.lo_out = oh && lo_out ? 1 : 0;
  YB_CK(prefill_gemm(A, B, g, s));
  return 0;
}

}  // namespace

// Whether the batched path covers this engine and prompt (else the per-token steps run).
static bool batched_ok(const yb_engine* e, int n, int pos0) {
  const yb_config& c = e->cfg;
  return e->tp_size == 1 && e->esz == 2 && c.act == 1 && n >= 2 && pos0 + n <= c.max_seq_len &&
         c.dim % 64 == 0 && e->q_rows % 64 == 0 && e->hid % 64 == 0 && (c.head_dim == 64 || c.head_dim == 128);
}

// The batched pass over tokens[0, n) at positions pos0.. (KV cache only).
static int prefill_batched(yb_engine* e, const int* tokens, int n, int pos0) {
  YB_CK(cudaSetDevice(e->device));
  int rc = ensure_buffers(e, n);
  if (rc) return rc;
  const yb_config& c = e->cfg;
  cudaStream_t s = e->stream;
  auto& p = e->pf;
  const int qkv_rows = e->q_rows + 2 * e->kv_rows;
  YB_CK(cudaMemcpyAsync(p.tokens, tokens, (size_t)n * 4, cudaMemcpyHostToDevice, s));
  prefill_embed_kernel<<<n, 256, 0, s>>>(e->emb, p.tokens, p.x, c.dim);
  YB_CK(cudaGetLastError());
  // which GEMMs take the remainder plane (bit 0 QKV, 1 wo, 2 gate/up, 3 w2)
  const int pm = e->tune.prefill_planes;
  auto planes = [pm](int bit) { return (pm >> bit) & 1 ? 2 : 1; };
  for (int l = 0; l < c.n_layers; ++l) {
    LayerBuffers& L = e->layers[l];
    YB_CK(prefill_rmsnorm(p.x, L.rms_att, p.xn, p.xn + (size_t)n * c.dim, n, c.dim, c.norm_eps, s));
    if ((rc = gemm(p.xn, L.wqkv, n, qkv_rows, c.dim, kPreStore, p.qkv, nullptr, qkv_rows, planes(0), false, s)))
      return rc;
    YB_CK(prefill_qkv_post(p.qkv, n, pos0, e->q_rows, e->kv_rows, c.head_dim, c.rotary_dim, c.max_seq_len, c.qkv_clip,
                           e->inv_freq, p.q, L.k_cache, L.v_cache, s));
    YB_CK(prefill_attention(p.q, L.k_cache, L.v_cache, p.att, p.att + (size_t)n * e->q_rows, n, pos0, e->nh, e->nkv,
                            c.head_dim, c.max_seq_len, e->status_d, s));
    if ((rc = gemm(p.att, L.wo, n, c.dim, e->q_rows, kPreAdd, p.x, nullptr, c.dim, planes(1), false, s))) return rc;
    YB_CK(prefill_rmsnorm(p.x, L.rms_ffn, p.xn, p.xn + (size_t)n * c.dim, n, c.dim, c.norm_eps, s));
    if ((rc = gemm(p.xn, L.w13, n, 2 * e->hid, c.dim, kPreSwiGLU, nullptr, p.h, e->hid, planes(2), planes(3) == 2, s)))
      return rc;
    if ((rc = gemm(p.h, L.w2, n, c.dim, e->hid, kPreAdd, p.x, nullptr, c.dim, planes(3), false, s))) return rc;
  }
  return 0;
}

extern "C" int yb_prefill(yb_engine* e, const int* tokens, int n, int pos0, float* logits) {
  if (!e || !tokens || n <= 0 || pos0 < 0) return set_error(YB_E_INVALID, "bad prefill arguments");
  for (int i = 0; i < n; ++i)
    if (tokens[i] < 0 || tokens[i] >= e->cfg.vocab_size) return set_error(YB_E_INVALID, "token out of range");
  // all but the last token in one batched pass when it covers them, else as yalm's prompt loop
  // runs them; the last token is one decode step (its logits when asked for)
  int first = 0;
  if (batched_ok(e, n - 1, pos0)) {
    int rc = prefill_batched(e, tokens, n - 1, pos0);
    if (rc) return rc;
    first = n - 1;
  }
  for (int i = first; i < n; ++i) {
    const bool last = i + 1 == n;
    int rc = yb_forward(e, tokens[i], pos0 + i, last && logits ? YB_MODE_OUTPUT_LOGITS : YB_MODE_HYDRATE_KV_CACHE,
                        last ? logits : nullptr);
    if (rc) return rc;
  }
  return yb_sync(e);
}
