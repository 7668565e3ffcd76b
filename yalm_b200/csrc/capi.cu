// Kernel-level C entry points: yalm's test-hook counterparts (host arrays in/out) and launches of
// the individual decode kernels on caller-owned device buffers.
#include "engine.h"

#include <cstring>
#include <map>
#include <mutex>
#include <tuple>
#include <vector>

using namespace yb;

namespace {

int current_sms() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 148;
  return n;
}

// Device buffer owned by one host-array hook call.
struct DevBuf {
  void* p = nullptr;
  ~DevBuf() {
    if (p) cudaFree(p);
  }
  cudaError_t alloc(size_t n) { return cudaMalloc(&p, n ? n : 16); }
  template <typename T>
  T* as() const {
    return static_cast<T*>(p);
  }
};

GemvArgs plain_args() {
  GemvArgs a;
  std::memset(&a, 0, sizeof(a));
  a.tp_size = 1;
  return a;
}

// Plans for standalone launches, cached per (device, shape, epilogue) so that repeated calls cost
// one map lookup on the host.
std::mutex g_plan_mu;
std::map<std::tuple<int, int, int, int, bool>, GemvPlan> g_gemv_plans;
std::map<std::tuple<int, int, int, int, int>, AttnPlan> g_attn_plans;

int cached_gemv_plan(int rows, int cols, int epi, bool norm, GemvPlan* out) {
  int dev = 0;
  YB_CK(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(g_plan_mu);
  auto key = std::make_tuple(dev, rows, cols, epi, norm);
  auto it = g_gemv_plans.find(key);
  if (it == g_gemv_plans.end()) {
    GemvPlan p = gemv_plan(rows, cols, epi, norm, current_sms(), LaunchTuning::from_env());
    if (!p.ok)
      return set_error(YB_E_UNSUPPORTED,
                       "no matvec configuration for rows=" + std::to_string(rows) + " cols=" + std::to_string(cols));
    YB_CK(gemv_prepare(p));
    it = g_gemv_plans.emplace(key, p).first;
  }
  *out = it->second;
  return 0;
}

int launch_gemv_common(GemvArgs a, int epi, cudaStream_t s) {
  GemvPlan p;
  int rc = cached_gemv_plan(a.rows, a.cols, epi, a.norm_w != nullptr, &p);
  if (rc) return rc;
  YB_CK(gemv_launch(p, a, s, false, LaunchTuning::from_env().l2_prefetch_stages));
  return 0;
}

}  // namespace

// Attention plans for standalone launches (yb_attention_dev, yb_attention_dev_noalloc), cached per
// (device, shape): attn_prepare runs on the first call for a shape only.
namespace yb {
int cached_attn_plan(int nh, int nkv, int hd, int msl, AttnPlan* out) {
  int dev = 0;
  YB_CK(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(g_plan_mu);
  auto key = std::make_tuple(dev, nh, nkv, hd, msl);
  auto it = g_attn_plans.find(key);
  if (it == g_attn_plans.end()) {
    AttnPlan p = attn_plan(nh, nkv, hd, msl);
    if (!p.ok) return set_error(YB_E_UNSUPPORTED, "no attention configuration for this shape");
    YB_CK(attn_prepare(p));
    it = g_attn_plans.emplace(key, p).first;
  }
  *out = it->second;
  return 0;
}
}  // namespace yb

extern "C" int yb_num_sms(void) { return current_sms(); }

extern "C" int yb_gemv_dev(float* y, const float* x, const uint16_t* w, int rows, int cols, const float* norm_w,
                           float eps, int accumulate, void* stream) {
  if (!y || !x || !w || rows <= 0 || cols <= 0 || cols % 8) return set_error(YB_E_INVALID, "bad gemv arguments");
  // column panels for rows wider than one kernel covers (the engine's w2 at hidden_dim 28672)
  int panels = 1;
  while (gemv_kpt_for(cols / panels, 2) < 0 || (cols / panels) % 8 || cols % panels)
    if (++panels > 16) return set_error(YB_E_UNSUPPORTED, "no matvec configuration for cols=" + std::to_string(cols));
  if (panels > 1 && norm_w)
    return set_error(YB_E_UNSUPPORTED, "the RMSNorm prologue needs the whole row in one kernel (cols=" +
                                           std::to_string(cols) + ")");
  const int pcols = cols / panels;
  for (int p = 0; p < panels; ++p) {
    GemvArgs a = plain_args();
    a.w = reinterpret_cast<const __half*>(w) + (size_t)p * pcols;
    a.ldw = cols;
    a.rows = rows;
    a.cols = pcols;
    a.x = x + (size_t)p * pcols;
    a.norm_w = norm_w;
    a.eps = eps;
    a.y = y;
    int rc = launch_gemv_common(a, (accumulate || p > 0) ? kEpiResid : kEpiStore, static_cast<cudaStream_t>(stream));
    if (rc) return rc;
  }
  return 0;
}

extern "C" int yb_gateup_dev(float* hb, const float* x, const uint16_t* w13, int hidden, int dim, const float* norm_w,
                             float eps, int act, void* stream) {
  if (!hb || !x || !w13 || hidden <= 0 || dim <= 0 || dim % 8) return set_error(YB_E_INVALID, "bad gate/up arguments");
  GemvArgs a = plain_args();
  a.w = reinterpret_cast<const __half*>(w13);
  a.ldw = dim;
  a.rows = 2 * hidden;
  a.cols = dim;
  a.x = x;
  a.norm_w = norm_w;
  a.eps = eps;
  a.y = hb;
  a.act_silu = act;
  return launch_gemv_common(a, kEpiGateUp, static_cast<cudaStream_t>(stream));
}

extern "C" int yb_qkv_dev(float* q_out, uint16_t* k_cache, uint16_t* v_cache, const float* x, const uint16_t* wqkv,
                          const float* norm_w, float eps, int dim, int n_heads, int n_kv_heads, int head_dim,
                          int rotary_dim, int max_seq_len, int pos, int kv_pos, int kv_sink, float qkv_clip,
                          const float* inv_freq_dev, void* stream) {
  if (!q_out || !k_cache || !v_cache || !x || !wqkv || !inv_freq_dev || dim <= 0 || dim % 8 || n_heads <= 0 ||
      n_kv_heads <= 0 || head_dim <= 0 || (head_dim & 1) || rotary_dim < 0 || rotary_dim > head_dim || (rotary_dim & 1) ||
      pos < 0 || kv_pos < 0 || kv_pos >= max_seq_len || kv_sink < 0 || kv_sink > kv_pos)
    return set_error(YB_E_INVALID, "bad qkv arguments");
  GemvArgs a = plain_args();
  a.w = reinterpret_cast<const __half*>(wqkv);
  a.ldw = dim;
  a.q_rows = n_heads * head_dim;
  a.kv_rows = n_kv_heads * head_dim;
  a.rows = a.q_rows + 2 * a.kv_rows;
  a.cols = dim;
  a.x = x;
  a.norm_w = norm_w;
  a.eps = eps;
  a.y = q_out;
  a.head_dim = head_dim;
  a.rotary_dim = rotary_dim;
  a.max_seq_len = max_seq_len;
  a.qkv_clip = qkv_clip;
  a.inv_freq = inv_freq_dev;
  a.k_cache = reinterpret_cast<__half*>(k_cache);
  a.v_cache = reinterpret_cast<__half*>(v_cache);
  a.pos = pos;
  a.kv_pos = kv_pos;
  a.kv_sink = kv_sink;
  return launch_gemv_common(a, kEpiQKV, static_cast<cudaStream_t>(stream));
}

extern "C" size_t yb_attention_scratch_bytes(int n_heads, int n_kv_heads, int head_dim, int max_seq_len) {
  AttnPlan p = attn_plan(n_heads, n_kv_heads, head_dim, max_seq_len);
  if (!p.ok) return 0;
  return (p.part_floats * 4 + 255) / 256 * 256 + (size_t)n_kv_heads * 4;
}

extern "C" int yb_attention_plan_info(int n_heads, int n_kv_heads, int head_dim, int max_seq_len, int* out20) {
  if (!out20) return set_error(YB_E_INVALID, "null argument");
  AttnPlan p;
  int rc = cached_attn_plan(n_heads, n_kv_heads, head_dim, max_seq_len, &p);
  if (rc) return rc;
  out20[0] = p.cluster;
  out20[1] = (int)p.grid.x / p.cluster;
  out20[2] = (int)(p.grid.x * p.grid.y);
  out20[3] = (int)p.smem;
  for (int c = 0; c < 16; ++c) out20[4 + c] = p.max_active[c];
  return 0;
}

extern "C" int yb_attention_dev(float* out, const float* q, const uint16_t* k_cache, const uint16_t* v_cache,
                                int n_heads, int n_kv_heads, int head_dim, int max_seq_len, int kv_len,
                                void* scratch_dev, void* stream) {
  if (!out || !q || !k_cache || !v_cache || !scratch_dev || kv_len <= 0 || kv_len > max_seq_len)
    return set_error(YB_E_INVALID, "bad attention arguments");
  AttnPlan p;
  int rc = cached_attn_plan(n_heads, n_kv_heads, head_dim, max_seq_len, &p);
  if (rc) return rc;
  AttnArgs a;
  std::memset(&a, 0, sizeof(a));
  a.q = q;
  a.k_cache = reinterpret_cast<const __half*>(k_cache);
  a.v_cache = reinterpret_cast<const __half*>(v_cache);
  a.out = out;
  a.part = static_cast<float*>(scratch_dev);
  a.counters = reinterpret_cast<unsigned*>(static_cast<char*>(scratch_dev) + (p.part_floats * 4 + 255) / 256 * 256);
  a.step = nullptr;
  a.kv_len = kv_len;
  a.max_seq_len = max_seq_len;
  a.cta_slots = LaunchTuning::from_env().attn_cta_slots;
  a.cluster_slots = LaunchTuning::from_env().attn_cluster_slots;
  AttnMaps m;
  if (!attn_maps(&m, a.k_cache, a.v_cache, n_kv_heads, max_seq_len, head_dim))
    return set_error(YB_E_CUDA, "tensor map encoding of the KV cache failed");
  YB_CK(attn_launch(p, a, m, static_cast<cudaStream_t>(stream), false));
  return 0;
}

// ---------------------------------------------------------------------------------- yalm test hooks
extern "C" int yb_matmul(float* xout, const float* x, const uint16_t* w, int n, int d) {
  if (!xout || !x || !w || n <= 0 || d <= 0 || n % 8) return set_error(YB_E_INVALID, "bad matmul arguments");
  DevBuf dw, dx, dy;
  YB_CK(dw.alloc((size_t)n * d * 2));
  YB_CK(dx.alloc((size_t)n * 4));
  YB_CK(dy.alloc((size_t)d * 4));
  YB_CK(cudaMemcpy(dw.p, w, (size_t)n * d * 2, cudaMemcpyHostToDevice));
  YB_CK(cudaMemcpy(dx.p, x, (size_t)n * 4, cudaMemcpyHostToDevice));
  int rc = yb_gemv_dev(dy.as<float>(), dx.as<float>(), dw.as<uint16_t>(), d, n, nullptr, 0.f, 0, nullptr);
  if (rc) return rc;
  YB_CK(cudaMemcpy(xout, dy.p, (size_t)d * 4, cudaMemcpyDeviceToHost));
  return 0;
}

extern "C" int yb_mha(float* xout, float* att, const uint16_t* kb, const uint16_t* vb, const float* q, int head_dim,
                      int kv_len, int max_seq_len, int n_heads, int n_kv_heads) {
  (void)att;
  if (!xout || !kb || !vb || !q || head_dim <= 0 || n_kv_heads <= 0 || kv_len <= 0 || kv_len > max_seq_len)
    return set_error(YB_E_INVALID, "bad mha arguments");
  // yalm layouts -> [n_kv][slot][head_dim]: K is 16-tiled (k_cache_idx, src/model.h:14-17),
  // V is [n_kv][head_dim][max_seq_len] (src/infer.cpp:304).
  const size_t hd = head_dim, msl = max_seq_len;
  std::vector<uint16_t> k((size_t)n_kv_heads * msl * hd), v(k.size());
  for (int g = 0; g < n_kv_heads; ++g)
    for (size_t t = 0; t < msl; ++t)
      for (size_t i = 0; i < hd; ++i) {
        const size_t kidx = (i / 16) * (16 * msl) + t * 16 + (i % 16);
        k[((size_t)g * msl + t) * hd + i] = kb[(size_t)g * hd * msl + kidx];
        v[((size_t)g * msl + t) * hd + i] = vb[(size_t)g * hd * msl + i * msl + t];
      }
  const size_t scratch = yb_attention_scratch_bytes(n_heads, n_kv_heads, head_dim, max_seq_len);
  if (!scratch) return set_error(YB_E_UNSUPPORTED, "no attention configuration for this shape");
  DevBuf dk, dv, dq, dout, ds;
  YB_CK(dk.alloc(k.size() * 2));
  YB_CK(dv.alloc(v.size() * 2));
  YB_CK(dq.alloc((size_t)n_heads * hd * 4));
  YB_CK(dout.alloc((size_t)n_heads * hd * 4));
  YB_CK(ds.alloc(scratch));
  YB_CK(cudaMemset(ds.p, 0, scratch));
  YB_CK(cudaMemcpy(dk.p, k.data(), k.size() * 2, cudaMemcpyHostToDevice));
  YB_CK(cudaMemcpy(dv.p, v.data(), v.size() * 2, cudaMemcpyHostToDevice));
  YB_CK(cudaMemcpy(dq.p, q, (size_t)n_heads * hd * 4, cudaMemcpyHostToDevice));
  int rc = yb_attention_dev(dout.as<float>(), dq.as<float>(), dk.as<uint16_t>(), dv.as<uint16_t>(), n_heads, n_kv_heads,
                            head_dim, max_seq_len, kv_len, ds.p, nullptr);
  if (rc) return rc;
  YB_CK(cudaMemcpy(xout, dout.p, (size_t)n_heads * hd * 4, cudaMemcpyDeviceToHost));
  return 0;
}

extern "C" int yb_ffn(float* xout, const float* x, const uint16_t* w1, const uint16_t* w2, const uint16_t* w3,
                      int hidden_dim, int dim, int act) {
  if (!xout || !x || !w1 || !w2 || !w3 || hidden_dim <= 0 || dim <= 0 || dim % 8 || hidden_dim % 8)
    return set_error(YB_E_INVALID, "bad ffn arguments");
  const size_t H = hidden_dim, D = dim;
  DevBuf dw13, dw2, dx, dh, dy;
  YB_CK(dw13.alloc(2 * H * D * 2));
  YB_CK(dw2.alloc(D * H * 2));
  YB_CK(dx.alloc(D * 4));
  YB_CK(dh.alloc(H * 4));
  YB_CK(dy.alloc(D * 4));
  YB_CK(cudaMemcpy2D(dw13.p, 2 * D * 2, w1, D * 2, D * 2, H, cudaMemcpyHostToDevice));
  YB_CK(cudaMemcpy2D(static_cast<char*>(dw13.p) + D * 2, 2 * D * 2, w3, D * 2, D * 2, H, cudaMemcpyHostToDevice));
  YB_CK(cudaMemcpy(dw2.p, w2, D * H * 2, cudaMemcpyHostToDevice));
  YB_CK(cudaMemcpy(dx.p, x, D * 4, cudaMemcpyHostToDevice));
  int rc = yb_gateup_dev(dh.as<float>(), dx.as<float>(), dw13.as<uint16_t>(), hidden_dim, dim, nullptr, 0.f, act, nullptr);
  if (rc) return rc;
  rc = yb_gemv_dev(dy.as<float>(), dh.as<float>(), dw2.as<uint16_t>(), dim, hidden_dim, nullptr, 0.f, 0, nullptr);
  if (rc) return rc;
  YB_CK(cudaMemcpy(xout, dy.p, D * 4, cudaMemcpyDeviceToHost));
  return 0;
}

// ------------------------------------------------------------------------ prefill GEMM (test hook)
#include "prefill.cuh"
#include "prefill_gemm.cuh"

extern "C" int yb_prefill_attention_dev(uint16_t* out, const float* q, const uint16_t* k_cache, const uint16_t* v_cache,
                                        int T, int pos0, int n_heads, int n_kv_heads, int head_dim, int max_seq_len,
                                        void* stream) {
  using namespace yb;
  if (!out || !q || !k_cache || !v_cache) return set_error(YB_E_INVALID, "null buffer");
  YB_CK(prefill_attention(q, reinterpret_cast<const __half*>(k_cache), reinterpret_cast<const __half*>(v_cache),
                          reinterpret_cast<__half*>(out), nullptr, T, pos0, n_heads, n_kv_heads, head_dim, max_seq_len,
                          nullptr, static_cast<cudaStream_t>(stream)));
  return 0;
}

extern "C" int yb_prefill_gemm_dev(float* out_f32, uint16_t* out_f16, const uint16_t* a, const uint16_t* b, int M,
                                   int N, int K, int epi, int ldo, void* stream) {
  using namespace yb;
  const int kind = epi & 3;
  if (epi < 0 || epi > 15 || ((epi & 8) && kind != kPreSwiGLU && kind != kPreStoreF16))
    return set_error(YB_E_INVALID, "bad epilogue");
  PrefillGemmArgs g{};
  g.M = M;
  g.N = N;
  g.K = K;
  g.epi = kind;
  g.a_planes = (epi & 4) ? 2 : 1;
  g.lo_out = (epi & 8) ? 1 : 0;
  g.ldo = ldo;
  g.out_f32 = out_f32;
  g.out_f16 = reinterpret_cast<__half*>(out_f16);
  g.status = nullptr;
  cudaError_t e = prefill_gemm(reinterpret_cast<const __half*>(a), reinterpret_cast<const __half*>(b), g,
                               static_cast<cudaStream_t>(stream));
  if (e == cudaErrorInvalidValue) return set_error(YB_E_INVALID, "unsupported GEMM shape or pointers (K % 64, N % 8, 16-byte alignment)");
  YB_CK(e);
  return 0;
}
