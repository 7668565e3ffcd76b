// TEST INFRASTRUCTURE ONLY — times yalm's own per-layer decode kernels (src/infer.cu) on the B200.
//
// The reference's CUDA source is compiled where it lies (the include below; oracle/Makefile passes
// its path as YALM_INFER_CU) for sm_100a, and its kernels run with the launch shapes its per-layer graph uses
// (Block::_block_cuda, src/infer.cu:891-1072): fused_qkv_matmul_clip, attn_fused (one CTA per query
// head, scores in shared memory), fused_matmul_add_residuals (wo), fused_ffn_w1_w3_glu_act and
// fused_matmul_add_residuals_row (w2).  Each kernel is launched `iters` times back to back over
// rotating copies of its weights / cache (more than 4 x the 126 MB L2 in total, so every launch
// streams from HBM as inside a decode step) and timed with CUDA events on its stream; the mean per
// launch is printed as one JSON line with the algorithmic bytes of a launch.
//
//   ref_kernels [iters] [kv_len ...]     (Mistral-7B shapes, fp16 weights, context 4096)
#include YALM_INFER_CU

#include <cstdint>
#include <string>
#include <vector>

namespace {

__global__ void fill_half(half* p, size_t n, uint32_t seed, float scale) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    uint32_t h = (uint32_t)i * 2654435761u ^ seed;
    h ^= h >> 15;
    h *= 2246822519u;
    h ^= h >> 13;
    // uniform in [-1, 1) times scale: the timing does not depend on the values
    p[i] = __float2half(((float)(h & 0xFFFFFF) / 8388608.0f - 1.0f) * scale);
  }
}

__global__ void fill_float(float* p, size_t n, uint32_t seed) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    uint32_t h = (uint32_t)i * 2246822519u ^ seed;
    h ^= h >> 16;
    h *= 2654435761u;
    p[i] = (float)(h & 0xFFFF) / 32768.0f - 1.0f;
  }
}

half* halves(size_t n, uint32_t seed, float scale) {
  half* p = nullptr;
  CUDA_CHECK(cudaMalloc(&p, n * sizeof(half)));
  fill_half<<<1184, 256>>>(p, n, seed, scale);
  CUDA_CHECK(cudaGetLastError());
  return p;
}

float* floats(size_t n, uint32_t seed) {
  float* p = nullptr;
  CUDA_CHECK(cudaMalloc(&p, n * sizeof(float)));
  fill_float<<<1184, 256>>>(p, n, seed);
  CUDA_CHECK(cudaGetLastError());
  return p;
}

template <typename F>
double time_us(cudaStream_t s, int iters, F launch) {
  for (int i = 0; i < 3; ++i) launch(i);
  CUDA_CHECK(cudaStreamSynchronize(s));
  cudaEvent_t a, b;
  CUDA_CHECK(cudaEventCreate(&a));
  CUDA_CHECK(cudaEventCreate(&b));
  CUDA_CHECK(cudaEventRecord(a, s));
  for (int i = 0; i < iters; ++i) launch(i);
  CUDA_CHECK(cudaEventRecord(b, s));
  CUDA_CHECK(cudaEventSynchronize(b));
  CUDA_CHECK(cudaGetLastError());
  float ms = 0.f;
  CUDA_CHECK(cudaEventElapsedTime(&ms, a, b));
  CUDA_CHECK(cudaEventDestroy(a));
  CUDA_CHECK(cudaEventDestroy(b));
  return 1000.0 * ms / iters;
}

}  // namespace

int main(int argc, char** argv) {
  const int iters = argc > 1 ? std::atoi(argv[1]) : 64;
  std::vector<int> kv_lens;
  for (int i = 2; i < argc; ++i) kv_lens.push_back(std::atoi(argv[i]));
  if (kv_lens.empty()) kv_lens = {76, 1024, 3232};

  // Mistral-7B: dim 4096, 32 / 8 heads of 128, SwiGLU 14336, context 4096
  const int dim = 4096, hidden = 14336, head_dim = 128, n_heads = 32, n_kv = 8, msl = 4096;
  const int q_dim = n_heads * head_dim, kv_dim = n_kv * head_dim;
  const float clip = FLT_MAX;
  set_cuda_device(0);  // the reference's own device setup (warp size, threads per block)
  cudaStream_t s;
  CUDA_CHECK(cudaStreamCreate(&s));
  cudaDeviceProp prop;
  CUDA_CHECK(cudaGetDeviceProperties(&prop, 0));

  const int NW = 6;    // weight copies: 6 x 440 MB per layer set
  const int NKV = 24;  // K/V copies: 24 x 16 MB
  std::vector<half*> wq(NW), wk(NW), wv(NW), wo(NW), w1(NW), w2(NW), w3(NW);
  for (int i = 0; i < NW; ++i) {
    wq[i] = halves((size_t)q_dim * dim, 11 + i, 0.03f);
    wk[i] = halves((size_t)kv_dim * dim, 21 + i, 0.03f);
    wv[i] = halves((size_t)kv_dim * dim, 31 + i, 0.03f);
    wo[i] = halves((size_t)dim * q_dim, 41 + i, 0.03f);
    w1[i] = halves((size_t)hidden * dim, 51 + i, 0.03f);
    w2[i] = halves((size_t)dim * hidden, 61 + i, 0.03f);
    w3[i] = halves((size_t)hidden * dim, 71 + i, 0.03f);
  }
  std::vector<half*> kb(NKV), vb(NKV);
  for (int i = 0; i < NKV; ++i) {
    kb[i] = halves((size_t)n_kv * head_dim * msl, 81 + i, 1.0f);
    vb[i] = halves((size_t)n_kv * head_dim * msl, 91 + i, 1.0f);
  }
  float* x = floats(dim, 1);
  float* xb = floats(dim, 2);
  float* xb2 = floats(q_dim, 3);
  float* q = floats(q_dim, 4);
  float* k = floats(kv_dim, 5);
  float* v = floats(kv_dim, 6);
  float* hb = floats(hidden, 7);
  CUDA_CHECK(cudaDeviceSynchronize());

  const int ws = warp_size, mtb = max_threads_per_block;
  std::string out = "{\"device\": \"" + std::string(prop.name) + "\", \"iters\": " + std::to_string(iters) +
                    ", \"shape\": \"mistral-7b (dim 4096, 32/8 heads x 128, hidden 14336, context 4096), fp16\"" +
                    ", \"launch\": \"Block::_block_cuda launch shapes (src/infer.cu:891-1072)\", \"kernels\": {";
  auto add = [&](const std::string& name, double us, double bytes, bool first = false) {
    char buf[256];
    std::snprintf(buf, sizeof(buf), "%s\"%s\": {\"us\": %.3f, \"bytes\": %.0f, \"gbs\": %.1f}", first ? "" : ", ",
                  name.c_str(), us, bytes, bytes / (us * 1e-6) / 1e9);
    out += buf;
  };

  double us = time_us(s, iters, [&](int i) {
    const int j = i % NW;
    fused_qkv_matmul_clip<half><<<(q_dim + 2 * kv_dim + 31) / 32, ws * 32, 0, s>>>(wq[j], wk[j], wv[j], xb, dim, q_dim,
                                                                                  kv_dim, clip, q, k, v);
  });
  add("fused_qkv_matmul_clip", us, 2.0 * (q_dim + 2 * kv_dim) * dim + 4.0 * dim + 4.0 * (q_dim + 2 * kv_dim), true);

  for (int kv_len : kv_lens) {
    us = time_us(s, iters, [&](int i) {
      const int j = i % NKV;
      attn_fused<<<n_heads, mtb, msl * sizeof(float), s>>>(kb[j], vb[j], q, head_dim, kv_len, msl, n_heads, n_kv, xb2);
    });
    add("attn_fused@kv_len=" + std::to_string(kv_len), us, 2.0 * 2 * n_kv * head_dim * kv_len + 8.0 * q_dim);
  }

  us = time_us(s, iters, [&](int i) {
    fused_matmul_add_residuals<half><<<dim / 32, ws * 32, 0, s>>>(wo[i % NW], xb2, q_dim, dim, x);
  });
  add("fused_matmul_add_residuals(wo)", us, 2.0 * dim * q_dim + 4.0 * q_dim + 8.0 * dim);

  us = time_us(s, iters, [&](int i) {
    const int j = i % NW;
    fused_ffn_w1_w3_glu_act<half, ActivationType::SILU><<<(hidden + 31) / 32, ws * 32, 0, s>>>(w1[j], w3[j], xb, dim,
                                                                                              hidden, hb);
  });
  add("fused_ffn_w1_w3_glu_act", us, 2.0 * 2 * hidden * dim + 4.0 * dim + 4.0 * hidden);

  us = time_us(s, iters, [&](int i) {
    fused_matmul_add_residuals_row<half><<<dim, ws, 0, s>>>(w2[i % NW], hb, hidden, dim, x);
  });
  add("fused_matmul_add_residuals_row(w2)", us, 2.0 * dim * hidden + 4.0 * hidden + 8.0 * dim);

  out += "}}";
  std::printf("%s\n", out.c_str());
  return 0;
}
