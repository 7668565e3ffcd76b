// Batched prefill kernels other than the GEMMs.  yalm prefills one token at a time
// (src/main.cpp:171-177); here the prompt goes through each layer as one [T][dim] activation
// matrix: RMSNorm rows -> QKV GEMM -> clip / RoPE / KV append -> causal attention -> wo GEMM
// (+ residual) -> RMSNorm rows -> gate/up GEMM (+ SwiGLU) -> w2 GEMM (+ residual).
#include "prefill.cuh"

#include <cstdlib>
#include <cstring>

#include <math.h>

namespace yb {

// ---------------------------------------------------------------------------------------- RMSNorm
// fp32 pair -> fp16 pair at hi[i] and, when lo is set, its fp16 remainder at lo[i] (the two sum to the
// fp32 values within about 2^-22 relative, for the tensor-core GEMMs that take both as planes).
__device__ __forceinline__ void store_hilo(__half* hi, __half* lo, size_t i, float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  *reinterpret_cast<__half2*>(hi + i) = h;
  if (lo) *reinterpret_cast<__half2*>(lo + i) = __floats2half2_rn(a - __low2float(h), b - __high2float(h));
}

__global__ void __launch_bounds__(256) prefill_rmsnorm_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                              __half* __restrict__ xn, __half* __restrict__ xn_lo,
                                                              int dim, float eps) {
  __shared__ float red[8];
  const float* xr = x + (size_t)blockIdx.x * dim;
  float ss = 0.f;
  for (int i = threadIdx.x * 4; i < dim; i += blockDim.x * 4) {
    const float4 v = *reinterpret_cast<const float4*>(xr + i);
    ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) tot += red[i];
  const float scale = 1.0f / sqrtf(tot / (float)dim + eps);
  const size_t row = (size_t)blockIdx.x * dim;
  for (int i = threadIdx.x * 4; i < dim; i += blockDim.x * 4) {
    const float4 v = *reinterpret_cast<const float4*>(xr + i);
    const float4 g = *reinterpret_cast<const float4*>(w + i);
    store_hilo(xn, xn_lo, row + i, v.x * scale * g.x, v.y * scale * g.y);
    store_hilo(xn, xn_lo, row + i + 2, v.z * scale * g.z, v.w * scale * g.w);
  }
}

cudaError_t prefill_rmsnorm(const float* x, const float* w, __half* xn, __half* xn_lo, int T, int dim, float eps,
                            cudaStream_t s) {
  if (T <= 0 || dim % 4) return cudaErrorInvalidValue;
  prefill_rmsnorm_kernel<<<T, 256, 0, s>>>(x, w, xn, xn_lo, dim, eps);
  return cudaGetLastError();
}

// ------------------------------------------------------------------------ clip / RoPE / KV append
// One CTA per token; thread j handles the element pair (2j, 2j+1) of the [q; k; v] row.  The same
// arithmetic as the decode QKV epilogue (gemv.cu, kEpiQKV).
__global__ void __launch_bounds__(256) prefill_qkv_post_kernel(const float* __restrict__ qkv, int pos0, int q_rows,
                                                               int kv_rows, int hd, int rotary_dim, int msl, float clip,
                                                               const float* __restrict__ inv_freq, float* __restrict__ q_out,
                                                               __half* k_cache, __half* v_cache) {
  const int t = blockIdx.x, pos = pos0 + t;
  const int rows = q_rows + 2 * kv_rows;
  const float* row = qkv + (size_t)t * rows;
  for (int j = threadIdx.x; j < rows / 2; j += blockDim.x) {
    const int gr = 2 * j;
    float s0 = row[gr], s1 = row[gr + 1];
    s0 = s0 < -clip ? -clip : (s0 > clip ? clip : s0);
    s1 = s1 < -clip ? -clip : (s1 > clip ? clip : s1);
    if (gr < q_rows + kv_rows) {
      const int jh = (gr < q_rows ? gr : gr - q_rows) % hd;
      float fcr = 1.f, fci = 0.f;
      if (jh < rotary_dim) {
        const float val = (float)pos * inv_freq[jh >> 1];
        sincosf(val, &fci, &fcr);
      }
      const float r0 = s0 * fcr - s1 * fci;
      const float r1 = s0 * fci + s1 * fcr;
      if (gr < q_rows) {
        q_out[(size_t)t * q_rows + gr] = r0;
        q_out[(size_t)t * q_rows + gr + 1] = r1;
      } else {
        const int g = (gr - q_rows) / hd;
        *reinterpret_cast<__half2*>(k_cache + ((size_t)g * msl + pos) * hd + jh) = __floats2half2_rn(r0, r1);
      }
    } else {
      const int vr = gr - q_rows - kv_rows;
      const int g = vr / hd, jh = vr % hd;
      *reinterpret_cast<__half2*>(v_cache + ((size_t)g * msl + pos) * hd + jh) = __floats2half2_rn(s0, s1);
    }
  }
}

cudaError_t prefill_qkv_post(const float* qkv, int T, int pos0, int q_rows, int kv_rows, int head_dim, int rotary_dim,
                             int max_seq_len, float qkv_clip, const float* inv_freq, float* q_out, __half* k_cache,
                             __half* v_cache, cudaStream_t s) {
  if (T <= 0 || pos0 < 0 || pos0 + T > max_seq_len) return cudaErrorInvalidValue;
  prefill_qkv_post_kernel<<<T, 256, 0, s>>>(qkv, pos0, q_rows, kv_rows, head_dim, rotary_dim, max_seq_len, qkv_clip,
                                            inv_freq, q_out, k_cache, v_cache);
  return cudaGetLastError();
}

// ----------------------------------------------------------------------------- causal attention
// CTA = (block of QB queries, kv head g); 8 warps, each owning R = 16 (query, head) rows: QW = 16 / GQ
// queries x the GQ heads of the group, so every K/V tile staged in shared memory serves the GQ query
// heads of its kv head.  Per key tile of 64 slots a warp works on the tensor cores (mma.sync
// m16n8k16, fp32 accumulate), flash-attention style:
//   S[16 rows][64 keys] = Q . K^T     (q split into fp16 hi + lo parts: the products keep ~22 bits)
//   causal mask, online softmax in base 2 (running max / sum per row, rescaling O when the max grows)
//   O[16 rows][HD] += P . V           (p split the same way)
// The S accumulator fragments become the P operand fragments in registers (same row / column
// layout).  K and V rows are staged with a padded stride (an odd multiple of 16 bytes) so the eight
// rows one ldmatrix reads fall in different bank groups.
namespace {
constexpr int kPaRows = 16;
constexpr int kPaKeys = 64;
__host__ __device__ constexpr int pa_row_bytes(int hd) { return hd * 2 + 16; }
}  // namespace

template <int HD, int GQ>
__global__ void __launch_bounds__(256, 1)
    prefill_attention_kernel(const float* __restrict__ q, const __half* __restrict__ k_cache,
                             const __half* __restrict__ v_cache, __half* __restrict__ out, __half* __restrict__ out_lo,
                             int T, int pos0, int n_heads, int msl) {
  constexpr int QW = kPaRows / GQ;  // queries per warp
  constexpr int QB = 8 * QW;        // queries per CTA
  constexpr int KS = HD / 16;       // k-steps of S over head_dim
  constexpr int NT = HD / 8;        // n-tiles of O
  constexpr int RB = pa_row_bytes(HD);
  constexpr int CPR = HD / 8;       // 16-byte chunks per cache row
  extern __shared__ __align__(16) unsigned char smem[];
  // two buffers (double-buffered key tiles), each K [64][RB] then V [64][RB]
  constexpr uint32_t TB = 2u * kPaKeys * RB;
  const uint32_t sm_s = smem_u32(smem);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g4 = lane >> 2, c4 = lane & 3;
  const int nqb = (T + QB - 1) / QB;
  const int qb = nqb - 1 - (int)blockIdx.x;  // longest blocks first
  const int g = blockIdx.y;
  const int q0 = qb * QB;
  const int kend = pos0 + min(q0 + QB, T);  // keys [0, kend)
  const __half* kg = k_cache + (size_t)g * msl * HD;
  const __half* vg = v_cache + (size_t)g * msl * HD;
  const int q_dim = n_heads * HD;

  // This lane's two rows: half hf holds row g4 + 8 hf = qi * GQ + h -> query q0 + warp * QW + qi,
  // head g * GQ + h.
  int tq[2], qpos[2];
  const float* qrow[2];
#pragma unroll
  for (int hf = 0; hf < 2; ++hf) {
    const int r = g4 + 8 * hf;
    tq[hf] = q0 + warp * QW + r / GQ;
    qpos[hf] = pos0 + tq[hf];
    qrow[hf] = q + (size_t)(tq[hf] < T ? tq[hf] : 0) * q_dim + (size_t)(g * GQ + r % GQ) * HD;
  }
  // Q as A fragments, k-step kk: {row g4, row g4 + 8} x {dims 16 kk + 2 c4 (+1), + 8}, hi and lo
  uint32_t qa[KS][4], ql[KS][4];
#pragma unroll
  for (int kk = 0; kk < KS; ++kk)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int hf = i & 1, d = 16 * kk + 8 * (i >> 1) + 2 * c4;
      float2 x = make_float2(0.f, 0.f);
      if (tq[hf] < T) x = *reinterpret_cast<const float2*>(qrow[hf] + d);
      split_f16x2(x.x, x.y, qa[kk][i], ql[kk][i]);
    }

  // scores q.k / sqrt(head_dim) are kept in base 2: t = q.k * log2(e) / sqrt(head_dim), p = 2^(t - max)
  const float sl2 = 1.4426950408889634f / sqrtf((float)HD);
  float o[NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int i = 0; i < 4; ++i) o[nt][i] = 0.f;
  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};

  // key tile it -> buffer it & 1; slots past kend are zero-filled
  auto stage = [&](int it) {
    const int kb0 = it * kPaKeys;
    const uint32_t kbuf = sm_s + (uint32_t)(it & 1) * TB, vbuf = kbuf + kPaKeys * RB;
    for (int e = threadIdx.x; e < kPaKeys * CPR; e += blockDim.x) {
      const int kk = e / CPR, c = e % CPR;
      const bool in = kb0 + kk < kend;
      const size_t off = in ? (size_t)(kb0 + kk) * HD + c * 8 : 0;
      cp_async16(kbuf + kk * RB + c * 16, kg + off, in ? 16u : 0u);
      cp_async16(vbuf + kk * RB + c * 16, vg + off, in ? 16u : 0u);
    }
    cp_async_commit();
  };
  const int ntile = (kend + kPaKeys - 1) / kPaKeys;
  stage(0);
  for (int it = 0; it < ntile; ++it) {
    const int k0 = it * kPaKeys;
    if (it + 1 < ntile) {
      stage(it + 1);  // its buffer was released by the barrier at the end of iteration it - 1
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();  // every thread's copies of tile it have landed
    const uint32_t ks_s = sm_s + (uint32_t)(it & 1) * TB, vs_s = ks_s + kPaKeys * RB;

    // S = Q . K^T: n-tile nt = keys k0 + 8 nt .. + 7; ldmatrix x4 gives the B fragments of n-tiles
    // 2 np and 2 np + 1 (matrix lane / 8 = (keys +0 | +8) x (dims +0 | +8))
    float s[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int i = 0; i < 4; ++i) s[nt][i] = 0.f;
    {
      const int key = 8 * ((lane >> 3) >> 1) + (lane & 7), hi = (lane >> 3) & 1;
#pragma unroll
      for (int kk = 0; kk < KS; ++kk) {
        // the eight hi products first, then the eight lo ones: dependent mma are 8 apart
        uint32_t B[4][4];
#pragma unroll
        for (int np = 0; np < 4; ++np) ldsm_x4(B[np], ks_s + (16 * np + key) * RB + (2 * kk + hi) * 16);
#pragma unroll
        for (int np = 0; np < 4; ++np) {
          mma_16816(s[2 * np], qa[kk], B[np][0], B[np][1]);
          mma_16816(s[2 * np + 1], qa[kk], B[np][2], B[np][3]);
        }
#pragma unroll
        for (int np = 0; np < 4; ++np) {
          mma_16816(s[2 * np], ql[kk], B[np][0], B[np][1]);
          mma_16816(s[2 * np + 1], ql[kk], B[np][2], B[np][3]);
        }
      }
    }

    // causal mask, online softmax: lane holds keys k0 + 8 nt + 2 c4 + e of rows g4 (i = e) and
    // g4 + 8 (i = 2 + e); a row's four lanes (same g4) reduce with xor 1, 2
    float alpha[2];
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      float mx = -INFINITY;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int key = k0 + 8 * nt + 2 * c4 + e;
          float v = s[nt][2 * hf + e] * sl2;
          if (tq[hf] >= T || key > qpos[hf]) v = -INFINITY;
          s[nt][2 * hf + e] = v;
          mx = fmaxf(mx, v);
        }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float mn = fmaxf(m[hf], mx);
      alpha[hf] = 1.f;
      float ps = 0.f;
      if (mn != -INFINITY) {
        alpha[hf] = exp2f(m[hf] - mn);  // 0 while m[hf] is still -inf
#pragma unroll
        for (int nt = 0; nt < 8; ++nt)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const float v = s[nt][2 * hf + e];
            const float pv = v == -INFINITY ? 0.f : exp2f(v - mn);
            s[nt][2 * hf + e] = pv;
            ps += pv;
          }
        m[hf] = mn;
      } else {
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) s[nt][2 * hf] = s[nt][2 * hf + 1] = 0.f;
      }
      l[hf] = l[hf] * alpha[hf] + ps;  // this lane's share; the row's four lanes are summed at the end
    }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      o[nt][0] *= alpha[0];
      o[nt][1] *= alpha[0];
      o[nt][2] *= alpha[1];
      o[nt][3] *= alpha[1];
    }

    // O += P . V: k-step ks = keys 16 ks .. + 15; P's A fragment is S n-tiles 2 ks, 2 ks + 1;
    // ldmatrix.trans x4 gives the B fragments of output n-tiles 2 np, 2 np + 1 (matrix lane / 8 =
    // (keys +0 | +8) x (dims +0 | +8))
    {
      const int key = 8 * ((lane >> 3) & 1) + (lane & 7), hi = (lane >> 3) >> 1;
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        uint32_t ph[4], pl[4];
        split_f16x2(s[2 * ks][0], s[2 * ks][1], ph[0], pl[0]);
        split_f16x2(s[2 * ks][2], s[2 * ks][3], ph[1], pl[1]);
        split_f16x2(s[2 * ks + 1][0], s[2 * ks + 1][1], ph[2], pl[2]);
        split_f16x2(s[2 * ks + 1][2], s[2 * ks + 1][3], ph[3], pl[3]);
        // hi products for every output n-tile, then lo: dependent mma are NT apart
#pragma unroll
        for (int np = 0; np < NT / 2; ++np) {
          uint32_t B[4];
          ldsm_x4_trans(B, vs_s + (16 * ks + key) * RB + (2 * np + hi) * 16);
          mma_16816(o[2 * np], ph, B[0], B[1]);
          mma_16816(o[2 * np + 1], ph, B[2], B[3]);
        }
#pragma unroll
        for (int np = 0; np < NT / 2; ++np) {
          uint32_t B[4];
          ldsm_x4_trans(B, vs_s + (16 * ks + key) * RB + (2 * np + hi) * 16);
          mma_16816(o[2 * np], pl, B[0], B[1]);
          mma_16816(o[2 * np + 1], pl, B[2], B[3]);
        }
      }
    }
    __syncthreads();  // tile it's buffer is free for tile it + 2
  }

  // normalise and store: lane holds dims 8 nt + 2 c4 (+1) of rows g4 (i = 0, 1) and g4 + 8 (i = 2, 3)
#pragma unroll
  for (int hf = 0; hf < 2; ++hf) {
    float lt = l[hf];
    lt += __shfl_xor_sync(0xffffffffu, lt, 1);
    lt += __shfl_xor_sync(0xffffffffu, lt, 2);
    if (tq[hf] < T) {
      const int r = g4 + 8 * hf;
      const size_t dst = (size_t)tq[hf] * q_dim + (size_t)(g * GQ + r % GQ) * HD + 2 * c4;
      const float inv = 1.f / lt;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) store_hilo(out, out_lo, dst + 8 * nt, o[nt][2 * hf] * inv, o[nt][2 * hf + 1] * inv);
    }
  }
}

namespace {
template <int HD>
const void* pick_pa(int gq) {
  switch (gq) {
    case 1: return reinterpret_cast<const void*>(&prefill_attention_kernel<HD, 1>);
    case 2: return reinterpret_cast<const void*>(&prefill_attention_kernel<HD, 2>);
    case 4: return reinterpret_cast<const void*>(&prefill_attention_kernel<HD, 4>);
    case 8: return reinterpret_cast<const void*>(&prefill_attention_kernel<HD, 8>);
  }
  return nullptr;
}
}  // namespace

cudaError_t prefill_attention(const float* q, const __half* k_cache, const __half* v_cache, __half* out, __half* out_lo,
                              int T, int pos0, int n_heads, int n_kv_heads, int head_dim, int max_seq_len,
                              unsigned* status, cudaStream_t s) {
  if (T <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads || pos0 + T > max_seq_len) return cudaErrorInvalidValue;
  const int gq = n_heads / n_kv_heads;
  // 0: mma.sync kernel; 1: tcgen05 where supported (default); 2: tcgen05 with the V descriptor's
  // byte offsets swapped (a layout check)
  static const int mode = [] {
    const char* v = std::getenv("YB_PREFILL_ATTN");
    if (!v) return 1;
    if (!std::strcmp(v, "mma")) return 0;
    if (!std::strcmp(v, "tc-swap")) return 2;
    return 1;
  }();
  if (mode && prefill_attention_tc_supported(head_dim, gq))
    return prefill_attention_tc(q, k_cache, v_cache, out, out_lo, T, pos0, n_heads, n_kv_heads, max_seq_len, status,
                                mode == 2 ? 1 : 0, s);
  const void* fn = head_dim == 128 ? pick_pa<128>(gq) : head_dim == 64 ? pick_pa<64>(gq) : nullptr;
  if (!fn) return cudaErrorInvalidValue;
  const size_t smem = (size_t)4 * kPaKeys * pa_row_bytes(head_dim);
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const int qb = 8 * (kPaRows / gq);
  const dim3 grid((T + qb - 1) / qb, n_kv_heads);
  void* args[] = {&q, &k_cache, &v_cache, &out, &out_lo, &T, &pos0, &n_heads, &max_seq_len};
  return cudaLaunchKernel(fn, grid, dim3(256), args, smem, s);
}

}  // namespace yb
