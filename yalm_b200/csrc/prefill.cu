// Batched prefill kernels other than the GEMMs.  yalm prefills one token at a time
// (src/main.cpp:171-177); here the prompt goes through each layer as one [T][dim] activation
// matrix: RMSNorm rows -> QKV GEMM -> clip / RoPE / KV append -> causal attention -> wo GEMM
// (+ residual) -> RMSNorm rows -> gate/up GEMM (+ SwiGLU) -> w2 GEMM (+ residual).
#include "prefill.cuh"

#include <math.h>

namespace yb {

// ---------------------------------------------------------------------------------------- RMSNorm
__global__ void __launch_bounds__(256) prefill_rmsnorm_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                              __half* __restrict__ xn, int dim, float eps) {
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
  __half* o = xn + (size_t)blockIdx.x * dim;
  for (int i = threadIdx.x * 4; i < dim; i += blockDim.x * 4) {
    const float4 v = *reinterpret_cast<const float4*>(xr + i);
    const float4 g = *reinterpret_cast<const float4*>(w + i);
    *reinterpret_cast<__half2*>(o + i) = __floats2half2_rn(v.x * scale * g.x, v.y * scale * g.y);
    *reinterpret_cast<__half2*>(o + i + 2) = __floats2half2_rn(v.z * scale * g.z, v.w * scale * g.w);
  }
}

cudaError_t prefill_rmsnorm(const float* x, const float* w, __half* xn, int T, int dim, float eps, cudaStream_t s) {
  if (T <= 0 || dim % 4) return cudaErrorInvalidValue;
  prefill_rmsnorm_kernel<<<T, 256, 0, s>>>(x, w, xn, dim, eps);
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
// queries x the GQ heads of the group.  Key tiles of 64 slots are staged in shared memory (K rows
// padded to a 16-byte-odd stride so lanes reading different rows hit different banks); per tile a
// warp scores its 16 rows against 2 keys per lane, updates the running max / sum (online softmax),
// stages the probabilities and accumulates P.V with each lane owning head_dim / 32 output dims.
namespace {
constexpr int kPaRows = 16;
constexpr int kPaKeys = 64;
}  // namespace

template <int HD, int GQ>
__global__ void __launch_bounds__(256, 1)
    prefill_attention_kernel(const float* __restrict__ q, const __half* __restrict__ k_cache,
                             const __half* __restrict__ v_cache, __half* __restrict__ out, int T, int pos0,
                             int n_heads, int msl) {
  constexpr int QW = kPaRows / GQ;  // queries per warp
  constexpr int QB = 8 * QW;        // queries per CTA
  constexpr int DPL = HD / 32;      // output dims per lane
  constexpr int KS = HD + 8;        // padded K row (halves): 16-byte stride odd
  extern __shared__ __align__(16) unsigned char smem[];
  float* Qs = reinterpret_cast<float*>(smem);                      // [8][16][HD]
  float* Ps = Qs + 8 * kPaRows * HD;                               // [8][16][64]
  __half* Ks = reinterpret_cast<__half*>(Ps + 8 * kPaRows * kPaKeys);  // [64][KS]
  __half* Vs = Ks + kPaKeys * KS;                                  // [64][HD]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nqb = (T + QB - 1) / QB;
  const int qb = nqb - 1 - (int)blockIdx.x;  // longest blocks first
  const int g = blockIdx.y;
  const int q0 = qb * QB;
  const int kend = pos0 + min(q0 + QB, T);  // keys [0, kend)
  const __half* kg = k_cache + (size_t)g * msl * HD;
  const __half* vg = v_cache + (size_t)g * msl * HD;
  const int q_dim = n_heads * HD;

  // this warp's rows: r = qi * GQ + h -> query q0 + warp * QW + qi, head g * GQ + h
  float* Qw = Qs + (size_t)warp * kPaRows * HD;
  for (int e = lane; e < kPaRows * HD; e += 32) {
    const int r = e / HD, d = e % HD;
    const int t = q0 + warp * QW + r / GQ;
    Qw[e] = t < T ? q[(size_t)t * q_dim + (size_t)(g * GQ + r % GQ) * HD + d] : 0.f;
  }
  const float rsq = sqrtf((float)HD);  // scores are q.k / sqrt(head_dim), as in the decode kernel
  float m[kPaRows], lsum[kPaRows], o[kPaRows][DPL];
#pragma unroll
  for (int r = 0; r < kPaRows; ++r) {
    m[r] = -INFINITY;
    lsum[r] = 0.f;
#pragma unroll
    for (int d = 0; d < DPL; ++d) o[r][d] = 0.f;
  }
  float* Pw = Ps + (size_t)warp * kPaRows * kPaKeys;

  for (int k0 = 0; k0 < kend; k0 += kPaKeys) {
    __syncthreads();  // the previous tile is no longer read
    for (int e = threadIdx.x; e < kPaKeys * (HD / 8); e += blockDim.x) {
      const int kk = e / (HD / 8), c = e % (HD / 8);
      uint4 kv = make_uint4(0u, 0u, 0u, 0u), vv = kv;
      if (k0 + kk < kend) {
        kv = *reinterpret_cast<const uint4*>(kg + (size_t)(k0 + kk) * HD + c * 8);
        vv = *reinterpret_cast<const uint4*>(vg + (size_t)(k0 + kk) * HD + c * 8);
      }
      *reinterpret_cast<uint4*>(Ks + kk * KS + c * 8) = kv;
      *reinterpret_cast<uint4*>(Vs + kk * HD + c * 8) = vv;
    }
    __syncthreads();
    // scores: rows x keys (k0 + lane, k0 + lane + 32)
    float sc[kPaRows][2];
#pragma unroll
    for (int r = 0; r < kPaRows; ++r) sc[r][0] = sc[r][1] = 0.f;
    for (int c = 0; c < HD / 8; ++c) {
      float kf[2][8];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const uint4 raw = *reinterpret_cast<const uint4*>(Ks + (lane + 32 * j) * KS + c * 8);
        const __half2* h2 = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = __half22float2(h2[i]);
          kf[j][2 * i] = f.x;
          kf[j][2 * i + 1] = f.y;
        }
      }
#pragma unroll
      for (int r = 0; r < kPaRows; ++r) {
        const float4 qa = *reinterpret_cast<const float4*>(Qw + r * HD + c * 8);
        const float4 qb4 = *reinterpret_cast<const float4*>(Qw + r * HD + c * 8 + 4);
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          float acc = sc[r][j];
          acc = fmaf(qa.x, kf[j][0], acc);
          acc = fmaf(qa.y, kf[j][1], acc);
          acc = fmaf(qa.z, kf[j][2], acc);
          acc = fmaf(qa.w, kf[j][3], acc);
          acc = fmaf(qb4.x, kf[j][4], acc);
          acc = fmaf(qb4.y, kf[j][5], acc);
          acc = fmaf(qb4.z, kf[j][6], acc);
          acc = fmaf(qb4.w, kf[j][7], acc);
          sc[r][j] = acc;
        }
      }
    }
    // causal mask, online softmax, probabilities to shared memory
#pragma unroll
    for (int r = 0; r < kPaRows; ++r) {
      const int t = q0 + warp * QW + r / GQ;
      const int qp = pos0 + t;
      float s0 = sc[r][0] / rsq, s1 = sc[r][1] / rsq;
      if (t >= T || k0 + lane > qp) s0 = -INFINITY;
      if (t >= T || k0 + lane + 32 > qp) s1 = -INFINITY;
      const float mx = warp_max(fmaxf(s0, s1));
      const float mn = fmaxf(m[r], mx);
      float p0 = 0.f, p1 = 0.f, alpha = 1.f;
      if (mn != -INFINITY) {
        alpha = expf(m[r] - mn);  // 0 while m[r] is still -inf
        p0 = s0 == -INFINITY ? 0.f : expf(s0 - mn);
        p1 = s1 == -INFINITY ? 0.f : expf(s1 - mn);
        m[r] = mn;
      }
      lsum[r] = lsum[r] * alpha + p0 + p1;
#pragma unroll
      for (int d = 0; d < DPL; ++d) o[r][d] *= alpha;
      Pw[r * kPaKeys + lane] = p0;
      Pw[r * kPaKeys + lane + 32] = p1;
    }
    __syncwarp();
    // o += P . V over the tile's keys
    const int nk = min(kPaKeys, kend - k0);
    for (int kk = 0; kk < nk; kk += 4) {
      float vf[4][DPL];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (DPL == 4) {
          const uint2 raw = *reinterpret_cast<const uint2*>(Vs + (kk + u) * HD + lane * 4);
          const float2 a0 = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
          const float2 a1 = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
          vf[u][0] = a0.x; vf[u][1 % DPL] = a0.y; vf[u][2 % DPL] = a1.x; vf[u][3 % DPL] = a1.y;
        } else {
          const float2 a0 = __half22float2(*reinterpret_cast<const __half2*>(Vs + (kk + u) * HD + lane * 2));
          vf[u][0] = a0.x; vf[u][1 % DPL] = a0.y;
        }
      }
#pragma unroll
      for (int r = 0; r < kPaRows; ++r) {
        const float4 pp = *reinterpret_cast<const float4*>(Pw + r * kPaKeys + kk);
#pragma unroll
        for (int d = 0; d < DPL; ++d) {
          float acc = o[r][d];
          acc = fmaf(pp.x, vf[0][d], acc);
          acc = fmaf(pp.y, vf[1][d], acc);
          acc = fmaf(pp.z, vf[2][d], acc);
          acc = fmaf(pp.w, vf[3][d], acc);
          o[r][d] = acc;
        }
      }
    }
    __syncwarp();  // Pw is rewritten by the next tile
  }
  // normalise and store
#pragma unroll
  for (int r = 0; r < kPaRows; ++r) {
    const int t = q0 + warp * QW + r / GQ;
    const float l = warp_sum(lsum[r]);
    if (t < T) {
      __half* dst = out + (size_t)t * q_dim + (size_t)(g * GQ + r % GQ) * HD + lane * DPL;
#pragma unroll
      for (int d = 0; d < DPL; ++d) dst[d] = __float2half_rn(o[r][d] / l);
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

cudaError_t prefill_attention(const float* q, const __half* k_cache, const __half* v_cache, __half* out, int T, int pos0,
                              int n_heads, int n_kv_heads, int head_dim, int max_seq_len, cudaStream_t s) {
  if (T <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads || pos0 + T > max_seq_len) return cudaErrorInvalidValue;
  const int gq = n_heads / n_kv_heads;
  const void* fn = head_dim == 128 ? pick_pa<128>(gq) : head_dim == 64 ? pick_pa<64>(gq) : nullptr;
  if (!fn) return cudaErrorInvalidValue;
  const size_t smem = (size_t)8 * kPaRows * head_dim * 4 + (size_t)8 * kPaRows * kPaKeys * 4 +
                      (size_t)kPaKeys * (head_dim + 8) * 2 + (size_t)kPaKeys * head_dim * 2;
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const int qb = 8 * (kPaRows / gq);
  const dim3 grid((T + qb - 1) / qb, n_kv_heads);
  void* args[] = {&q, &k_cache, &v_cache, &out, &T, &pos0, &n_heads, &max_seq_len};
  return cudaLaunchKernel(fn, grid, dim3(256), args, smem, s);
}

}  // namespace yb
