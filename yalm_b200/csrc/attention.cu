// Split-K GQA decode attention over the head-major fp16 KV cache.
//
// yalm computes, per query head h with kv group g = h / (n_heads / n_kv_heads):
//   s_t = q_h . k_t / sqrt(head_dim),  p = softmax(s[0..kv_len)),  out_h = sum_t p_t v_t
// (src/infer.cpp:218-250; the CUDA kernel attn_fused, src/infer.cu:625-667, runs one CTA per q head
// and reads each K/V head once per q head).  Here one CTA serves all GQ query heads of a kv head for
// one slice of cache slots, so K/V bytes cross HBM once per kv head.  Slices are staged into shared
// memory with 1-D TMA (K and V rows are contiguous [slot][head_dim]); each CTA keeps a running
// max / sum / output per head (online softmax), writes (m, l, o) for its slice, and the last CTA of
// a kv head to finish merges the slices with a log-sum-exp rescale and writes the head outputs.
#include "attention.cuh"
#include "launch.h"

#include <math.h>

namespace yb {

constexpr int kAttnThreads = 256;
constexpr int kAttnSub = 64;  // cache slots per staged sub-chunk (8 warps x 8 slots)

template <int HD, int GQ>
__global__ void __launch_bounds__(kAttnThreads) attn_decode_kernel(const AttnArgs a) {
  constexpr int DPL = HD / 32;                  // head dims per lane
  constexpr int NV = (8 * GQ < 32) ? 8 * GQ : 32;  // partial scores per reduce-scatter round
  constexpr int ROUNDS = (8 * GQ + 31) / 32;
  constexpr int PR = NV / GQ;                    // slots per round per warp
  constexpr int LOG_NV = (NV == 8) ? 3 : (NV == 16) ? 4 : 5;
  constexpr int SLOTS = 2;                       // sub-chunks per CTA (capacity 128 slots)

  extern __shared__ __align__(128) unsigned char smem[];
  __half* Ks = reinterpret_cast<__half*>(smem);                         // [SLOTS][64][HD]
  __half* Vs = Ks + SLOTS * kAttnSub * HD;                              // [SLOTS][64][HD]
  float* S = reinterpret_cast<float*>(Vs + SLOTS * kAttnSub * HD);       // [2][GQ][64]
  uint64_t* bar = reinterpret_cast<uint64_t*>(S + 2 * GQ * kAttnSub);    // [SLOTS]
  __shared__ int s_last;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sidx = blockIdx.x, g = blockIdx.y;

  pdl_trigger();
  pdl_wait();  // q and the newest K/V slot come from the QKV kernel

  const int kv_len = a.step ? a.step->kv_len : a.kv_len;
  const int s_max = gridDim.x;
  // slices of at least one staged sub-chunk: short contexts need no merge at all
  int chunk = (kv_len + s_max - 1) / s_max;
  chunk = ((chunk + 15) / 16) * 16;
  if (chunk < kAttnSub) chunk = kAttnSub;
  const int n_act = (kv_len + chunk - 1) / chunk;
  const int t0 = sidx * chunk;
  if (t0 >= kv_len) return;  // inactive slice: not counted by the merge
  const int t1 = min(kv_len, t0 + chunk);
  const int n = t1 - t0;
  const int n_sub = (n + kAttnSub - 1) / kAttnSub;

  const __half* kg = a.k_cache + (size_t)g * a.max_seq_len * HD;
  const __half* vg = a.v_cache + (size_t)g * a.max_seq_len * HD;
  if (threadIdx.x == 0) {
    for (int j = 0; j < SLOTS; ++j) mbar_init(&bar[j], 1);
    mbar_fence_init();
    for (int j = 0; j < n_sub; ++j) {
      const int c0 = t0 + j * kAttnSub;
      const int cn = min(kAttnSub, t1 - c0);
      const unsigned bytes = (unsigned)cn * HD * 2u;
      mbar_arrive_expect_tx(&bar[j], 2u * bytes);
      bulk_g2s_nohint(Ks + (size_t)j * kAttnSub * HD, kg + (size_t)c0 * HD, bytes, &bar[j]);
      bulk_g2s_nohint(Vs + (size_t)j * kAttnSub * HD, vg + (size_t)c0 * HD, bytes, &bar[j]);
    }
  }

  // q for the GQ heads of this kv group, this lane's DPL dims
  float qr[GQ][DPL];
#pragma unroll
  for (int h = 0; h < GQ; ++h)
#pragma unroll
    for (int d = 0; d < DPL; ++d) qr[h][d] = a.q[(size_t)(g * GQ + h) * HD + lane * DPL + d];
  const float rsq = sqrtf((float)HD);

  float m_run[GQ], l_w[GQ], o_w[GQ][DPL];
#pragma unroll
  for (int h = 0; h < GQ; ++h) {
    m_run[h] = -INFINITY;
    l_w[h] = 0.f;
#pragma unroll
    for (int d = 0; d < DPL; ++d) o_w[h][d] = 0.f;
  }
  __syncthreads();  // barrier init visible before anyone waits

  bool ok = true;
  for (int j = 0; j < n_sub; ++j) {
    if (!mbar_wait(&bar[j], 0, a.status)) ok = false;
    if (!__all_sync(0xffffffffu, ok)) ok = false;
    const __half* Kj = Ks + (size_t)j * kAttnSub * HD;
    const __half* Vj = Vs + (size_t)j * kAttnSub * HD;
    float* Sj = S + (j & 1) * GQ * kAttnSub;
    const int cn = min(kAttnSub, n - j * kAttnSub);

    // scores for this warp's 8 slots, GQ heads
    float sc[ROUNDS];
#pragma unroll
    for (int r = 0; r < ROUNDS; ++r) {
      float part[NV];
#pragma unroll
      for (int i = 0; i < PR; ++i) {
        const int p = warp * 8 + r * PR + i;
        float kf[DPL];
        if (p < cn) {
          if (DPL == 4) {
            uint2 raw = *reinterpret_cast<const uint2*>(Kj + (size_t)p * HD + lane * 4);
            float2 a0 = __half22float2(*reinterpret_cast<__half2*>(&raw.x));
            float2 a1 = __half22float2(*reinterpret_cast<__half2*>(&raw.y));
            kf[0] = a0.x; kf[1 % DPL] = a0.y; kf[2 % DPL] = a1.x; kf[3 % DPL] = a1.y;
          } else {
            float2 a0 = __half22float2(*reinterpret_cast<const __half2*>(Kj + (size_t)p * HD + lane * 2));
            kf[0] = a0.x; kf[1 % DPL] = a0.y;
          }
        } else {
#pragma unroll
          for (int d = 0; d < DPL; ++d) kf[d] = 0.f;
        }
#pragma unroll
        for (int h = 0; h < GQ; ++h) {
          float acc = 0.f;
#pragma unroll
          for (int d = 0; d < DPL; ++d) acc = fmaf(qr[h][d], kf[d], acc);
          part[i * GQ + h] = acc;
        }
      }
      const float tot = warp_reduce_scatter<NV>(part, lane);
      const int idx = lane >> (5 - LOG_NV);
      const int p = warp * 8 + r * PR + idx / GQ;
      const int h = idx % GQ;
      sc[r] = (p < cn) ? tot / rsq : -INFINITY;
      if ((lane & ((32 >> LOG_NV) - 1)) == 0) Sj[h * kAttnSub + p] = sc[r];
    }
    __syncthreads();

    // online softmax: every warp derives the same running max from all 64 scores
    float m_new[GQ], alpha[GQ];
#pragma unroll
    for (int h = 0; h < GQ; ++h) {
      float mx = fmaxf(Sj[h * kAttnSub + lane], Sj[h * kAttnSub + lane + 32]);
      mx = warp_max(mx);
      m_new[h] = fmaxf(m_run[h], mx);
      alpha[h] = expf(m_run[h] - m_new[h]);
      m_run[h] = m_new[h];
      l_w[h] *= alpha[h];
#pragma unroll
      for (int d = 0; d < DPL; ++d) o_w[h][d] *= alpha[h];
    }
    // probabilities for the slots this lane scored, then broadcast per slot
    float pv[ROUNDS];
#pragma unroll
    for (int r = 0; r < ROUNDS; ++r) {
      const int idx = lane >> (5 - LOG_NV);
      const int h = idx % GQ;
      float mh = m_new[0];
#pragma unroll
      for (int hh = 0; hh < GQ; ++hh)
        if (hh == h) mh = m_new[hh];
      pv[r] = (sc[r] == -INFINITY) ? 0.f : expf(sc[r] - mh);
    }
#pragma unroll
    for (int r = 0; r < ROUNDS; ++r) {
#pragma unroll
      for (int i = 0; i < PR; ++i) {
        const int p = warp * 8 + r * PR + i;
        float vf[DPL];
        const bool valid = p < cn;
        if (valid) {
          if (DPL == 4) {
            uint2 raw = *reinterpret_cast<const uint2*>(Vj + (size_t)p * HD + lane * 4);
            float2 a0 = __half22float2(*reinterpret_cast<__half2*>(&raw.x));
            float2 a1 = __half22float2(*reinterpret_cast<__half2*>(&raw.y));
            vf[0] = a0.x; vf[1 % DPL] = a0.y; vf[2 % DPL] = a1.x; vf[3 % DPL] = a1.y;
          } else {
            float2 a0 = __half22float2(*reinterpret_cast<const __half2*>(Vj + (size_t)p * HD + lane * 2));
            vf[0] = a0.x; vf[1 % DPL] = a0.y;
          }
        }
#pragma unroll
        for (int h = 0; h < GQ; ++h) {
          const float ph = __shfl_sync(0xffffffffu, pv[r], ((i * GQ + h) << (5 - LOG_NV)));
          if (valid) {
            l_w[h] += ph;
#pragma unroll
            for (int d = 0; d < DPL; ++d) o_w[h][d] = fmaf(ph, vf[d], o_w[h][d]);
          }
        }
      }
    }
  }

  // combine the 8 warps (identical running max) through shared memory reused from the K stage
  __syncthreads();
  float* red = reinterpret_cast<float*>(smem);  // [8][GQ][HD + 1]
  constexpr int RS = HD + 1;
#pragma unroll
  for (int h = 0; h < GQ; ++h) {
#pragma unroll
    for (int d = 0; d < DPL; ++d) red[(warp * GQ + h) * RS + lane * DPL + d] = o_w[h][d];
    if (lane == 0) red[(warp * GQ + h) * RS + HD] = l_w[h];
  }
  __syncthreads();
  const bool single = (n_act == 1);
  for (int e = threadIdx.x; e < GQ * (HD + 1); e += kAttnThreads) {
    const int h = e / (HD + 1), d = e % (HD + 1);
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) s += red[(w * GQ + h) * RS + d];
    const int hq = g * GQ + h;
    if (single) {
      if (d < HD) {
        float l = 0.f;
#pragma unroll
        for (int w = 0; w < 8; ++w) l += red[(w * GQ + h) * RS + HD];
        a.out[(size_t)hq * HD + d] = s / l;
      }
    } else {
      float* pp = a.part + ((size_t)hq * s_max + sidx) * (HD + 2);
      pp[d == HD ? HD + 1 : d] = s;  // o[0..HD), l at HD+1
      if (d == 0) pp[HD] = m_run[h];
    }
  }
  if (single || !ok) return;

  // last-arriving slice of this kv head merges all slices
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned prev = atomicAdd(&a.counters[g], 1u);
    s_last = (prev == (unsigned)(n_act - 1));
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int e = threadIdx.x; e < GQ * HD; e += kAttnThreads) {
    const int h = e / HD, d = e % HD;
    const int hq = g * GQ + h;
    const float* base = a.part + (size_t)hq * s_max * (HD + 2);
    float M = -INFINITY;
    for (int s = 0; s < n_act; ++s) M = fmaxf(M, __ldcg(base + (size_t)s * (HD + 2) + HD));
    float O = 0.f, L = 0.f;
    for (int s = 0; s < n_act; ++s) {
      const float* ps = base + (size_t)s * (HD + 2);
      const float wgt = expf(__ldcg(ps + HD) - M);
      O = fmaf(wgt, __ldcg(ps + d), O);
      L = fmaf(wgt, __ldcg(ps + HD + 1), L);
    }
    a.out[(size_t)hq * HD + d] = O / L;
  }
  if (threadIdx.x == 0) a.counters[g] = 0u;  // ready for the next launch
}

// ---------------------------------------------------------------------------------- host side
namespace {
template <int HD>
const void* pick_gq(int gq) {
  switch (gq) {
    case 1: return reinterpret_cast<const void*>(&attn_decode_kernel<HD, 1>);
    case 2: return reinterpret_cast<const void*>(&attn_decode_kernel<HD, 2>);
    case 4: return reinterpret_cast<const void*>(&attn_decode_kernel<HD, 4>);
    case 8: return reinterpret_cast<const void*>(&attn_decode_kernel<HD, 8>);
  }
  return nullptr;
}
}  // namespace

AttnPlan attn_plan(int n_heads, int n_kv_heads, int head_dim, int max_seq_len) {
  AttnPlan p{};
  p.ok = false;
  if (n_kv_heads <= 0 || n_heads % n_kv_heads) return p;
  const int gq = n_heads / n_kv_heads;
  if (head_dim == 128) p.fn = pick_gq<128>(gq);
  else if (head_dim == 64) p.fn = pick_gq<64>(gq);
  else p.fn = nullptr;
  if (!p.fn) return p;
  p.s_max = (max_seq_len + kAttnCapacity - 1) / kAttnCapacity;
  p.grid = dim3(p.s_max, n_kv_heads);
  const size_t kv = (size_t)2 * 2 * kAttnSub * head_dim * 2;     // K,V x 2 slots
  const size_t sc = (size_t)2 * gq * kAttnSub * 4;
  const size_t red = (size_t)8 * gq * (head_dim + 1) * 4;
  // the combine buffer reuses the K/V stage (red <= kv for every instantiated HD, GQ)
  p.smem = kv + sc + 2 * 8;
  if (red > kv) return p;
  p.part_floats = (size_t)n_heads * p.s_max * (head_dim + 2);
  p.ok = p.smem <= 226 * 1024;
  return p;
}

cudaError_t attn_prepare(const AttnPlan& p) { return raise_smem_cap(p.fn); }

cudaError_t attn_launch(const AttnPlan& p, AttnArgs a, cudaStream_t stream, bool pdl) {
  return launch_kernel(p.fn, p.grid, dim3(kAttnThreads), p.smem, stream, pdl, &a);
}

}  // namespace yb
