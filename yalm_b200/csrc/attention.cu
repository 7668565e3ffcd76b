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
// Slice partial record: o[0..HD), m at HD, l at HD + 1, padded to a 16-byte multiple.
constexpr int attn_part_stride(int hd) { return hd + 4; }
constexpr int kAttnSub = 64;  // cache slots per staged sub-chunk (8 warps x 8 slots)

template <int HD, int GQ>
__global__ void __launch_bounds__(kAttnThreads) attn_decode_kernel(const AttnArgs a) {
  constexpr int DPL = HD / 32;                  // head dims per lane
  constexpr int NV = (8 * GQ < 32) ? 8 * GQ : 32;  // partial scores per reduce-scatter round
  constexpr int ROUNDS = (8 * GQ + 31) / 32;
  constexpr int PR = NV / GQ;                    // slots per round per warp
  constexpr int LOG_NV = (NV == 8) ? 3 : (NV == 16) ? 4 : 5;
  constexpr int SLOTS = 2;                       // sub-chunks per CTA (capacity 128 slots)
  constexpr int PS = attn_part_stride(HD);

  extern __shared__ __align__(128) unsigned char smem[];
  __half* Ks = reinterpret_cast<__half*>(smem);                         // [SLOTS][64][HD]
  __half* Vs = Ks + SLOTS * kAttnSub * HD;                              // [SLOTS][64][HD]
  const bool merge_smem = attn_merge_in_smem(HD, GQ, gridDim.x);
  float* S = reinterpret_cast<float*>(smem + attn_region_bytes(HD, GQ, gridDim.x));  // [2][GQ][64]
  uint64_t* bar = reinterpret_cast<uint64_t*>(S + 2 * GQ * kAttnSub);  // [SLOTS] stages, [SLOTS] merge
  __shared__ int s_last;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sidx = blockIdx.x, g = blockIdx.y;

  pdl_trigger();
  unsigned long long* const tr =
      a.trace ? a.trace + (size_t)blockIdx.y * gridDim.x * a.trace_stride : nullptr;  // row of this CTA
  if (threadIdx.x == 0) timeline_stamp(tr, a.trace_stride, 0);

  const int s_max = gridDim.x;
  // A cache of at most one CTA's capacity goes to slice 0 alone (no merge); longer ones split into
  // slices of at least one staged sub-chunk. Slice sidx of a cache of len slots covers [t0, t1) in
  // n_sub sub-chunks (0 = inactive).
  auto partition = [&](int len, int& t0_, int& t1_, int& nsub_, int& nact_) {
    int ch = (len + s_max - 1) / s_max;
    ch = ((ch + 15) / 16) * 16;
    if (len <= kAttnCapacity) ch = kAttnCapacity;
    else if (ch < kAttnSub) ch = kAttnSub;
    nact_ = (len + ch - 1) / ch;
    t0_ = sidx * ch;
    t1_ = min(len, t0_ + ch);
    nsub_ = t0_ < len ? (t1_ - t0_ + kAttnSub - 1) / kAttnSub : 0;
  };
  const __half* kg = a.k_cache + (size_t)g * a.max_seq_len * HD;
  const __half* vg = a.v_cache + (size_t)g * a.max_seq_len * HD;
  auto issue = [&](int c_begin, int c_end, int j) {
    const int c0 = c_begin + j * kAttnSub;
    const int cn = min(kAttnSub, c_end - c0);
    const unsigned bytes = (unsigned)cn * HD * 2u;
    mbar_arrive_expect_tx(&bar[j], 2u * bytes);
    bulk_g2s_nohint(Ks + (size_t)j * kAttnSub * HD, kg + (size_t)c0 * HD, bytes, &bar[j]);
    bulk_g2s_nohint(Vs + (size_t)j * kAttnSub * HD, vg + (size_t)c0 * HD, bytes, &bar[j]);
  };

  // Before the wait on the QKV kernel: stage the cache slots of this slice for the kv_len the step
  // state shows now (normally this step's, possibly the previous step's: it is only a hint).  All
  // slots but the one the QKV kernel is appending (and, past the context, the two re-rotated sink
  // keys) already hold their final values; those few rows are patched from global memory below.
  int h0, h1, hsub, hact;
  {
    int hlen = a.step ? *reinterpret_cast<const volatile int*>(&a.step->kv_len) : a.kv_len;
    hlen = hlen < 1 ? 1 : (hlen > a.max_seq_len ? a.max_seq_len : hlen);
    partition(hlen, h0, h1, hsub, hact);
  }
  if (threadIdx.x == 0) {
    for (int j = 0; j <= SLOTS; ++j) mbar_init(&bar[j], 1);
    mbar_fence_init();
    for (int j = 0; j < hsub; ++j) issue(h0, h1, j);
  }

  pdl_wait();  // q and the newest K/V slot come from the QKV kernel
  if (threadIdx.x == 0) timeline_stamp(tr, a.trace_stride, 1);

  const int kv_len = a.step ? a.step->kv_len : a.kv_len;
  const int kv_pos = a.step ? a.step->kv_pos : -1;
  const int kv_sink = a.step ? a.step->kv_sink : 0;
  int t0, t1, n_sub, n_act;
  partition(kv_len, t0, t1, n_sub, n_act);
  // the staged rows can be used when they cover the slice, apart from the appended slot
  const bool reuse = n_sub == hsub && t0 == h0 && (t1 <= h1 || (t1 == h1 + 1 && kv_pos == h1));
  if (n_sub == 0) {
    // inactive slice (not counted by the merge): let any staged copy land before leaving
    if (threadIdx.x == 0)
      for (int j = 0; j < hsub; ++j) mbar_wait(&bar[j], 0, a.status);
    return;
  }
  const int n = t1 - t0;
  // a sub-chunk whose stale staging had to be replaced completes its barrier's second phase
  if (!reuse && threadIdx.x == 0) {
    for (int j = 0; j < hsub; ++j) mbar_wait(&bar[j], 0, a.status);
    for (int j = 0; j < n_sub; ++j) issue(t0, t1, j);
  }

  // Rows this step's QKV kernel wrote after the staging was issued (src/infer.cpp:296-325): warp 0
  // loads the appended K/V slot, warp 1 the re-rotated sink keys, together with q below; they are
  // stored over the staged copies once their sub-chunk has landed.
  constexpr int CH = HD / 8;  // 16-byte chunks per row
  uint4 patch = make_uint4(0u, 0u, 0u, 0u);
  int patch_row = -1, patch_col = 0;
  bool patch_k = true;
  if (reuse && a.step) {
    if (warp == 0 && lane < 2 * CH && kv_pos >= t0 && kv_pos < t1) {
      patch_k = lane < CH;
      patch_col = lane % CH;
      patch_row = kv_pos;
    } else if (warp == 1 && lane < kv_sink * CH && lane / CH >= t0 && lane / CH < t1) {
      patch_row = lane / CH;
      patch_col = lane % CH;
    }
    if (patch_row >= 0)
      patch = __ldcg(reinterpret_cast<const uint4*>((patch_k ? kg : vg) + (size_t)patch_row * HD + patch_col * 8));
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
  // Scores of every staged slot (both sub-chunks) first, then one softmax over the slice and one
  // pass over V: the slice is at most 128 slots, so no running rescale is needed.
  // The sub-chunk loops stay rolled: this code runs once per CTA, so its instruction fetches miss
  // the instruction cache; a smaller body is faster than an unrolled one here.
  float sc[SLOTS][ROUNDS];
#pragma unroll 1
  for (int j = 0; j < SLOTS; ++j) {
#pragma unroll
    for (int r = 0; r < ROUNDS; ++r) sc[j][r] = -INFINITY;
    if (j < n_sub) {  // CTA-uniform
      if (!mbar_wait(&bar[j], (!reuse && j < hsub) ? 1 : 0, a.status)) ok = false;
      if (!__all_sync(0xffffffffu, ok)) ok = false;
      if (j == 0 && threadIdx.x == 0) timeline_stamp(tr, a.trace_stride, 2);
      const __half* Kj = Ks + (size_t)j * kAttnSub * HD;
      float* Sj = S + j * GQ * kAttnSub;
      const int cn = min(kAttnSub, n - j * kAttnSub);
      if (reuse && a.step) {
        const int c0 = t0 + j * kAttnSub;
        if ((kv_pos >= c0 && kv_pos < c0 + cn) || (kv_sink > 0 && c0 < kv_sink)) {  // CTA-uniform
          if (patch_row >= c0 && patch_row < c0 + cn)
            *reinterpret_cast<uint4*>((patch_k ? Ks : Vs) + ((size_t)j * kAttnSub + (patch_row - c0)) * HD + patch_col * 8) = patch;
          __syncthreads();
        }
      }
      // scores for this warp's 8 slots, GQ heads
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
        sc[j][r] = (p < cn) ? tot / rsq : -INFINITY;
        if ((lane & ((32 >> LOG_NV) - 1)) == 0) Sj[h * kAttnSub + p] = sc[j][r];
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) timeline_stamp(tr, a.trace_stride, 5);

  // softmax over the slice: every warp derives the same max from all staged scores
#pragma unroll
  for (int h = 0; h < GQ; ++h) {
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < SLOTS; ++j)
      if (j < n_sub) mx = fmaxf(mx, fmaxf(S[(j * GQ + h) * kAttnSub + lane], S[(j * GQ + h) * kAttnSub + lane + 32]));
    m_run[h] = warp_max(mx);
  }
#pragma unroll 1
  for (int j = 0; j < SLOTS; ++j) {
    if (j >= n_sub) break;
    const __half* Vj = Vs + (size_t)j * kAttnSub * HD;
    const int cn = min(kAttnSub, n - j * kAttnSub);
    // probabilities for the slots this lane scored, then broadcast per slot
    float pv[ROUNDS];
#pragma unroll
    for (int r = 0; r < ROUNDS; ++r) {
      const int idx = lane >> (5 - LOG_NV);
      const int h = idx % GQ;
      float mh = m_run[0];
#pragma unroll
      for (int hh = 0; hh < GQ; ++hh)
        if (hh == h) mh = m_run[hh];
      pv[r] = (sc[j][r] == -INFINITY) ? 0.f : expf(sc[j][r] - mh);
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

  if (threadIdx.x == 0) timeline_stamp(tr, a.trace_stride, 6);
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
      float* pp = a.part + ((size_t)hq * s_max + sidx) * PS;
      pp[d == HD ? HD + 1 : d] = s;  // o[0..HD), l at HD+1
      if (d == 0) pp[HD] = m_run[h];
    }
  }
  if (threadIdx.x == 0) timeline_stamp(tr, a.trace_stride, 3);
  if (single || !ok) {
    if (threadIdx.x == 0) timeline_stamp(tr, a.trace_stride, 4);
    return;
  }

  // last-arriving slice of this kv head merges all slices
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned prev = atomicAdd(&a.counters[g], 1u);
    s_last = (prev == (unsigned)(n_act - 1));
  }
  __syncthreads();
  if (!s_last) {
    if (threadIdx.x == 0) timeline_stamp(tr, a.trace_stride, 4);
    return;
  }
  __threadfence();
  __syncthreads();  // smem reuse: the combine buffer is no longer read
  if (merge_smem) {
    // Merge (log-sum-exp) in shared memory: one bulk copy per head brings every slice's
    // (o, m, l) record; slice weights exp(m_s - M) and the outputs are then formed from there.
    constexpr int PSm = attn_part_stride(HD);
    float* P = reinterpret_cast<float*>(smem);  // [GQ][n_act][PS]
    float* sm_w = P + (size_t)GQ * n_act * PSm;  // [GQ][n_act]
    float* sm_l = sm_w + GQ * n_act;             // [GQ] totals
    if (threadIdx.x == 0) {
      // the partials were written by other CTAs' generic stores, read here by the async proxy
      asm volatile("fence.proxy.async.global;" ::: "memory");
      const unsigned bytes = (unsigned)n_act * PSm * 4u;
      mbar_arrive_expect_tx(&bar[SLOTS], GQ * bytes);
      for (int h = 0; h < GQ; ++h)
        bulk_g2s_nohint(P + (size_t)h * n_act * PSm, a.part + (size_t)(g * GQ + h) * s_max * PSm, bytes, &bar[SLOTS]);
    }
    const bool landed = mbar_wait(&bar[SLOTS], 0, a.status);
    if (!__syncthreads_and(landed)) {  // timed out (status set): leave the counter ready
      if (threadIdx.x == 0) a.counters[g] = 0u;
      return;
    }
    if (warp < GQ) {
      const int h = warp;
      const float* ph = P + (size_t)h * n_act * PSm;
      float M = -INFINITY;
      for (int sl = lane; sl < n_act; sl += 32) M = fmaxf(M, ph[(size_t)sl * PSm + HD]);
      M = warp_max(M);
      float L = 0.f;
      for (int sl = lane; sl < n_act; sl += 32) {
        const float w = expf(ph[(size_t)sl * PSm + HD] - M);
        sm_w[h * n_act + sl] = w;
        L = fmaf(w, ph[(size_t)sl * PSm + HD + 1], L);
      }
      L = warp_sum(L);
      if (lane == 0) sm_l[h] = L;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < GQ * HD; e += kAttnThreads) {
      const int h = e / HD, d = e % HD;
      const float* ph = P + (size_t)h * n_act * PSm + d;
      const float* w = sm_w + h * n_act;
      float O = 0.f;
      for (int sl = 0; sl < n_act; ++sl) O = fmaf(w[sl], ph[(size_t)sl * PSm], O);
      a.out[(size_t)(g * GQ + h) * HD + d] = O / sm_l[h];
    }
  } else {
    // Merge (log-sum-exp): stage every slice's (m, l) for the GQ heads in shared memory, derive the
    // slice weights exp(m_s - M) once per (head, slice), then each output element sums its slices
    // with batches of independent loads (the partials are in L2).
    float* sm_w = reinterpret_cast<float*>(smem);  // [GQ][n_act] slice weights
    float* sm_l = sm_w + GQ * n_act;               // [GQ][n_act] slice sums, then [GQ] totals
    for (int e = threadIdx.x; e < GQ * n_act; e += kAttnThreads) {
      const int h = e / n_act, sl = e % n_act;
      const float* ps = a.part + ((size_t)(g * GQ + h) * s_max + sl) * PS;
      sm_w[e] = __ldcg(ps + HD);
      sm_l[e] = __ldcg(ps + HD + 1);
    }
    __syncthreads();
    if (warp < GQ) {
      const int h = warp;
      float M = -INFINITY;
      for (int sl = lane; sl < n_act; sl += 32) M = fmaxf(M, sm_w[h * n_act + sl]);
      M = warp_max(M);
      float L = 0.f;
      for (int sl = lane; sl < n_act; sl += 32) {
        const float w = expf(sm_w[h * n_act + sl] - M);
        sm_w[h * n_act + sl] = w;
        L = fmaf(w, sm_l[h * n_act + sl], L);
      }
      L = warp_sum(L);
      __syncwarp();
      if (lane == 0) sm_l[h * n_act] = L;  // slot 0 of the head's row now holds the total
    }
    __syncthreads();
    {
      // WPH warps per head, each summing every WPH-th slice over this lane's DPL dims with
      // independent vector loads, then combined through shared memory
      constexpr int WPH = 8 / GQ;
      const int h = warp % GQ, q0 = warp / GQ;
      const float* base = a.part + (size_t)(g * GQ + h) * s_max * PS + lane * DPL;
      const float* w = sm_w + h * n_act;
      float acc[DPL];
#pragma unroll
      for (int d = 0; d < DPL; ++d) acc[d] = 0.f;
      int sl = q0;
      for (; sl + 3 * WPH < n_act; sl += 4 * WPH) {
        float v[4][DPL];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const float* src = base + (size_t)(sl + u * WPH) * PS;
          if (DPL == 4) {
            const float4 t4 = __ldcg(reinterpret_cast<const float4*>(src));
            v[u][0] = t4.x; v[u][1 % DPL] = t4.y; v[u][2 % DPL] = t4.z; v[u][3 % DPL] = t4.w;
          } else {
            const float2 t2 = __ldcg(reinterpret_cast<const float2*>(src));
            v[u][0] = t2.x; v[u][1 % DPL] = t2.y;
          }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u)
#pragma unroll
          for (int d = 0; d < DPL; ++d) acc[d] = fmaf(w[sl + u * WPH], v[u][d], acc[d]);
      }
      for (; sl < n_act; sl += WPH) {
        const float* src = base + (size_t)sl * PS;
#pragma unroll
        for (int d = 0; d < DPL; ++d) acc[d] = fmaf(w[sl], __ldcg(src + d), acc[d]);
      }
      float* cmb = sm_l + GQ * n_act;  // [8 warps][HD]
#pragma unroll
      for (int d = 0; d < DPL; ++d) cmb[warp * HD + lane * DPL + d] = acc[d];
      __syncthreads();
      if (warp < GQ) {
        const float L = sm_l[warp * n_act];
#pragma unroll
        for (int d = 0; d < DPL; ++d) {
          float o = 0.f;
#pragma unroll
          for (int q = 0; q < WPH; ++q) o += cmb[(q * GQ + warp) * HD + lane * DPL + d];
          a.out[(size_t)(g * GQ + warp) * HD + lane * DPL + d] = o / L;
        }
      }
    }
  }
  if (threadIdx.x == 0) {
    a.counters[g] = 0u;  // ready for the next launch
    timeline_stamp(tr, a.trace_stride, 4);
  }
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
  const size_t kv = attn_stage_bytes(head_dim);  // K,V x 2 sub-chunk slots
  const size_t sc = (size_t)2 * gq * kAttnSub * 4;
  const size_t red = (size_t)8 * gq * (head_dim + 1) * 4;
  // the combine buffer and the merge reuse the K/V stage region (red <= kv for every instantiated
  // HD, GQ; the region grows to the merge records when they are larger and fit)
  p.smem = attn_region_bytes(head_dim, gq, p.s_max) + sc + 2 * 8 + 8;
  if (red > kv) return p;
  p.part_floats = (size_t)n_heads * p.s_max * attn_part_stride(head_dim);
  p.ok = p.smem <= 226 * 1024;
  return p;
}

cudaError_t attn_prepare(const AttnPlan& p) { return raise_smem_cap(p.fn); }

cudaError_t attn_launch(const AttnPlan& p, AttnArgs a, cudaStream_t stream, bool pdl) {
  return launch_kernel(p.fn, p.grid, dim3(kAttnThreads), p.smem, stream, pdl, &a);
}

}  // namespace yb
