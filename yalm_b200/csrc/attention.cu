// Split-K GQA decode attention over the head-major fp16 KV cache.
//
// yalm computes, per query head h with kv group g = h / (n_heads / n_kv_heads):
//   s_t = q_h . k_t / sqrt(head_dim),  p = softmax(s[0..kv_len)),  out_h = sum_t p_t v_t
// (src/infer.cpp:218-250; the CUDA kernel attn_fused, src/infer.cu:625-667, runs one CTA per q head
// and reads each K/V head once per q head).  Here one CTA serves all GQ query heads of a kv head for
// one slice of at most 128 cache slots, so K/V bytes cross HBM once per kv head:
//
//   * after the wait on the QKV kernel (whose producers have already warmed L2 with this layer's
//     K/V rows) the slice's K and V rows are copied to shared memory with cp.async, rows padded to
//     an odd multiple of 16 bytes so one ldmatrix touches eight bank groups;
//   * each of the 8 warps takes 16 slots and works on the tensor cores (mma.sync m16n8k16, fp32
//     accumulate): S^T[16 slots][8 heads] = K . Q^T, a softmax over its 16 slots per head, then
//     O^T[head_dim][8 heads] = V^T . P^T.  q and p are fp32 values split into an fp16 value and its
//     fp16 remainder (two mma passes), so the products keep about 22 bits, as the fp32 loops do;
//   * the 8 warps' (max, sum, o) are combined in shared memory; a slice of a longer cache writes its
//     (m, l, o) record and the last CTA of a kv head to finish merges the slices with a log-sum-exp
//     rescale and writes the head outputs.
//
// The work is a few hundred mma per CTA: the kernel is bound by the K/V read and by latency, and
// the tensor cores serve to keep the instruction count (and so the latency) small.
#include "attention.cuh"
#include "launch.h"

#include <math.h>

namespace yb {

constexpr int kAttnThreads = 256;
// Slice partial record: o[0..HD), m at HD, l at HD + 1, padded to a 16-byte multiple.
constexpr int attn_part_stride(int hd) { return hd + 4; }
constexpr int kAttnSub = 64;  // minimum slice of a cache longer than one CTA's capacity

// One warp's group of 16 staged slots (rows r0 .. r0 + 15 of the K rows at shared address kb and
// the V rows at vb, RB bytes apart; my_n of them valid): scores, softmax and output on the tensor
// cores, then the group's (o, m, l) per head into the combine buffer (rw: [GQ][HD + 4], rm, rl:
// [GQ]).  Fragment layouts: see mma_16816 in common.cuh.
template <int HD, int GQ, int RB>
__device__ __forceinline__ void attn_group(uint32_t kb, uint32_t vb, int r0, int my_n, int lane,
                                           const uint32_t (&qh)[HD / 16][2], const uint32_t (&ql)[HD / 16][2],
                                           float* rw, float* rm, float* rl) {
  constexpr int KS = HD / 16;
  constexpr int RS = HD + 4;
  const int gh = lane >> 2, c4 = lane & 3;
  // S^T = K . Q^T over HD in KS k-steps; four independent accumulators (hi / lo x even / odd step)
  float acc[4][4];
#pragma unroll
  for (int u = 0; u < 4; ++u)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[u][i] = 0.f;
  {
    // ldmatrix rows: matrix lane / 8 = (slots 0-7 | 8-15) x (dims +0 | +8) in A-fragment order
    const int lr = r0 + 8 * ((lane >> 3) & 1) + (lane & 7);
    const int lc = lane >> 4;
#pragma unroll
    for (int kk = 0; kk < KS; ++kk) {
      uint32_t A[4];
      ldsm_x4(A, kb + lr * RB + (2 * kk + lc) * 16);
      mma_16816(acc[(kk & 1) * 2], A, qh[kk][0], qh[kk][1]);
      mma_16816(acc[(kk & 1) * 2 + 1], A, ql[kk][0], ql[kk][1]);
    }
  }
  // lane holds slots gh (i = 0, 1) and gh + 8 (i = 2, 3) of heads 2 c4 + (i & 1)
  const float scale = 1.0f / sqrtf((float)HD);
  const bool v0 = gh < my_n, v1 = gh + 8 < my_n;
  float s[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float t = ((acc[0][i] + acc[2][i]) + (acc[1][i] + acc[3][i])) * scale;
    s[i] = (i < 2 ? v0 : v1) ? t : -INFINITY;
  }
  float m0 = fmaxf(s[0], s[2]), m1 = fmaxf(s[1], s[3]);
#pragma unroll
  for (int off = 4; off < 32; off <<= 1) {
    m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, off));
    m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, off));
  }
  // slot 0 of the group is always valid, so m0, m1 are finite
  const float p0 = v0 ? expf(s[0] - m0) : 0.f, p1 = v0 ? expf(s[1] - m1) : 0.f;
  const float p2 = v1 ? expf(s[2] - m0) : 0.f, p3 = v1 ? expf(s[3] - m1) : 0.f;
  float l0 = p0 + p2, l1 = p1 + p3;
#pragma unroll
  for (int off = 4; off < 32; off <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, off);
    l1 += __shfl_xor_sync(0xffffffffu, l1, off);
  }

  // P^T as the B operand of the output mma: the lane's (slot, head pair) rows transposed to
  // (head, slot pair) by movmatrix, hi and lo parts
  uint32_t x0h, x0l, x1h, x1l;
  split_f16x2(p0, p1, x0h, x0l);
  split_f16x2(p2, p3, x1h, x1l);
  const uint32_t bh0 = movm_trans(x0h), bh1 = movm_trans(x1h);
  const uint32_t bl0 = movm_trans(x0l), bl1 = movm_trans(x1l);

  // O^T = V^T . P^T: m-tile mt covers dims 16 mt .. 16 mt + 15
  float o[KS][4];
  {
    // ldmatrix.trans rows: matrix lane / 8 = (slots 0-7 | 8-15) x (dims +0 | +8), A order
    const int vr = r0 + 8 * (lane >> 4) + (lane & 7);
    const int vc = (lane >> 3) & 1;
#pragma unroll
    for (int mt = 0; mt < KS; ++mt) {
#pragma unroll
      for (int i = 0; i < 4; ++i) o[mt][i] = 0.f;
      uint32_t A[4];
      ldsm_x4_trans(A, vb + vr * RB + (2 * mt + vc) * 16);
      mma_16816(o[mt], A, bh0, bh1);
      mma_16816(o[mt], A, bl0, bl1);
    }
  }

  // lane holds dims 16 mt + gh (+8) of heads 2 c4, 2 c4 + 1
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const int h = 2 * c4 + e;
    if (h < GQ) {
      float* r = rw + h * RS;
#pragma unroll
      for (int mt = 0; mt < KS; ++mt) {
        r[16 * mt + gh] = o[mt][e];
        r[16 * mt + gh + 8] = o[mt][2 + e];
      }
      if (gh == 0) {
        rm[h] = e ? m1 : m0;
        rl[h] = e ? l1 : l0;
      }
    }
  }
}

template <int HD, int GQ>
__global__ void __launch_bounds__(kAttnThreads, 2) attn_decode_kernel(const AttnArgs a) {
  static_assert(GQ >= 1 && GQ <= 8, "the score mma has 8 head columns");
  constexpr int KS = HD / 16;                // k-steps of the score mma = m-tiles of the output mma
  constexpr int CH = HD / 8;                 // 16-byte chunks per cache row
  constexpr int RB = attn_row_bytes(HD);     // padded shared-memory row
  constexpr int SLOTS = 2;                   // the merge barrier is bar[SLOTS]
  constexpr int PS = attn_part_stride(HD);
  constexpr int RS = HD + 4;                 // warp-combine row stride (floats)
  constexpr int DPL = HD / 32;               // head dims per lane in the slice merge

  extern __shared__ __align__(128) unsigned char smem[];
  // [0, region): K rows [128][RB] then V rows [128][RB], or the slice records of the merge
  const uint32_t ks_s = smem_u32(smem), vs_s = ks_s + kAttnCapacity * RB;
  const bool merge_smem = attn_merge_in_smem(HD, GQ, gridDim.x);
  const size_t region = attn_region_bytes(HD, GQ, gridDim.x);
  float* red = reinterpret_cast<float*>(smem + region);  // [8][GQ][RS]
  float* red_m = red + 8 * GQ * RS;  // [8][GQ] warp max
  float* red_l = red_m + 8 * GQ;     // [8][GQ] warp sum
  float* wgt = red_l + 8 * GQ;       // [8][GQ] warp weight exp(m_w - M)
  float* tot = wgt + 8 * GQ;         // [GQ] CTA max M, [GQ] CTA sum L
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + region + (attn_red_bytes(HD, GQ) + 15) / 16 * 16);
  __shared__ int s_last;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sidx = blockIdx.x, g = blockIdx.y;

  pdl_trigger();
  unsigned long long* const tr =
      a.trace ? a.trace + (size_t)blockIdx.y * gridDim.x * a.trace_stride : nullptr;  // row of this CTA
  if (threadIdx.x == 0) {
    timeline_stamp(tr, a.trace_stride, 0);
    mbar_init(&bar[SLOTS], 1);
    mbar_fence_init();
  }

  const int s_max = gridDim.x;
  // A cache of at most one CTA's capacity goes to slice 0 alone (no merge); longer ones split into
  // slices of at least kAttnSub slots. Slice sidx covers [t0, t1); n_act slices are active.
  auto slice = [s_max, sidx](int len, int& t0_, int& t1_, int& nact_) {
    int ch = (len + s_max - 1) / s_max;
    ch = ((ch + 15) / 16) * 16;
    if (len <= kAttnCapacity) ch = kAttnCapacity;
    else if (ch < kAttnSub) ch = kAttnSub;
    nact_ = (len + ch - 1) / ch;
    t0_ = sidx * ch;
    t1_ = min(len, t0_ + ch);
  };
  // cache rows [r_lo, r_hi) of this kv head to shared rows r - base (K and V)
  const __half* kg = a.k_cache + (size_t)g * a.max_seq_len * HD;
  const __half* vg = a.v_cache + (size_t)g * a.max_seq_len * HD;
  auto stage = [&](int base, int r_lo, int r_hi) {
    for (int e = threadIdx.x; e < (r_hi - r_lo) * CH; e += kAttnThreads) {
      const int r = r_lo + e / CH, c = e % CH;
      const size_t off = (size_t)r * HD + c * 8;
      cp_async16(ks_s + (r - base) * RB + c * 16, kg + off, 16u);
      cp_async16(vs_s + (r - base) * RB + c * 16, vg + off, 16u);
    }
  };

  // Before the wait on the QKV kernel: stage the rows of this slice that are final already, for
  // the kv_len the step state shows now (normally this step's, possibly the previous step's: it is
  // only a hint) -- all but its newest slot (the one this step's QKV kernel may be appending) and,
  // past the context, the re-rotated sink keys.  The check after the wait keeps them only when they
  // still fit the slice and hold neither slot the QKV kernel writes.
  int h0, h1, hact, ps0, ps1;
  {
    int hlen = a.step ? *reinterpret_cast<const volatile int*>(&a.step->kv_len) : a.kv_len;
    const int hsink = a.step ? *reinterpret_cast<const volatile int*>(&a.step->kv_sink) : 0;
    hlen = hlen < 1 ? 1 : (hlen > a.max_seq_len ? a.max_seq_len : hlen);
    slice(hlen, h0, h1, hact);
    ps0 = max(h0, hsink > 0 ? 2 : 0);
    ps1 = min(h1, hlen - 1);
    if (ps1 < ps0) ps1 = ps0;
  }
  stage(h0, ps0, ps1);
  cp_async_commit();

  pdl_wait();  // q and the newest K/V slot come from the QKV kernel
  if (threadIdx.x == 0) timeline_stamp(tr, a.trace_stride, 1);

  const int kv_len = a.step ? a.step->kv_len : a.kv_len;
  const int kv_pos = a.step ? a.step->kv_pos : -1;
  const int kv_sink = a.step ? a.step->kv_sink : 0;
  int t0, t1, n_act;
  slice(kv_len, t0, t1, n_act);
  if (t0 >= kv_len) {  // inactive slice (not counted by the merge): let the early copies land
    cp_async_wait<0>();
    return;
  }
  const int n = t1 - t0;
  const int nw = (n + 15) / 16;  // warps with slots
  const bool keep = ps1 > ps0 && t0 == h0 && ps1 <= t1 && !(kv_pos >= ps0 && kv_pos < ps1) && ps0 >= kv_sink;
  if (!keep) {
    if (ps1 > ps0) {  // the early copies land before their rows are written again
      cp_async_wait<0>();
      __syncthreads();
    }
    ps0 = ps1 = t0;
  }
  // the rest of [t0, t1); V rows up to the last warp's 16-slot boundary are zero-filled so
  // 0 * v stays 0 (K rows there are masked out of the softmax)
  stage(t0, t0, ps0);
  stage(t0, ps1, t1);
  for (int e = threadIdx.x; e < (nw * 16 - n) * CH; e += kAttnThreads) {
    const int r = n + e / CH, c = e % CH;
    cp_async16(vs_s + r * RB + c * 16, vg, 0u);
  }
  cp_async_commit();

  // q of the GQ heads as the B operand of the score mma: lane (gh = lane / 4, c4 = lane % 4) holds
  // head gh, dims 16 kk + 2 c4 (+1) and 16 kk + 8 + 2 c4 (+1), as hi and lo fp16 pairs
  const int gh = lane >> 2, c4 = lane & 3;
  uint32_t qh[KS][2], ql[KS][2];
  {
    const float* qp = a.q + (size_t)(g * GQ + (gh < GQ ? gh : 0)) * HD + 2 * c4;
#pragma unroll
    for (int kk = 0; kk < KS; ++kk) {
      float2 x0 = make_float2(0.f, 0.f), x1 = x0;
      if (gh < GQ) {
        x0 = __ldcg(reinterpret_cast<const float2*>(qp + 16 * kk));
        x1 = __ldcg(reinterpret_cast<const float2*>(qp + 16 * kk + 8));
      }
      split_f16x2(x0.x, x0.y, qh[kk][0], ql[kk][0]);
      split_f16x2(x1.x, x1.y, qh[kk][1], ql[kk][1]);
    }
  }
  cp_async_wait<0>();
  __syncthreads();  // every thread's rows have landed
  if (threadIdx.x == 0) timeline_stamp(tr, a.trace_stride, 2);

  // this warp's 16 slots: rows 16 warp ..
  const int my_n = min(16, n - warp * 16);
  if (my_n > 0)
    attn_group<HD, GQ, RB>(ks_s, vs_s, warp * 16, my_n, lane, qh, ql, red + warp * GQ * RS, red_m + warp * GQ,
                           red_l + warp * GQ);
  __syncthreads();
  if (threadIdx.x == 0) timeline_stamp(tr, a.trace_stride, 5);

  // CTA max per head, warp weights and the CTA sum (warp 0; lanes in groups of 8 = warps of a head)
  if (warp == 0) {
#pragma unroll
    for (int base = 0; base < 8 * GQ; base += 32) {
      const int idx = base + lane, h = idx >> 3, w = idx & 7;
      const bool v = idx < 8 * GQ && w < nw;
      const float mw = v ? red_m[w * GQ + h] : -INFINITY;
      float M = mw;
#pragma unroll
      for (int off = 1; off < 8; off <<= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
      const float wt = v ? expf(mw - M) : 0.f;
      float L = v ? wt * red_l[w * GQ + h] : 0.f;
#pragma unroll
      for (int off = 1; off < 8; off <<= 1) L += __shfl_xor_sync(0xffffffffu, L, off);
      if (idx < 8 * GQ) {
        wgt[w * GQ + h] = wt;
        if (w == 0) {
          tot[h] = M;
          tot[GQ + h] = L;
        }
      }
    }
  }
  __syncthreads();
  const bool single = (n_act == 1);
  for (int e = threadIdx.x; e < GQ * HD; e += kAttnThreads) {
    const int h = e / HD, d = e % HD;
    float O = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w)
      if (w < nw) O = fmaf(wgt[w * GQ + h], red[(w * GQ + h) * RS + d], O);
    const int hq = g * GQ + h;
    if (single) {
      a.out[(size_t)hq * HD + d] = O / tot[GQ + h];
    } else {
      float* pp = a.part + ((size_t)hq * s_max + sidx) * PS;
      pp[d] = O;  // o[0..HD), m at HD, l at HD + 1
      if (d == 0) {
        pp[HD] = tot[h];
        pp[HD + 1] = tot[GQ + h];
      }
    }
  }
  if (threadIdx.x == 0) timeline_stamp(tr, a.trace_stride, 3);
  if (single) {
    if (threadIdx.x == 0) timeline_stamp(tr, a.trace_stride, 4);
    return;
  }

  // last-arriving slice of this kv head merges all slices (the merge's bulk copy reuses the rows'
  // shared memory: order the earlier writes to it before the async proxy)
  // The counter's release (by thread 0, after the barrier) publishes this CTA's partial record; the
  // last arrival's acquire makes every slice's record visible to the reads below.
  fence_proxy_async_smem();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned prev = atom_add_acq_rel_gpu(&a.counters[g], 1u);
    s_last = (prev == (unsigned)(n_act - 1));
  }
  __syncthreads();  // also: the combine buffer is no longer read (smem reuse below)
  if (!s_last) {
    if (threadIdx.x == 0) timeline_stamp(tr, a.trace_stride, 4);
    return;
  }
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
  // the rows / merge region, the warp-combine buffer, 3 barriers
  p.smem = attn_region_bytes(head_dim, gq, p.s_max) + (attn_red_bytes(head_dim, gq) + 15) / 16 * 16 + 3 * 8;
  p.part_floats = (size_t)n_heads * p.s_max * attn_part_stride(head_dim);
  p.ok = p.smem <= 226 * 1024;  // two CTAs per SM up to 113 KB
  return p;
}

cudaError_t attn_prepare(const AttnPlan& p) { return raise_smem_cap(p.fn); }

cudaError_t attn_launch(const AttnPlan& p, AttnArgs a, cudaStream_t stream, bool pdl) {
  return launch_kernel(p.fn, p.grid, dim3(kAttnThreads), p.smem, stream, pdl, &a);
}

}  // namespace yb
