// Split-K GQA decode attention over the head-major fp16 KV cache, one thread-block cluster per kv
// head.
//
// yalm computes, per query head h with kv group g = h / (n_heads / n_kv_heads):
//   s_t = q_h . k_t / sqrt(head_dim),  p = softmax(s[0..kv_len)),  out_h = sum_t p_t v_t
// (src/infer.cpp:218-250; the CUDA kernel attn_fused, src/infer.cu:625-667, runs one CTA per q head
// and reads each K/V head once per q head).  Here a cluster of C CTAs (C <= 16, sized by
// attn_prepare so that the kv heads' clusters fill the SMs at once) serves the GQ query heads of one
// kv head, so K/V bytes cross HBM once per kv head; the cache is split over as many of the
// cluster's CTAs as it has 128-slot portions, CTA r taking the r-th equal slice (a multiple of 16
// slots):
//
//   * a producer warp streams the slice through a ring of 64-slot stages with 2-D TMA (tensor maps
//     over the [kv_heads * max_seq_len][head_dim] caches, 64 x 64 boxes with the 128-byte swizzle,
//     no multicast), completing on the stage's mbarrier; the first four stages are issued before the
//     wait on the QKV kernel for the kv_len the step state shows then (a hint), and after the wait
//     the rows that kernel rewrote this step (the newest slot, the re-rotated sink keys) are
//     written into the staged copy from global memory;
//   * eight consumer warps, four per stage, each fold 16 slots of a stage on the tensor cores
//     (mma.sync m16n8k16, fp32 accumulate; operands by ldmatrix from the swizzled rows): S^T[16
//     slots][8 heads] = K . Q^T, an online softmax (running max and sum per head, the output
//     rescaled when the max grows), O^T += V^T . P^T.  q and p are fp32 values split into an fp16
//     value and its fp16 remainder (two mma passes), so the products keep about 22 bits, as the
//     fp32 loops do;
//   * the warps' (m, l, o) are combined in shared memory into the CTA's record, and after a cluster
//     barrier each CTA merges one share of the outputs from the records through distributed shared
//     memory (log-sum-exp rescale).  Long caches of few kv heads (a tensor-parallel rank's) take
//     several clusters per kv head; their records meet in global scratch and the last CTA to arrive
//     on the kv head's counter merges them.  A cache of one portion goes to one CTA, which writes
//     the outputs itself.
#include "attention.cuh"
#include "launch.h"
#include "tmap.h"

#include <math.h>

#include <algorithm>

namespace yb {

constexpr int kAttnThreads = 288;   // 8 consumer warps (two halves of four) + 1 producer warp
constexpr int kAttnChunk = 64;      // cache slots per ring stage (one TMA box of rows)
constexpr int kAttnStages = 4;
constexpr int kAttnMaxCluster = 16;
constexpr int kAttnCtaSlots = 128;    // slots per CTA before a kv head's cache splits further
constexpr int kAttnMaxClusters = 32;  // clusters per kv head
constexpr int kAttnClusterSlots = 1024;  // slots per CTA of one cluster before more clusters share a kv head
constexpr int kAttnBox = 64 * 128;    // one 64-row x 128-byte swizzled box

// ---------------------------------------------------------------- cluster helpers
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_nctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
  return r;
}
// Every thread of every CTA of the cluster arrives (release: its shared-memory writes become
// visible to the other CTAs) and waits for all others (acquire).
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
// Generic address of the same shared-memory variable in CTA `rank` of the cluster (distributed
// shared memory): plain loads through it, which the compiler may batch, read the peer's copy.
__device__ __forceinline__ const float* dsmem_ptr(const float* local, uint32_t rank) {
  uint64_t r;
  asm volatile("mapa.u64 %0, %1, %2;" : "=l"(r) : "l"(local), "r"(rank));
  return reinterpret_cast<const float*>(r);
}

// Shared-memory byte offset of 16-byte chunk q (0 .. HD / 8 - 1) of row i in a staged K or V block:
// HD / 64 boxes of 64 rows x 128 bytes, each row's eight 16-byte chunks permuted by the 128-byte
// swizzle (chunk j of row i at position j ^ (i % 8)); the blocks are 1024-byte aligned.
__device__ __forceinline__ uint32_t sw_off(int i, int q) {
  return (uint32_t)((q >> 3) * kAttnBox + i * 128 + (((q & 7) ^ (i & 7)) << 4));
}

// Shared memory of one CTA, in order (1024-byte aligned base): kAttnStages stages of [K block][V
// block] (HD / 64 boxes each); the warp-combine buffer red[8][GQ][HD + 4], red_m[8][GQ],
// red_l[8][GQ]; the CTA record rec_o[GQ][HD], rec_m[GQ], rec_l[GQ] (read by the cluster); the
// merge's slice weights mw[16][GQ], sums ml[GQ], maxima mM[GQ] and cluster weights
// sw[kAttnMaxClusters][GQ], the warp weights wgt[8][GQ] and CTA totals tot[2][GQ]; then the
// mbarriers full[kAttnStages], empty[kAttnStages], early[kAttnStages].
__host__ __device__ constexpr size_t attn_stage_region(int hd) { return (size_t)2 * (hd / 64) * kAttnBox; }
__host__ __device__ constexpr size_t attn_red_floats(int hd, int gq) { return (size_t)8 * gq * (hd + 4) + 16 * gq; }
__host__ __device__ constexpr size_t attn_rec_floats(int hd, int gq) { return (size_t)gq * hd + 2 * gq; }
__host__ __device__ constexpr size_t attn_merge_floats(int gq) { return (size_t)(kAttnMaxCluster + 2 + kAttnMaxClusters + 8 + 2) * gq; }
__host__ __device__ constexpr size_t attn_bar_offset(int hd, int gq) {
  return (kAttnStages * attn_stage_region(hd) +
          (attn_red_floats(hd, gq) + attn_rec_floats(hd, gq) + attn_merge_floats(gq)) * 4 + 15) / 16 * 16;
}
__host__ __device__ constexpr size_t attn_smem_bytes(int hd, int gq) {
  return attn_bar_offset(hd, gq) + 3 * kAttnStages * 8 + 1024;  // + base alignment
}

// One warp's running softmax state over the slots it has seen: per head pair (2 c4, 2 c4 + 1) the
// running max and sum, and O^T accumulators in the output-mma layout (dims 16 mt + gh (+8)).
template <int KS>
struct AttnAcc {
  float o[KS][4];
  float m0, m1, l0, l1;
};

// 16 staged slots (rows r0 .. r0 + 15 of the swizzled K block at shared address kb and V block at
// vb, my_n of them valid) folded into the warp's running state.  Fragment layouts: mma_16816 in
// common.cuh.
template <int HD>
__device__ __forceinline__ void attn_fold16(AttnAcc<HD / 16>& st, uint32_t kb, uint32_t vb, int r0, int my_n, int lane,
                                            const uint32_t (&qh)[HD / 16][2], const uint32_t (&ql)[HD / 16][2]) {
  constexpr int KS = HD / 16;
  const int gh = lane >> 2;
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
      ldsm_x4(A, kb + sw_off(lr, 2 * kk + lc));
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
  float gm0 = fmaxf(s[0], s[2]), gm1 = fmaxf(s[1], s[3]);
#pragma unroll
  for (int off = 4; off < 32; off <<= 1) {
    gm0 = fmaxf(gm0, __shfl_xor_sync(0xffffffffu, gm0, off));
    gm1 = fmaxf(gm1, __shfl_xor_sync(0xffffffffu, gm1, off));
  }
  // slot 0 of the group is always valid, so the new maxima are finite; a first group rescales
  // the empty state by exp(-inf) = 0
  const float n0 = fmaxf(st.m0, gm0), n1 = fmaxf(st.m1, gm1);
  const float a0 = expf(st.m0 - n0), a1 = expf(st.m1 - n1);
  st.m0 = n0;
  st.m1 = n1;
  const float p0 = v0 ? expf(s[0] - n0) : 0.f, p1 = v0 ? expf(s[1] - n1) : 0.f;
  const float p2 = v1 ? expf(s[2] - n0) : 0.f, p3 = v1 ? expf(s[3] - n1) : 0.f;
  float l0 = p0 + p2, l1 = p1 + p3;
#pragma unroll
  for (int off = 4; off < 32; off <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, off);
    l1 += __shfl_xor_sync(0xffffffffu, l1, off);
  }
  st.l0 = fmaf(st.l0, a0, l0);
  st.l1 = fmaf(st.l1, a1, l1);

  // P^T as the B operand of the output mma: the lane's (slot, head pair) rows transposed to
  // (head, slot pair) by movmatrix, hi and lo parts
  uint32_t x0h, x0l, x1h, x1l;
  split_f16x2(p0, p1, x0h, x0l);
  split_f16x2(p2, p3, x1h, x1l);
  const uint32_t bh0 = movm_trans(x0h), bh1 = movm_trans(x1h);
  const uint32_t bl0 = movm_trans(x0l), bl1 = movm_trans(x1l);
  {
    // ldmatrix.trans rows: matrix lane / 8 = (slots 0-7 | 8-15) x (dims +0 | +8), A order
    const int vr = r0 + 8 * (lane >> 4) + (lane & 7);
    const int vc = (lane >> 3) & 1;
#pragma unroll
    for (int mt = 0; mt < KS; ++mt) {
      st.o[mt][0] *= a0;
      st.o[mt][2] *= a0;
      st.o[mt][1] *= a1;
      st.o[mt][3] *= a1;
      uint32_t A[4];
      ldsm_x4_trans(A, vb + sw_off(vr, 2 * mt + vc));
      mma_16816(st.o[mt], A, bh0, bh1);
      mma_16816(st.o[mt], A, bl0, bl1);
    }
  }
}

template <int HD, int GQ>
__global__ void __launch_bounds__(kAttnThreads, 1)
    attn_decode_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                       const AttnArgs a) {
  static_assert(GQ >= 1 && GQ <= 8, "the score mma has 8 head columns");
  static_assert(HD == 64 || HD == 128, "rows of one or two 128-byte swizzle boxes");
  constexpr int KS = HD / 16;               // k-steps of the score mma = m-tiles of the output mma
  constexpr int CH = HD / 8;                // 16-byte chunks per cache row
  constexpr int NB = HD / 64;               // boxes per row
  constexpr int RS = HD + 4;                // warp-combine row stride (floats)
  constexpr uint32_t STAGE = (uint32_t)attn_stage_region(HD);
  constexpr uint32_t VOFF = NB * kAttnBox;  // V block after the K block

  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // stages on a 1024-byte boundary of the shared window (the swizzle atom); the pointer steps by
  // the same pad and keeps its provenance
  unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const uint32_t s_base = smem_u32(smem);
  float* red = reinterpret_cast<float*>(smem + kAttnStages * STAGE);  // [8][GQ][RS]
  float* red_m = red + 8 * GQ * RS;                                   // [8][GQ]
  float* red_l = red_m + 8 * GQ;                                      // [8][GQ]
  float* rec_o = red + attn_red_floats(HD, GQ);                      // [GQ][HD]
  float* rec_m = rec_o + GQ * HD;                                     // [GQ]
  float* rec_l = rec_m + GQ;                                          // [GQ]
  float* mw = rec_l + GQ;                                             // [kAttnMaxCluster][GQ] slice weights
  float* ml = mw + kAttnMaxCluster * GQ;                              // [GQ] sums
  float* mM = ml + GQ;                                                // [GQ] maxima
  float* sw = mM + GQ;                                                // [kAttnMaxClusters][GQ] cluster weights
  float* wgt = sw + kAttnMaxClusters * GQ;                            // [8][GQ] warp weights
  float* tot = wgt + 8 * GQ;                                          // [GQ] CTA max, [GQ] CTA sum
  const uint32_t full_s = s_base + (uint32_t)attn_bar_offset(HD, GQ), empty_s = full_s + kAttnStages * 8,
                 early_s = empty_s + kAttnStages * 8;

  __shared__ int s_last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = blockIdx.y;
  const int C = (int)cluster_nctarank(), rank = (int)cluster_ctarank();
  const int cl = (int)blockIdx.x / C;  // this CTA's cluster among the kv head's gridDim.x / C
  int n_cl = 1;                        // clusters of the kv head with slots this step
  int c_eff = 1;                       // CTAs of this cluster with slots

  pdl_trigger();
  unsigned long long* const tr =
      a.trace ? a.trace + (size_t)blockIdx.y * gridDim.x * a.trace_stride : nullptr;  // row of this CTA
  if (threadIdx.x == 0) {
    timeline_stamp(tr, a.trace_stride, 0);
    for (int i = 0; i < kAttnStages; ++i) {
      mbar_init_s(full_s + 8 * i, 1);
      mbar_init_s(empty_s + 8 * i, 4);  // the four consumer warps of the stage's half
    }
    for (int i = 0; i < kAttnStages; ++i) mbar_init_s(early_s + 8 * i, 1);
    mbar_fence_init();
  }
  __syncthreads();

  // A cache of len slots is shared by ceil(len / cta_slots) CTAs at most: by c_eff CTAs of one
  // cluster, or, when the CTAs of one cluster would hold more than cluster_slots slots each, by all C
  // CTAs of each of n_cl > 1 clusters; each takes an equal slice (a multiple of 16 slots): this
  // CTA's is [t0, t1), possibly empty.  Clusters cl >= n_cl have nothing to do;
  // with one active CTA (single) it writes the outputs itself and no cluster barrier runs.
  const int n_clusters = (int)gridDim.x / C;
  const int cta_slots = a.cta_slots > 0 ? a.cta_slots : kAttnCtaSlots;
  const int cluster_slots = a.cluster_slots > 0 ? a.cluster_slots : kAttnClusterSlots;
  auto slice = [C, rank, cl, n_clusters, cta_slots, cluster_slots](int len, int& t0_, int& t1_, int& ncl_,
                                                                   int& ceff_) {
    const int want = max(1, (len + cta_slots - 1) / cta_slots);
    ncl_ = min(n_clusters, max(1, (len + C * cluster_slots - 1) / (C * cluster_slots)));
    ceff_ = ncl_ > 1 ? C : min(C, want);
    const int ns = ncl_ * ceff_;
    const int ch = ((len + ns - 1) / ns + 15) / 16 * 16;
    t0_ = rank < ceff_ ? min(len, (cl * ceff_ + rank) * ch) : len;
    t1_ = min(len, t0_ + ch);
  };
  const long long row0 = (long long)g * a.max_seq_len;  // this kv head's first row in the tensor maps

  int kv_len = 0, t0 = 0, t1 = 0;
  bool single = false;
  if (warp == 8) {
    // ------------------------------------------------------------------ producer
    // chunk c (rows t0_ + 64 c ..) of a slice starting at t0_ into stage s, completing on bar
    auto load = [&](int t0_, int c, int s, uint32_t bar) {
      const uint32_t st = s_base + (uint32_t)s * STAGE;
      const int y = (int)(row0 + t0_ + c * kAttnChunk);
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        tma_load_2d_s(st + b * kAttnBox, &kmap, 64 * b, y, bar);
        tma_load_2d_s(st + VOFF + b * kAttnBox, &vmap, 64 * b, y, bar);
      }
    };
    // Before the wait on the QKV kernel: the first stages of the slice for the kv_len the step
    // state shows now (this step's, or the previous step's when this step's state is not written
    // yet).  After the wait they are kept when the slice starts at the same slot (the chunk ->
    // stage mapping is then the same; rows past the slice end are masked); only rows the QKV
    // kernel rewrote this step can differ from what a copy made now would read, and those are
    // written into the staged copy from global memory.
    int h0 = 0, n_early = 0;
    {
      int hlen = a.step ? *reinterpret_cast<const volatile int*>(&a.step->kv_len) : a.kv_len;
      hlen = hlen < 1 ? 1 : (hlen > a.max_seq_len ? a.max_seq_len : hlen);
      int hcl, hce, h1;
      slice(hlen, h0, h1, hcl, hce);
      if (cl < hcl) n_early = min(kAttnStages, (h1 - h0 + kAttnChunk - 1) / kAttnChunk);
    }
    // every stage's early barrier completes its first phase: on the early copy, or at once
    if (lane == 0) {
      for (int c = 0; c < kAttnStages; ++c) {
        mbar_arrive_expect_tx_s(early_s + 8 * c, c < n_early ? STAGE : 0u);
        if (c < n_early) load(h0, c, c, early_s + 8 * c);
      }
      timeline_stamp(tr, a.trace_stride, 7);
    }
    __syncwarp();
    // waits (bounded) for every early copy to have landed
    auto wait_early = [&]() {
      bool ok = true;
      for (int c = 0; c < n_early; ++c) ok = mbar_wait_s(early_s + 8 * c, 0, a.status) && ok;
      return ok;
    };

    pdl_wait();  // q and this step's K/V rows come from the QKV kernel
    kv_len = a.step ? a.step->kv_len : a.kv_len;
    const int kv_pos = a.step ? a.step->kv_pos : -1;
    const int kv_sink = a.step ? a.step->kv_sink : 0;
    int ceff;
    slice(kv_len, t0, t1, n_cl, ceff);
    c_eff = ceff;
    single = n_cl == 1 && c_eff == 1;
    if (cl >= n_cl || (single && rank > 0)) {  // nothing to do: the early copies land, then leave
      wait_early();
      return;
    }
    const int nchunks = (t1 - t0 + kAttnChunk - 1) / kAttnChunk;
    const bool keep = n_early > 0 && h0 == t0;
    const int n_kept = keep ? min(n_early, nchunks) : 0;
    // the early copies have landed before their stages are loaded again
    if (!keep && n_early > 0 && !wait_early()) return;  // timed out (status set)
    auto patch = [&](int t) {  // row t into its kept stage, K and V, swizzled as TMA writes it
      const int i = t - t0, c = i / kAttnChunk, r = i % kAttnChunk;
      const uint32_t st = s_base + (uint32_t)c * STAGE;
      if (lane < 2 * CH) {
        const int q = lane % CH;
        const __half* src = (lane < CH ? a.k_cache : a.v_cache) + (size_t)(row0 + t) * HD + q * 8;
        const uint4 v = __ldcg(reinterpret_cast<const uint4*>(src));
        const uint32_t dst = st + (lane < CH ? 0u : VOFF) + sw_off(r, q);
        asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(dst), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                     : "memory");
      }
    };
    // Kept chunks: the rows the QKV kernel rewrote this step (the newest slot, the sink keys) are
    // written over the chunk's early copy once it has landed; the chunk is then released (its
    // full barrier completes with no bytes).  Other chunks load now, into free stages.
    for (int c = 0; c < nchunks; ++c) {
      const int s = c % kAttnStages;
      if (c < n_kept) {
        const int c0 = t0 + c * kAttnChunk, c1 = c0 + kAttnChunk;
        const bool pos_dirty = kv_pos >= c0 && kv_pos < c1;
        const int sink_end = kv_sink > 0 ? min(kv_sink, c1) : 0;
        if (pos_dirty || sink_end > c0) {
          if (!mbar_wait_s(early_s + 8 * c, 0, a.status)) break;  // timed out (status set)
          if (pos_dirty) patch(kv_pos);
          for (int t = c0; t < sink_end; ++t) patch(t);
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // before TMA writes the stage again
          __syncwarp();
        }
        if (lane == 0) mbar_arrive_expect_tx_s(full_s + 8 * s, 0u);
        continue;
      }
      if (lane == 0) {
        if (c >= kAttnStages && !mbar_wait_s(empty_s + 8 * s, (unsigned)((c / kAttnStages) - 1) & 1u, a.status)) break;
        mbar_arrive_expect_tx_s(full_s + 8 * s, STAGE);
        load(t0, c, s, full_s + 8 * s);
      }
    }
    // early copies of chunks past the slice (a hint longer than the cache) land before the CTA can
    // leave; the consumers wait for every other copy
    if (n_early > n_kept) wait_early();
    // the producer joins the barriers below
  } else {
    // ------------------------------------------------------------------ consumers
    pdl_wait();
    if (threadIdx.x == 0) timeline_stamp(tr, a.trace_stride, 1);
    kv_len = a.step ? a.step->kv_len : a.kv_len;
    int ceff;
    slice(kv_len, t0, t1, n_cl, ceff);
    c_eff = ceff;
    single = n_cl == 1 && c_eff == 1;
    if (cl >= n_cl || (single && rank > 0)) return;
    // q of the GQ heads as the B operand of the score mma: lane (gh = lane / 4, c4 = lane % 4)
    // holds head gh, dims 16 kk + 2 c4 (+1) and 16 kk + 8 + 2 c4 (+1), as hi and lo fp16 pairs
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
    AttnAcc<KS> st;
#pragma unroll
    for (int mt = 0; mt < KS; ++mt)
#pragma unroll
      for (int i = 0; i < 4; ++i) st.o[mt][i] = 0.f;
    st.m0 = st.m1 = -INFINITY;
    st.l0 = st.l1 = 0.f;

    const int nchunks = (t1 - t0 + kAttnChunk - 1) / kAttnChunk;
    const int half = warp >> 2, sub = warp & 3;
    for (int c = half; c < nchunks; c += 2) {
      const int s = c % kAttnStages;
      if (c < kAttnStages) mbar_wait_s(early_s + 8 * s, 0, a.status);  // the stage's early copy, if any
      mbar_wait_s(full_s + 8 * s, (unsigned)(c / kAttnStages) & 1u, a.status);
      if (threadIdx.x == 0 && c == 0) timeline_stamp(tr, a.trace_stride, 2);
      const int n = min(kAttnChunk, t1 - t0 - c * kAttnChunk);
      const int my_n = min(16, n - 16 * sub);
      const uint32_t kb = s_base + (uint32_t)s * STAGE;
      if (my_n > 0) {
        if (my_n < 16) {
          // V rows past the slice end (another slot's or head's data) are zero for this group:
          // 0 * v must stay 0 (K rows there are masked out of the softmax)
          for (int e = lane; e < (16 - my_n) * CH; e += 32) {
            const int r = 16 * sub + my_n + e / CH, q = e % CH;
            asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(kb + VOFF + sw_off(r, q)), "r"(0u)
                         : "memory");
          }
          __syncwarp();
        }
        attn_fold16<HD>(st, kb, kb + VOFF, 16 * sub, my_n, lane, qh, ql);
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // the zeros before the next TMA write
      __syncwarp();
      if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(empty_s + 8 * s) : "memory");
    }
    // the warp's state into the combine buffer: lane holds dims 16 mt + gh (+8) of heads 2 c4, 2 c4 + 1
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int h = 2 * c4 + e;
      if (h < GQ) {
        float* r = red + (warp * GQ + h) * RS;
#pragma unroll
        for (int mt = 0; mt < KS; ++mt) {
          r[16 * mt + gh] = st.o[mt][e];
          r[16 * mt + gh + 8] = st.o[mt][2 + e];
        }
        if (gh == 0) {
          red_m[warp * GQ + h] = e ? st.m1 : st.m0;
          red_l[warp * GQ + h] = e ? st.l1 : st.l0;
        }
      }
    }
    named_sync(1, 256);
    if (threadIdx.x == 0) timeline_stamp(tr, a.trace_stride, 5);
    // per head (eight lanes, one per warp): the max over the warps M, each warp's weight
    // exp(m_w - M) and the CTA sum L (a warp that saw no slot has m = -inf and weighs 0; a CTA that
    // saw none records m = -inf, l = 0, o = 0)
    if (warp < (8 * GQ + 31) / 32) {  // whole warps, so the shuffles see every lane
      const bool valid = (int)threadIdx.x < 8 * GQ;
      const int h = threadIdx.x >> 3, w = threadIdx.x & 7;
      const float mv = valid ? red_m[w * GQ + h] : -INFINITY;
      float M = mv;
#pragma unroll
      for (int off = 1; off < 8; off <<= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off, 8));
      const float wt = mv > -INFINITY ? expf(mv - M) : 0.f;
      float L = valid ? wt * red_l[w * GQ + h] : 0.f;
#pragma unroll
      for (int off = 1; off < 8; off <<= 1) L += __shfl_xor_sync(0xffffffffu, L, off, 8);
      if (valid) {
        wgt[w * GQ + h] = wt;
        if (w == 0) {
          tot[h] = M;
          tot[GQ + h] = L;
        }
      }
    }
    named_sync(1, 256);
    if (threadIdx.x == 0) timeline_stamp(tr, a.trace_stride, 6);
    for (int e = threadIdx.x; e < GQ * HD; e += 256) {
      const int h = e / HD, d = e % HD;
      float O = 0.f;
#pragma unroll
      for (int w = 0; w < 8; ++w) O = fmaf(wgt[w * GQ + h], red[(w * GQ + h) * RS + d], O);
      if (single) {  // this CTA holds every slot: the outputs directly
        a.out[(size_t)g * GQ * HD + e] = O / tot[GQ + h];
        continue;
      }
      rec_o[e] = O;
      if (d == 0) {
        rec_m[h] = tot[h];
        rec_l[h] = tot[GQ + h];
      }
    }
    if (threadIdx.x == 0) timeline_stamp(tr, a.trace_stride, 3);
  }
  if (single) {
    // every CTA of the cluster leaves without a cluster barrier; no copy is in flight (the
    // producer's loads all completed on barriers the consumers waited for)
    if (threadIdx.x == 0) timeline_stamp(tr, a.trace_stride, 4);
    return;
  }

  // ------------------------------------------------------------------ cluster merge
  cluster_sync_all();  // every CTA's record is written and visible cluster-wide
  // per head (sixteen lanes, one per CTA of the cluster): the max M over the slices, each slice's
  // weight exp(m_j - M) and the weighted sum L (an empty slice has m = -inf and weighs 0; the
  // cluster's first slice holds slots whenever any does).  Only the first c_eff CTAs hold slots;
  // every CTA of the cluster merges a share of the outputs.
  if (warp < (16 * GQ + 31) / 32) {  // whole warps, so the shuffles see every lane
    const int h = threadIdx.x >> 4, j = threadIdx.x & 15;
    const bool valid = h < GQ && j < c_eff;
    const float mj = valid ? *dsmem_ptr(rec_m + h, (uint32_t)j) : -INFINITY;
    const float lj = valid ? *dsmem_ptr(rec_l + h, (uint32_t)j) : 0.f;
    float M = mj;
#pragma unroll
    for (int off = 1; off < 16; off <<= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off, 16));
    const float w = mj > -INFINITY ? expf(mj - M) : 0.f;
    float L = w * lj;
#pragma unroll
    for (int off = 1; off < 16; off <<= 1) L += __shfl_xor_sync(0xffffffffu, L, off, 16);
    if (h < GQ) {
      mw[j * GQ + h] = w;
      if (j == 0) {
        ml[h] = L;
        mM[h] = M;
      }
    }
  }
  __syncthreads();
  // this CTA's share of the GQ * HD outputs: the final values when one cluster covers the cache,
  // else the cluster's (o, m, l) record for the merge over clusters
  float* rec_g = n_cl > 1 ? a.part + (size_t)(g * n_clusters + cl) * GQ * (HD + 2) : nullptr;
  {
    const int per = (GQ * HD + C - 1) / C;
    const int o0 = rank * per, o1 = min(GQ * HD, o0 + per);
    for (int e = o0 + (int)threadIdx.x; e < o1; e += kAttnThreads) {
      const int h = e / HD, d = e % HD;
      float v[kAttnMaxCluster];
#pragma unroll
      for (int j = 0; j < kAttnMaxCluster; ++j) v[j] = j < c_eff ? *dsmem_ptr(rec_o + e, (uint32_t)j) : 0.f;
      float O = 0.f;
#pragma unroll
      for (int j = 0; j < kAttnMaxCluster; ++j)
        if (j < c_eff) O = fmaf(mw[j * GQ + h], v[j], O);
      if (n_cl == 1) a.out[(size_t)g * GQ * HD + e] = O / ml[h];
      else rec_g[h * (HD + 2) + d] = O;
    }
    if (n_cl > 1 && rank == 0 && threadIdx.x < GQ) {
      rec_g[threadIdx.x * (HD + 2) + HD] = mM[threadIdx.x];
      rec_g[threadIdx.x * (HD + 2) + HD + 1] = ml[threadIdx.x];
    }
  }
  // done reading the other CTAs' records; the matching wait (before this CTA leaves) keeps its own
  // record in place until every CTA of the cluster is done reading it
  asm volatile("barrier.cluster.arrive.release;" ::: "memory");
  if (n_cl > 1) {
    // The clusters' records merge in the CTA that arrives last on the kv head's counter: one
    // acquire-release add per CTA (after a barrier, so it publishes the CTA's record writes; the
    // last arrival's acquire makes every record visible to its reads).
    __syncthreads();
    if (threadIdx.x == 0) {
      const unsigned prev = atom_add_acq_rel_gpu(&a.counters[g], 1u);
      s_last = prev == (unsigned)(n_cl * C - 1);
    }
    __syncthreads();
    if (s_last) {
      // Every record of the kv head (contiguous in the scratch) into the CTA's idle stage ring in one
      // pass of independent 8-byte loads, then the merge from shared memory: one round trip to L2
      // for the records instead of one per dependent read.
      const float* recs = a.part + (size_t)g * n_clusters * GQ * (HD + 2);
      float* rs = reinterpret_cast<float*>(smem);  // [n_cl][GQ][HD + 2]
      const int n2 = n_cl * GQ * (HD + 2) / 2;
      constexpr int U = 8;
      for (int i0 = (int)threadIdx.x; i0 < n2; i0 += U * kAttnThreads) {
        float2 v[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int i = i0 + u * kAttnThreads;
          v[u] = i < n2 ? __ldcg(reinterpret_cast<const float2*>(recs) + i) : make_float2(0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int i = i0 + u * kAttnThreads;
          if (i < n2) reinterpret_cast<float2*>(rs)[i] = v[u];
        }
      }
      __syncthreads();
      if (threadIdx.x < GQ) {
        const int h = threadIdx.x;
        float M = -INFINITY;
        for (int q = 0; q < n_cl; ++q) M = fmaxf(M, rs[(q * GQ + h) * (HD + 2) + HD]);
        float L = 0.f;
        for (int q = 0; q < n_cl; ++q) {
          const float* r = rs + (q * GQ + h) * (HD + 2);
          const float w = r[HD] > -INFINITY ? expf(r[HD] - M) : 0.f;
          sw[q * GQ + h] = w;
          L = fmaf(w, r[HD + 1], L);
        }
        ml[h] = L;
      }
      __syncthreads();
      for (int e = threadIdx.x; e < GQ * HD; e += kAttnThreads) {
        const int h = e / HD, d = e % HD;
        float O = 0.f;
        for (int q = 0; q < n_cl; ++q) O = fmaf(sw[q * GQ + h], rs[(q * GQ + h) * (HD + 2) + d], O);
        a.out[(size_t)g * GQ * HD + e] = O / ml[h];
      }
      if (threadIdx.x == 0) a.counters[g] = 0u;  // ready for the next launch
    }
  }
  asm volatile("barrier.cluster.wait.acquire;" ::: "memory");
  if (threadIdx.x == 0) timeline_stamp(tr, a.trace_stride, 4);
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
  if (n_kv_heads <= 0 || n_heads % n_kv_heads || max_seq_len <= 0) return p;
  const int gq = n_heads / n_kv_heads;
  if (head_dim == 128) p.fn = pick_gq<128>(gq);
  else if (head_dim == 64) p.fn = pick_gq<64>(gq);
  else p.fn = nullptr;
  if (!p.fn) return p;
  p.smem = head_dim == 128 ? attn_smem_bytes(128, gq) : attn_smem_bytes(64, gq);
  // Until attn_prepare sizes it for the device: one cluster of 16 per kv head.  The scratch for the
  // merge over clusters is sized for any device: at most kAttnMaxClusters clusters of a kv head, no
  // more than one per kAttnCtaSlots slots of the context, and no more records than the stage ring
  // of the merging CTA holds.
  p.cluster = kAttnMaxCluster;
  p.grid = dim3(p.cluster, n_kv_heads);
  const int ring_records = (int)(kAttnStages * attn_stage_region(head_dim) / 4 / ((size_t)gq * (head_dim + 2)));
  p.s_max = std::min({kAttnMaxClusters, (max_seq_len + kAttnCtaSlots - 1) / kAttnCtaSlots, ring_records});
  p.part_floats = (size_t)n_kv_heads * p.s_max * gq * (head_dim + 2);
  p.max_seq_len = max_seq_len;
  p.ok = p.smem <= 227 * 1024;
  return p;
}

cudaError_t attn_prepare(AttnPlan& p) {
  cudaError_t e = raise_smem_cap(p.fn);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(p.fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  if (e != cudaSuccess) return e;
  const int n_kv = (int)p.grid.y;
  auto max_clusters = [&](int c, int* n) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(c, n_kv);
    cfg.blockDim = dim3(kAttnThreads);
    cfg.dynamicSmemBytes = p.smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = c;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaOccupancyMaxActiveClusters(n, p.fn, &cfg);
  };
  // The largest cluster (1..16 CTAs, any size: the merge does not need a power of two) of which the
  // GPU holds one per kv head at once: the kv heads run in one wave and merge through distributed
  // shared memory only.  A cluster lies inside one GPC, so on a B200 (148 SMs) seven clusters of 16
  // fit at once but eleven of 10.  Only where that leaves most SMs idle (few kv heads, a
  // tensor-parallel rank's) does a kv head get more clusters, as many as still run at once and the
  // context can fill at cluster_slots slots per CTA; the kernel then takes the extra ones only for
  // caches that long, since their merge goes through global scratch.
  const LaunchTuning tune = LaunchTuning::from_env();
  int dev = 0, n_sms = 148;
  if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
  if ((e = cudaDeviceGetAttribute(&n_sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
  int best_c = 1;
  for (int c = kAttnMaxCluster; c >= 1; --c) {
    int n = 0;
    if ((e = max_clusters(c, &n)) != cudaSuccess) return e;
    p.max_active[c - 1] = n;
    if (best_c == 1 && n >= n_kv) best_c = c;
  }
  int best_s = 1;
  if (2 * best_c * n_kv <= n_sms) {
    const int cs = std::max(16, tune.attn_cluster_slots);
    best_s = std::max(1, p.max_active[best_c - 1] / n_kv);
    best_s = std::min(best_s, std::max(1, (p.max_seq_len + best_c * cs - 1) / (best_c * cs)));
    best_s = std::min(best_s, p.s_max);
  }
  if (tune.attn_cluster > 0) best_c = std::min(tune.attn_cluster, kAttnMaxCluster);
  if (tune.attn_clusters_per_head > 0) best_s = std::min(tune.attn_clusters_per_head, p.s_max);
  p.cluster = best_c;
  p.grid = dim3(best_c * best_s, n_kv);
  return cudaSuccess;
}

bool attn_maps(AttnMaps* m, const __half* k_cache, const __half* v_cache, int n_kv_heads, int max_seq_len,
               int head_dim) {
  const long long rows = (long long)n_kv_heads * max_seq_len;
  return tmap_f16_2d_sw128(&m->k, k_cache, rows, head_dim, 64, kAttnChunk) &&
         tmap_f16_2d_sw128(&m->v, v_cache, rows, head_dim, 64, kAttnChunk);
}

cudaError_t attn_launch(const AttnPlan& p, AttnArgs a, const AttnMaps& m, cudaStream_t stream, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = p.grid;
  cfg.blockDim = dim3(kAttnThreads);
  cfg.dynamicSmemBytes = p.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = p.cluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2 : 1;
  CUtensorMap km = m.k, vm = m.v;
  void* params[] = {&km, &vm, &a};
  return cudaLaunchKernelExC(&cfg, p.fn, params);
}

}  // namespace yb
