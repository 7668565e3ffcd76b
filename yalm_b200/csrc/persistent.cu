// Persistent decode step: one cooperative launch runs a whole token.
//
// Grid: two CTAs per SM, all co-resident.  Each CTA = one TMA producer warp + 8 consumer warps.
// The producer walks the CTA's share of the whole step in order — per layer: its rows of
// [Wq;Wk;Wv], its attention K/V sub-chunks, its rows of Wo, W1/W3 (interleaved), W2; then its rows of
// the classifier — and streams each stage into a 3 x 32 KB shared-memory ring with cp.async.bulk.
// It waits only for free ring slots, never for the phase barriers, so while consumers wait at a
// barrier the ring keeps filling with the next phase's weights and HBM stays busy across phase
// boundaries.  Consumers run the phases of yalm's Block::forward (src/infer.cpp:256-392):
//   QKV (RMSNorm prologue; clip, RoPE, KV append, sink rotation epilogue)      | grid barrier
//   attention over the cache (online softmax per slice, log-sum-exp merge)     | grid barrier
//   wo (+ residual)                                                            | grid barrier
//   W1/W3 (RMSNorm prologue; SwiGLU epilogue)                                  | grid barrier
//   W2 (+ residual)                                                            | grid barrier
// and finally the classifier (final RMSNorm prologue).  Every wait is bounded: a CTA that gives up
// records a status bit and raises a global flag that makes every other CTA stop waiting too.
#include "persistent.cuh"
#include "launch.h"

#include <math.h>

namespace yb {

namespace {

constexpr unsigned kStatusGridTimeout = 1u << 3;
constexpr int kPAttnMinSlice = 256;

struct PSmem {
  unsigned char* ring;
  float* red;
  float* S;        // [2][GQ][64] attention scores / probabilities
  float* scratch;  // 256 floats
  uint64_t* full;
  uint64_t* empty;
};

__device__ __forceinline__ unsigned long long ld_acquire_gpu_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long v;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(v));
  return v;
}
__device__ __forceinline__ void stamp(const PArgs& a, int ev) {
  if (a.trace && ev < kTraceEvents) a.trace[(size_t)blockIdx.x * kTraceEvents + ev] = global_ns();
}
__device__ __forceinline__ unsigned ld_volatile_u32(const unsigned* p) {
  return *reinterpret_cast<const volatile unsigned*>(p);
}

__device__ __forceinline__ void give_up(const PArgs& a, unsigned bit, int* s_abort) {
  atomicOr(a.status, bit);
  atomicExch(a.fail, 1u);
  *reinterpret_cast<volatile int*>(s_abort) = 1;
}

// mbarrier wait that also stops when another CTA has failed.
__device__ __forceinline__ bool pwait(uint64_t* bar, unsigned parity, const PArgs& a, int* s_abort) {
  if (mbar_try_wait(bar, parity)) return true;
  long long t0 = clock64();
  int n = 0;
  while (!mbar_try_wait(bar, parity)) {
    if ((++n & 255) == 0) {
      if (ld_volatile_u32(a.fail) || *reinterpret_cast<volatile int*>(s_abort)) {
        *reinterpret_cast<volatile int*>(s_abort) = 1;
        return false;
      }
      if (clock64() - t0 > kWaitBudgetCycles) {
        give_up(a, kStatusMbarTimeout, s_abort);
        return false;
      }
    }
  }
  return true;
}

__device__ __forceinline__ void split_range(int units, int G, int b, int& u0, int& u1) {
  u0 = (int)((long long)units * b / G);
  u1 = (int)((long long)units * (b + 1) / G);
}

// Attention slicing of the cache for this step: S slices of `chunk` slots per kv head (chunk a
// multiple of the 64-slot stage), at most kPMaxSplits, at most one slice per CTA.
__device__ __forceinline__ void attn_slicing(int kv_len, int n_kv, int G, int& S, int& chunk) {
  // slices of at least kPAttnMinSlice slots: a short cache is one slice per kv head, no merge
  int s = (kv_len + kPAttnMinSlice - 1) / kPAttnMinSlice;
  if (s > kPMaxSplits) s = kPMaxSplits;
  int cap = G / n_kv;
  if (cap < 1) cap = 1;
  if (s > cap) s = cap;
  chunk = (kv_len + s - 1) / s;
  chunk = (chunk + kPAttnSub - 1) / kPAttnSub * kPAttnSub;
  S = (kv_len + chunk - 1) / chunk;
}

// ------------------------------------------------------------------------------------ work split
// Phases of one step, in order: per layer p = 0 QKV, 1 attention, 2 Wo, 3 W1/W3, 4 W2; then the
// classifier.  A matvec phase has T stages of RT whole rows, split into contiguous per-CTA shares
// (static_pct = 100), or a contiguous share of static_pct percent plus stages claimed one at a time
// from per-phase counters (at most `dyn_cap` per CTA).  Attention units are (kv head, slice) items,
// all claimed dynamically.
enum : int { kFlagLastOfPhase = 1, kFlagEmpty = 2, kFlagItemFirst = 4, kFlagItemLast = 8 };

struct PhaseInfo {
  int kind;   // 0 QKV, 1 attention, 2 Wo, 3 W1/W3, 4 W2, 5 classifier
  int layer;
  int rows, cols, rt;  // matvec phases
  int T, q, R, dyn_cap;
  int S, chunk, n_items;  // attention
};

template <int RD, int RO, int RH>
__device__ __forceinline__ PhaseInfo phase_info(const PArgs& a, int ph) {
  PhaseInfo f;
  const int G = gridDim.x;
  f.layer = ph / 5;
  f.kind = f.layer < a.n_layers ? ph % 5 : 5;
  f.rows = f.cols = f.rt = f.T = f.q = f.R = f.dyn_cap = 0;
  f.S = f.chunk = f.n_items = 0;
  switch (f.kind) {
    case 0: f.rows = a.q_rows + 2 * a.kv_rows; f.cols = a.dim; f.rt = RD; break;
    case 2: f.rows = a.dim; f.cols = a.q_rows; f.rt = RO; break;
    case 3: f.rows = 2 * a.hid; f.cols = a.dim; f.rt = RD; break;
    case 4: f.rows = a.dim; f.cols = a.hid; f.rt = RH; break;
    case 5: f.rows = a.vocab_rows; f.cols = a.dim; f.rt = RD; break;
    default: break;
  }
  if (f.kind == 1) {
    attn_slicing(a.kv_len, a.n_kv, G, f.S, f.chunk);
    f.n_items = f.S * a.n_kv;
    f.T = f.n_items;
    f.q = 0;
    f.R = f.n_items;
    f.dyn_cap = f.n_items;
  } else {
    f.T = (f.rows + f.rt - 1) / f.rt;
    f.q = (int)((long long)f.T * a.static_pct / (100ll * G));
    if (f.q * G > f.T) f.q = f.T / G;
    f.R = f.T - G * f.q;
    f.dyn_cap = 2 * ((f.R + G - 1) / G) + 1;
  }
  return f;
}

// Claims the next dynamic unit of a phase: the R dynamic units are spread over nc counters
// (unit d belongs to counter d mod nc); a CTA starts at counter (blockIdx mod nc) and moves on when
// one runs dry.  Returns R when none is left.
__device__ __forceinline__ int claim_unit(unsigned* ctr, int ph, int nc, int R, int& cj, int& tried) {
  while (tried < nc) {
    const unsigned v = atomicAdd(&ctr[ph * nc + cj], 1u);
    const int d = (int)v * nc + cj;
    if (d < R) return d;
    cj = (cj + 1) % nc;
    ++tried;
  }
  return R;
}

// ------------------------------------------------------------------------------------ producer
struct Producer {
  const PArgs& a;
  const PSmem& sm;
  int* s_abort;
  int* tag;  // [kPSlots][4]: phase, unit, c0 (attention), flags
  unsigned* ctr;
  uint64_t pol;
  int i = 0;
  bool ok = true;

  __device__ Producer(const PArgs& a_, const PSmem& sm_, int* ab, int* tg, unsigned* c)
      : a(a_), sm(sm_), s_abort(ab), tag(tg), ctr(c) {
    pol = l2_evict_first_policy();
  }
  __device__ unsigned char* acquire() {
    const int slot = i % kPSlots;
    if (i >= kPSlots && !pwait(&sm.empty[slot], ((i / kPSlots) - 1) & 1, a, s_abort)) ok = false;
    return sm.ring + (size_t)slot * kPSlotBytes;
  }
  __device__ void set_tag(int slot, int ph, int unit, int c0, int flags) {
    volatile int* t = tag + slot * 4;
    t[0] = ph;
    t[1] = unit;
    t[2] = c0;
    t[3] = flags;
  }
  __device__ void empty_marker(int ph) {
    acquire();
    if (!ok) return;
    const int slot = i % kPSlots;
    set_tag(slot, ph, -1, 0, kFlagEmpty | kFlagLastOfPhase);
    mbar_arrive(&sm.full[slot]);
    ++i;
  }
  __device__ void rows_stage(const __half* w, const PhaseInfo& f, int ph, int unit, int flags) {
    unsigned char* dst = acquire();
    if (!ok) return;
    const int slot = i % kPSlots;
    const int r0 = unit * f.rt;
    const int nr = min(f.rt, f.rows - r0);
    const unsigned rb = (unsigned)f.cols * 2u;
    set_tag(slot, ph, unit, 0, flags);
    mbar_arrive_expect_tx(&sm.full[slot], (unsigned)nr * rb);
    bulk_g2s(dst, reinterpret_cast<const unsigned char*>(w) + (size_t)r0 * rb, (unsigned)nr * rb, &sm.full[slot], pol);
    ++i;
  }
  __device__ void kv_stage(const PLayer& L, int hd, int ph, int item, int c0, int cn, int flags) {
    unsigned char* dst = acquire();
    if (!ok) return;
    const int slot = i % kPSlots;
    const int g = item % a.n_kv;
    const unsigned bytes = (unsigned)cn * hd * 2u;
    const size_t off = ((size_t)g * a.max_seq_len + c0) * hd;
    set_tag(slot, ph, item, c0, flags);
    mbar_arrive_expect_tx(&sm.full[slot], 2u * bytes);
    bulk_g2s_nohint(dst, L.k_cache + off, bytes, &sm.full[slot]);
    bulk_g2s_nohint(dst + (size_t)kPAttnSub * hd * 2, L.v_cache + off, bytes, &sm.full[slot]);
    ++i;
  }

  template <int RD, int RO, int RH, int HD>
  __device__ void run() {
    const int G = gridDim.x, b = blockIdx.x;
    const int n_phases = 5 * a.n_layers + (a.mode ? 1 : 0);
    for (int ph = 0; ph < n_phases && ok; ++ph) {
      const PhaseInfo f = phase_info<RD, RO, RH>(a, ph);
      int issued = 0;
      const int nc = a.claim_ctrs;
      int cj = b % nc, tried = 0;
      if (f.kind == 1) {
        const PLayer& L = a.layers[f.layer];
        int item = claim_unit(ctr, ph, nc, f.n_items, cj, tried);
        int n_claimed = 0;
        while (ok && item < f.n_items) {
          ++n_claimed;
          const int nxt = n_claimed < f.dyn_cap ? claim_unit(ctr, ph, nc, f.n_items, cj, tried) : f.n_items;
          const int t0 = (item / a.n_kv) * f.chunk, t1 = min(a.kv_len, t0 + f.chunk);
          for (int c0 = t0; c0 < t1 && ok; c0 += kPAttnSub) {
            const bool last_sub = c0 + kPAttnSub >= t1;
            int flags = (c0 == t0 ? kFlagItemFirst : 0) | (last_sub ? kFlagItemLast : 0);
            if (last_sub && nxt >= f.n_items) flags |= kFlagLastOfPhase;
            kv_stage(L, HD, ph, item, c0, min(kPAttnSub, t1 - c0), flags);
            ++issued;
          }
          item = nxt;
        }
      } else {
        const __half* w;
        if (f.kind == 5) {
          w = a.wcls;
        } else {
          const PLayer& L = a.layers[f.layer];
          w = f.kind == 0 ? L.wqkv : f.kind == 2 ? L.wo : f.kind == 3 ? L.w13 : L.w2;
        }
        // Static contiguous share (stages [T b / G, T (b+1) / G)) for static_pct = 100 (the measured
        // best); with static_pct < 100 a contiguous share of that size, then the rest claimed one
        // stage at a time from the phase's counters.
        int s0, s1;
        if (a.static_pct >= 100) {
          split_range(f.T, G, b, s0, s1);
          for (int s2 = s0; s2 < s1 && ok; ++s2) {
            rows_stage(w, f, ph, s2, s2 + 1 == s1 ? kFlagLastOfPhase : 0);
            ++issued;
          }
        } else {
          int pending = (f.dyn_cap > 0 && f.R > 0) ? claim_unit(ctr, ph, nc, f.R, cj, tried) : f.R;
          int n_dyn = 0;
          for (int k = 0; k < f.q && ok; ++k) {
            const bool last = (k + 1 == f.q) && pending >= f.R;
            rows_stage(w, f, ph, b * f.q + k, last ? kFlagLastOfPhase : 0);
            ++issued;
          }
          while (ok && pending < f.R) {
            const int cur = pending;
            ++n_dyn;
            pending = n_dyn < f.dyn_cap ? claim_unit(ctr, ph, nc, f.R, cj, tried) : f.R;
            rows_stage(w, f, ph, G * f.q + cur, pending >= f.R ? kFlagLastOfPhase : 0);
            ++issued;
          }
        }
      }
      if (issued == 0 && ok) empty_marker(ph);
    }
  }

  __device__ void drain() {
    for (int k = max(0, i - kPSlots); k < i; ++k) mbar_wait(&sm.full[k % kPSlots], (k / kPSlots) & 1, nullptr);
  }
};

// ------------------------------------------------------------------------------------ consumers
struct Consumer {
  const PArgs& a;
  const PSmem& sm;
  int* s_abort;
  int* s_flag;
  const int* tag;
  int* mine;        // stage units this CTA processed in the current phase
  int i = 0;        // ring stage counter (mirrors the producer's)
  int bar_idx = 0;  // grid barriers passed this step
  const int t = threadIdx.x;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  static constexpr int NT = kPWarps * 32;

  __device__ Consumer(const PArgs& a_, const PSmem& sm_, int* ab, int* fl, const int* tg, int* mn)
      : a(a_), sm(sm_), s_abort(ab), s_flag(fl), tag(tg), mine(mn) {}

  __device__ bool aborted() const { return *reinterpret_cast<volatile int*>(s_abort) != 0; }

  __device__ bool grid_sync() {
    named_sync(1, NT);
    ++bar_idx;
    if (t == 0 && !aborted()) {
      stamp(a, 2 * bar_idx - 1);
      __threadfence();
      atomicAdd(a.bar, 1ull);
      const unsigned long long target = (unsigned long long)bar_idx * gridDim.x;
      long long t0 = clock64();
      while (ld_acquire_gpu_u64(a.bar) < target) {
        if (ld_volatile_u32(a.fail)) {
          *reinterpret_cast<volatile int*>(s_abort) = 1;
          break;
        }
        if (clock64() - t0 > kWaitBudgetCycles) {
          give_up(a, kStatusGridTimeout, s_abort);
          break;
        }
        __nanosleep(32);
      }
      __threadfence();
      stamp(a, 2 * bar_idx);
    }
    named_sync(1, NT);
    return !aborted();
  }

  // waits for the next ring slot; returns its index or -1
  __device__ int next_slot() {
    const int slot = i % kPSlots;
    if (!pwait(&sm.full[slot], (i / kPSlots) & 1, a, s_abort)) return -1;
    return slot;
  }
  __device__ void release(int slot) {
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm.empty[slot]);
  }

  template <int KPT>
  __device__ void load_x(float4 (&xr)[KPT][2], int cols, const float* x, const __half* emb_row, float* x_out) {
    const int nch = cols >> 3;
    int w0 = 0, w1 = 0;
    if (x_out) split_range(nch, gridDim.x, blockIdx.x, w0, w1);
#pragma unroll
    for (int k = 0; k < KPT; ++k) {
      const int c = k * NT + t;
      if (c < nch) {
        if (emb_row) {
          const uint4 raw = __ldg(reinterpret_cast<const uint4*>(emb_row) + c);
          const __half2* h = reinterpret_cast<const __half2*>(&raw);
          const float2 f0 = __half22float2(h[0]), f1 = __half22float2(h[1]);
          const float2 f2 = __half22float2(h[2]), f3 = __half22float2(h[3]);
          xr[k][0] = make_float4(f0.x, f0.y, f1.x, f1.y);
          xr[k][1] = make_float4(f2.x, f2.y, f3.x, f3.y);
        } else {
          xr[k][0] = __ldcg(reinterpret_cast<const float4*>(x) + 2 * c);
          xr[k][1] = __ldcg(reinterpret_cast<const float4*>(x) + 2 * c + 1);
        }
        if (x_out && c >= w0 && c < w1) {
          __stcg(reinterpret_cast<float4*>(x_out) + 2 * c, xr[k][0]);
          __stcg(reinterpret_cast<float4*>(x_out) + 2 * c + 1, xr[k][1]);
        }
      } else {
        xr[k][0] = make_float4(0.f, 0.f, 0.f, 0.f);
        xr[k][1] = xr[k][0];
      }
    }
  }

  // RMSNorm of the distributed vector (yalm src/infer.cpp:136-146)
  template <int KPT>
  __device__ void rmsnorm(float4 (&xr)[KPT][2], int cols, const float* w) {
    const int nch = cols >> 3;
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < KPT; ++k) {
      ss += xr[k][0].x * xr[k][0].x + xr[k][0].y * xr[k][0].y + xr[k][0].z * xr[k][0].z + xr[k][0].w * xr[k][0].w;
      ss += xr[k][1].x * xr[k][1].x + xr[k][1].y * xr[k][1].y + xr[k][1].z * xr[k][1].z + xr[k][1].w * xr[k][1].w;
    }
    ss = warp_sum(ss);
    if (lane == 0) sm.scratch[warp] = ss;
    named_sync(1, NT);
    float tot = 0.f;
#pragma unroll
    for (int v = 0; v < kPWarps; ++v) tot += sm.scratch[v];
    named_sync(1, NT);  // scratch is reused right after
    const float scale = 1.0f / sqrtf(tot / (float)cols + a.eps);
#pragma unroll
    for (int k = 0; k < KPT; ++k) {
      const int c = k * NT + t;
      if (c < nch) {
        const float4 n0 = __ldg(reinterpret_cast<const float4*>(w) + 2 * c);
        const float4 n1 = __ldg(reinterpret_cast<const float4*>(w) + 2 * c + 1);
        xr[k][0] = make_float4(xr[k][0].x * scale * n0.x, xr[k][0].y * scale * n0.y, xr[k][0].z * scale * n0.z,
                               xr[k][0].w * scale * n0.w);
        xr[k][1] = make_float4(xr[k][1].x * scale * n1.x, xr[k][1].y * scale * n1.y, xr[k][1].z * scale * n1.z,
                               xr[k][1].w * scale * n1.w);
      }
    }
  }

  // Consumes this CTA's stages of one matvec phase (as tagged by the producer); leaves per-(row,
  // warp) partial sums in sm.red in local order and the stage units in mine[].  Returns the number
  // of local stages, or -1 when aborted.
  template <int KPT, int RT>
  __device__ int stream_rows(int ph, int n_rows, int cols, const float4 (&xr)[KPT][2]) {
    constexpr int LOG_RT = (RT == 1) ? 0 : (RT == 2) ? 1 : (RT == 4) ? 2 : 3;
    const int nch = cols >> 3;
    const unsigned rb = (unsigned)cols * 2u;
    int n_local = 0;
    while (true) {
      const int slot = next_slot();
      if (slot < 0) return -1;
      const volatile int* tg = tag + slot * 4;
      const int tph = tg[0], unit = tg[1], flags = tg[3];
      if (tph != ph) {
        give_up(a, kStatusBadArgs, s_abort);
        return -1;
      }
      if (flags & kFlagEmpty) {
        release(slot);
        ++i;
        break;
      }
      const unsigned char* st = sm.ring + (size_t)slot * kPSlotBytes;
      const int nr = min(RT, n_rows - unit * RT);
      float acc[RT];
#pragma unroll
      for (int r = 0; r < RT; ++r) {
        uint4 wv[KPT];
#pragma unroll
        for (int k = 0; k < KPT; ++k) {
          const int c = k * NT + t;
          wv[k] = (r < nr && c < nch) ? lds128(st + (size_t)r * rb + (size_t)c * 16) : make_uint4(0, 0, 0, 0);
        }
        float sacc = 0.f;
#pragma unroll
        for (int k = 0; k < KPT; ++k) sacc += dot8(wv[k], xr[k][0], xr[k][1]);
        acc[r] = sacc;
      }
      release(slot);
      ++i;
      const float v = warp_reduce_scatter<RT>(acc, lane);
      const int rr = lane >> (5 - LOG_RT);
      if ((lane & ((32 >> LOG_RT) - 1)) == 0 && rr < nr) sm.red[(n_local * RT + rr) * kPWarps + warp] = v;
      if (t == 0) mine[n_local] = unit;
      ++n_local;
      if (flags & kFlagLastOfPhase) break;
    }
    named_sync(1, NT);
    return n_local;
  }

  __device__ float row_sum(int lr) const {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kPWarps; ++w) s += sm.red[lr * kPWarps + w];
    return s;
  }

  // ---- matvec phases
  template <int KPT, int RT>
  __device__ bool qkv(int ph, const PLayer& L, int layer) {
    float4 xr[KPT][2];
    const __half* emb_row = layer == 0 ? a.emb + (size_t)a.token * a.dim : nullptr;
    load_x<KPT>(xr, a.dim, a.x, emb_row, layer == 0 ? a.x : nullptr);
    rmsnorm<KPT>(xr, a.dim, L.rms_att);
    const int n_rows = a.q_rows + 2 * a.kv_rows;
    const int n = stream_rows<KPT, RT>(ph, n_rows, a.dim, xr);
    if (n < 0) return false;
    const int hd = a.head_dim;
    for (int lp = t; lp < n * RT / 2; lp += NT) {
      const int lr = 2 * lp;
      const int gr = mine[lr / RT] * RT + lr % RT;
      if (gr >= n_rows) continue;
      float s0 = row_sum(lr), s1 = row_sum(lr + 1);
      s0 = s0 < -a.qkv_clip ? -a.qkv_clip : (s0 > a.qkv_clip ? a.qkv_clip : s0);  // src/infer.cpp:283-290
      s1 = s1 < -a.qkv_clip ? -a.qkv_clip : (s1 > a.qkv_clip ? a.qkv_clip : s1);
      if (gr < a.q_rows + a.kv_rows) {
        const int jh = (gr < a.q_rows ? gr : gr - a.q_rows) % hd;  // RoPE, src/infer.cpp:202-215
        float fcr = 1.f, fci = 0.f;
        if (jh < a.rotary_dim) sincosf((float)a.pos * a.inv_freq[jh >> 1], &fci, &fcr);
        const float r0 = s0 * fcr - s1 * fci, r1 = s0 * fci + s1 * fcr;
        if (gr < a.q_rows) {
          __stcg(a.q + gr, r0);
          __stcg(a.q + gr + 1, r1);
        } else {
          const int kr = gr - a.q_rows;
          __half* kh = L.k_cache + (size_t)(kr / hd) * a.max_seq_len * hd;
          *reinterpret_cast<__half2*>(kh + (size_t)a.kv_pos * hd + jh) = __floats2half2_rn(r0, r1);
          if (a.kv_sink > 0 && jh < a.rotary_dim) {  // sinks, src/infer.cpp:307-325
            float c1, sn;
            sincosf(a.inv_freq[jh >> 1], &sn, &c1);
            for (int r = 0; r < a.kv_sink; ++r) {
              __half2* p = reinterpret_cast<__half2*>(kh + (size_t)r * hd + jh);
              const float2 kv = __half22float2(__ldcg(p));
              *p = __floats2half2_rn(kv.x * c1 - kv.y * sn, kv.x * sn + kv.y * c1);
            }
          }
        }
      } else {
        const int vr = gr - a.q_rows - a.kv_rows;
        __half* vh = L.v_cache + (size_t)(vr / hd) * a.max_seq_len * hd;
        *reinterpret_cast<__half2*>(vh + (size_t)a.kv_pos * hd + vr % hd) = __floats2half2_rn(s0, s1);
      }
    }
    return true;
  }

  template <int KPT, int RT>
  __device__ bool resid(int ph, int cols, const float* xin, float* y) {
    float4 xr[KPT][2];
    load_x<KPT>(xr, cols, xin, nullptr, nullptr);
    const int n = stream_rows<KPT, RT>(ph, a.dim, cols, xr);
    if (n < 0) return false;
    for (int lr = t; lr < n * RT; lr += NT) {
      const int row = mine[lr / RT] * RT + lr % RT;
      if (row < a.dim) __stcg(y + row, __ldcg(y + row) + row_sum(lr));
    }
    return true;
  }

  template <int KPT, int RT>
  __device__ bool gateup(int ph, const PLayer& L) {
    float4 xr[KPT][2];
    load_x<KPT>(xr, a.dim, a.x, nullptr, nullptr);
    rmsnorm<KPT>(xr, a.dim, L.rms_ffn);
    const int n = stream_rows<KPT, RT>(ph, 2 * a.hid, a.dim, xr);
    if (n < 0) return false;
    for (int lp = t; lp < n * RT / 2; lp += NT) {  // src/infer.cpp:367-382
      const int lr = 2 * lp;
      const int gr = mine[lr / RT] * RT + lr % RT;
      if (gr >= 2 * a.hid) continue;
      const float g = row_sum(lr), u = row_sum(lr + 1);
      const float act = a.act_silu ? g / (1.0f + expf(-g))
                                   : 0.5f * g * (1.0f + tanhf(0.797885f * (g + 0.044715f * g * g * g)));
      __stcg(a.hb + gr / 2, act * u);
    }
    return true;
  }

  template <int KPT, int RT>
  __device__ bool classifier(int ph) {
    float4 xr[KPT][2];
    load_x<KPT>(xr, a.dim, a.x, nullptr, nullptr);
    rmsnorm<KPT>(xr, a.dim, a.rms_final);
    const int n = stream_rows<KPT, RT>(ph, a.vocab_rows, a.dim, xr);
    if (n < 0) return false;
    for (int lr = t; lr < n * RT; lr += NT) {
      const int row = mine[lr / RT] * RT + lr % RT;
      if (row < a.vocab_rows) a.logits[row] = row_sum(lr);
    }
    return true;
  }

  // ---- attention: the (kv head, slice) items this CTA claimed, K/V staged by the producer
  template <int HD, int GQ>
  __device__ bool attention(int ph, const PLayer& L) {
    constexpr int DPL = HD / 32;
    constexpr int PPW = kPAttnSub / kPWarps;  // cache slots per warp per stage
    constexpr int NV = (PPW * GQ < 32) ? PPW * GQ : 32;
    constexpr int ROUNDS = (PPW * GQ + 31) / 32;
    constexpr int PR = NV / GQ;
    constexpr int LOG_NV = (NV == 4) ? 2 : (NV == 8) ? 3 : (NV == 16) ? 4 : 5;
    static_assert(PPW * kPWarps == kPAttnSub, "stage slots must split evenly over the warps");
    int S, chunk;
    attn_slicing(a.kv_len, a.n_kv, gridDim.x, S, chunk);
    const float rsq = sqrtf((float)HD);
    float qr[GQ][DPL];
    float m_run[GQ], l_w[GQ], o_w[GQ][DPL];
    int j = 0;
    while (true) {
      const int slot = next_slot();
      if (slot < 0) return false;
      const volatile int* tg = tag + slot * 4;
      const int tph = tg[0], item = tg[1], c0 = tg[2], flags = tg[3];
      if (tph != ph) {
        give_up(a, kStatusBadArgs, s_abort);
        return false;
      }
      if (flags & kFlagEmpty) {
        release(slot);
        ++i;
        break;
      }
      const int g = item % a.n_kv, sidx = item / a.n_kv;
      const int t1 = min(a.kv_len, sidx * chunk + chunk);
      const int cn = min(kPAttnSub, t1 - c0);
      if (flags & kFlagItemFirst) {
#pragma unroll
        for (int h = 0; h < GQ; ++h) {
#pragma unroll
          for (int d = 0; d < DPL; ++d) qr[h][d] = __ldcg(a.q + (size_t)(g * GQ + h) * HD + lane * DPL + d);
          m_run[h] = -INFINITY;
          l_w[h] = 0.f;
#pragma unroll
          for (int d = 0; d < DPL; ++d) o_w[h][d] = 0.f;
        }
      }
      unsigned char* base = sm.ring + (size_t)slot * kPSlotBytes;
      __half* Ks = reinterpret_cast<__half*>(base);
      __half* Vs = reinterpret_cast<__half*>(base + (size_t)kPAttnSub * HD * 2);
      // Rows this step wrote (the new slot, re-rotated sinks) may have been staged before the QKV
      // phase stored them: take them from global memory.
      for (int e = t; e < 3 * (HD / 8); e += NT) {
        const int which = e / (HD / 8), part = e % (HD / 8);
        const int slot_pos = which == 0 ? a.kv_pos : which - 1;
        if (which > 0 && which - 1 >= a.kv_sink) continue;
        if (slot_pos < c0 || slot_pos >= c0 + cn) continue;
        const size_t goff = ((size_t)g * a.max_seq_len + slot_pos) * HD + part * 8;
        const size_t soff = (size_t)(slot_pos - c0) * HD + part * 8;
        *reinterpret_cast<uint4*>(Ks + soff) = __ldcg(reinterpret_cast<const uint4*>(L.k_cache + goff));
        *reinterpret_cast<uint4*>(Vs + soff) = __ldcg(reinterpret_cast<const uint4*>(L.v_cache + goff));
        fence_proxy_async_smem();
      }
      named_sync(1, NT);
      float* Sj = sm.S + (j & 1) * GQ * kPAttnSub;
      float sc[ROUNDS];
#pragma unroll
      for (int r = 0; r < ROUNDS; ++r) {
        float part[NV];
#pragma unroll
        for (int ii = 0; ii < PR; ++ii) {
          const int p = warp * PPW + r * PR + ii;
          float kf[DPL];
#pragma unroll
          for (int d = 0; d < DPL; ++d) kf[d] = 0.f;
          if (p < cn) {
            if (DPL == 4) {
              const uint2 raw = *reinterpret_cast<const uint2*>(Ks + (size_t)p * HD + lane * 4);
              const float2 a0 = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
              const float2 a1 = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
              kf[0] = a0.x; kf[1 % DPL] = a0.y; kf[2 % DPL] = a1.x; kf[3 % DPL] = a1.y;
            } else {
              const float2 a0 = __half22float2(*reinterpret_cast<const __half2*>(Ks + (size_t)p * HD + lane * 2));
              kf[0] = a0.x; kf[1 % DPL] = a0.y;
            }
          }
#pragma unroll
          for (int h = 0; h < GQ; ++h) {
            float acc = 0.f;
#pragma unroll
            for (int d = 0; d < DPL; ++d) acc = fmaf(qr[h][d], kf[d], acc);
            part[ii * GQ + h] = acc;
          }
        }
        const float tot = warp_reduce_scatter<NV>(part, lane);
        const int idx = lane >> (5 - LOG_NV);
        const int p = warp * PPW + r * PR + idx / GQ;
        sc[r] = (p < cn) ? tot / rsq : -INFINITY;
        if ((lane & ((32 >> LOG_NV) - 1)) == 0) Sj[(idx % GQ) * kPAttnSub + p] = sc[r];
      }
      named_sync(1, NT);
      float m_new[GQ];
#pragma unroll
      for (int h = 0; h < GQ; ++h) {
        const float mx = warp_max(fmaxf(Sj[h * kPAttnSub + lane], Sj[h * kPAttnSub + lane + 32]));
        m_new[h] = fmaxf(m_run[h], mx);
        const float alpha = expf(m_run[h] - m_new[h]);
        m_run[h] = m_new[h];
        l_w[h] *= alpha;
#pragma unroll
        for (int d = 0; d < DPL; ++d) o_w[h][d] *= alpha;
      }
      float pv[ROUNDS];
#pragma unroll
      for (int r = 0; r < ROUNDS; ++r) {
        const int h = (lane >> (5 - LOG_NV)) % GQ;
        float mh = m_new[0];
#pragma unroll
        for (int hh = 0; hh < GQ; ++hh)
          if (hh == h) mh = m_new[hh];
        pv[r] = (sc[r] == -INFINITY) ? 0.f : expf(sc[r] - mh);
      }
#pragma unroll
      for (int r = 0; r < ROUNDS; ++r) {
#pragma unroll
        for (int ii = 0; ii < PR; ++ii) {
          const int p = warp * PPW + r * PR + ii;
          float vf[DPL];
#pragma unroll
          for (int d = 0; d < DPL; ++d) vf[d] = 0.f;
          const bool valid = p < cn;
          if (valid) {
            if (DPL == 4) {
              const uint2 raw = *reinterpret_cast<const uint2*>(Vs + (size_t)p * HD + lane * 4);
              const float2 a0 = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
              const float2 a1 = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
              vf[0] = a0.x; vf[1 % DPL] = a0.y; vf[2 % DPL] = a1.x; vf[3 % DPL] = a1.y;
            } else {
              const float2 a0 = __half22float2(*reinterpret_cast<const __half2*>(Vs + (size_t)p * HD + lane * 2));
              vf[0] = a0.x; vf[1 % DPL] = a0.y;
            }
          }
#pragma unroll
          for (int h = 0; h < GQ; ++h) {
            const float ph2 = __shfl_sync(0xffffffffu, pv[r], ((ii * GQ + h) << (5 - LOG_NV)));
            if (valid) {
              l_w[h] += ph2;
#pragma unroll
              for (int d = 0; d < DPL; ++d) o_w[h][d] = fmaf(ph2, vf[d], o_w[h][d]);
            }
          }
        }
      }
      ++i;
      ++j;
      if (!(flags & kFlagItemLast)) {
        release(slot);
        continue;
      }
      // end of an item: combine the warps (identical running max) inside this slot, HPP heads at a
      // time so [warps][HPP][HD] floats fit the slot
      constexpr int HPP = (kPWarps * GQ * HD * 4 <= kPSlotBytes) ? GQ : (kPSlotBytes / (kPWarps * HD * 4));
      static_assert(HPP >= 1 && GQ % HPP == 0, "combine does not fit a ring slot");
      named_sync(1, NT);
      float* red = reinterpret_cast<float*>(base);  // [warps][HPP][HD]
      if (lane == 0) {
#pragma unroll
        for (int h = 0; h < GQ; ++h) sm.scratch[warp * GQ + h] = l_w[h];
      }
#pragma unroll
      for (int h0 = 0; h0 < GQ; h0 += HPP) {
#pragma unroll
        for (int hh = 0; hh < HPP; ++hh) {
#pragma unroll
          for (int d = 0; d < DPL; ++d) red[(warp * HPP + hh) * HD + lane * DPL + d] = o_w[h0 + hh][d];
        }
        named_sync(1, NT);
        for (int e = t; e < HPP * HD; e += NT) {
          const int hh = e / HD, d = e % HD, h = h0 + hh;
          float sum = 0.f, l = 0.f;
#pragma unroll
          for (int w = 0; w < kPWarps; ++w) {
            sum += red[(w * HPP + hh) * HD + d];
            l += sm.scratch[w * GQ + h];
          }
          const int hq = g * GQ + h;
          if (S == 1) {
            __stcg(a.att + (size_t)hq * HD + d, sum / l);
          } else {
            float* pp = a.attn_part + ((size_t)hq * kPMaxSplits + sidx) * (HD + 2);
            __stcg(pp + d, sum);
            if (d == 0) {
              float mh = m_run[0];
#pragma unroll
              for (int k2 = 0; k2 < GQ; ++k2)
                if (k2 == h) mh = m_run[k2];
              __stcg(pp + HD, mh);
              __stcg(pp + HD + 1, l);
            }
          }
        }
        named_sync(1, NT);
      }
      fence_proxy_async_smem();  // the combine wrote into the slot the producer refills next
      named_sync(1, NT);
      release(slot);
      if (S > 1) {
        __threadfence();
        named_sync(1, NT);
        if (t == 0) *s_flag = (atomicAdd(&a.attn_cnt[g], 1u) == (unsigned)(S - 1));
        named_sync(1, NT);
        if (*s_flag) {  // last slice of this kv head: log-sum-exp merge of the S slices
          __threadfence();
          for (int e = t; e < GQ * HD; e += NT) {
            const int h = e / HD, d = e % HD;
            const float* pb = a.attn_part + (size_t)(g * GQ + h) * kPMaxSplits * (HD + 2);
            float ms[kPMaxSplits];
            float M = -INFINITY;
#pragma unroll
            for (int s2 = 0; s2 < kPMaxSplits; ++s2) {
              ms[s2] = s2 < S ? __ldcg(pb + (size_t)s2 * (HD + 2) + HD) : -INFINITY;
              M = fmaxf(M, ms[s2]);
            }
            float O = 0.f, Lsum = 0.f;
#pragma unroll
            for (int s2 = 0; s2 < kPMaxSplits; ++s2) {
              if (s2 < S) {
                const float wgt = expf(ms[s2] - M);
                O = fmaf(wgt, __ldcg(pb + (size_t)s2 * (HD + 2) + d), O);
                Lsum = fmaf(wgt, __ldcg(pb + (size_t)s2 * (HD + 2) + HD + 1), Lsum);
              }
            }
            __stcg(a.att + (size_t)(g * GQ + h) * HD + d, O / Lsum);
          }
          if (t == 0) a.attn_cnt[g] = 0u;
        }
        named_sync(1, NT);
      }
      if (flags & kFlagLastOfPhase) break;
    }
    return true;
  }
};

template <int KD, int RD, int KO, int RO, int KH, int RH, int HD, int GQ>
__global__ void __launch_bounds__(kPThreads, 1) persistent_step_kernel(const PArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ int s_abort, s_flag;
  __shared__ int s_tag[kPSlots * 4];
  PSmem sm;
  sm.ring = smem;
  sm.red = reinterpret_cast<float*>(smem + (size_t)kPSlots * kPSlotBytes);
  sm.S = sm.red + a.red_floats;
  sm.scratch = sm.S + 2 * 8 * kPAttnSub;
  sm.full = reinterpret_cast<uint64_t*>(sm.scratch + 256);
  sm.empty = sm.full + kPSlots;
  int* mine = reinterpret_cast<int*>(sm.empty + kPSlots);
  unsigned* ctr = reinterpret_cast<unsigned*>(a.bar + 1) + 1;  // per-phase claim counters
  if (threadIdx.x == 0) {
    s_abort = 0;
    s_flag = 0;
    for (int k = 0; k < kPSlots; ++k) {
      mbar_init(&sm.full[k], 1);
      mbar_init(&sm.empty[k], kPWarps);
    }
    mbar_fence_init();
  }
  __syncthreads();

  if ((threadIdx.x >> 5) == kPWarps) {
    if ((threadIdx.x & 31) == 0) {
      Producer p(a, sm, &s_abort, s_tag, ctr);
      p.template run<RD, RO, RH, HD>();
      p.drain();
      stamp(a, kTraceEvents - 1);
    }
    return;
  }

  Consumer c(a, sm, &s_abort, &s_flag, s_tag, mine);
  if (threadIdx.x == 0) stamp(a, 0);
  bool ok = true;
  for (int l = 0; l < a.n_layers && ok; ++l) {
    const PLayer L = a.layers[l];
    const int ph = 5 * l;
    ok = c.template qkv<KD, RD>(ph, L, l) && c.grid_sync() &&
         c.template attention<HD, GQ>(ph + 1, L) && c.grid_sync() &&
         c.template resid<KO, RO>(ph + 2, a.q_rows, a.att, a.x) && c.grid_sync() &&
         c.template gateup<KD, RD>(ph + 3, L) && c.grid_sync() &&
         c.template resid<KH, RH>(ph + 4, a.hid, a.hb, a.x) && c.grid_sync();
  }
  if (ok && a.mode) c.template classifier<KD, RD>(5 * a.n_layers);
  if (threadIdx.x == 0) stamp(a, kTraceEvents - 2);
}

struct Inst {
  int kd, rd, ko, ro, kh, rh, hd, gq;
  const void* fn;
};

#define YB_PINST(KD, RD, KO, RO, KH, RH, HD, GQ) \
  {KD, RD, KO, RO, KH, RH, HD, GQ, reinterpret_cast<const void*>(&persistent_step_kernel<KD, RD, KO, RO, KH, RH, HD, GQ>)}

// Shapes with an instantiation (per tensor-parallel rank):
//   tiny (dim 512, hidden 1408, head_dim 64, 4 q / kv) at TP 1-2;
//   Mistral-7B (dim 4096, hidden 14336, head_dim 128, GQ 4) at TP 1, 2, 4, 8;
//   70B-class (dim 8192, hidden 28672, GQ 8) at TP 2, 4, 8.
const Inst kInsts[] = {
    YB_PINST(1, 8, 1, 8, 1, 8, 64, 4),
    YB_PINST(1, 4, 1, 4, 4, 1, 128, 4),
    YB_PINST(1, 4, 1, 8, 2, 2, 128, 4),
    YB_PINST(1, 4, 1, 8, 1, 4, 128, 4),
    YB_PINST(1, 4, 1, 8, 1, 8, 128, 4),
    YB_PINST(2, 2, 1, 4, 4, 1, 128, 8),
    YB_PINST(2, 2, 1, 8, 2, 2, 128, 8),
    YB_PINST(2, 2, 1, 8, 1, 4, 128, 8),
};

// 16-byte column chunks per consumer thread for a row of `cols` fp16 values
int chunks_per_thread(int cols) {
  const int chunks = cols / 8;
  const int per = (chunks + kPWarps * 32 - 1) / (kPWarps * 32);
  if (per <= 1) return 1;
  if (per <= 2) return 2;
  if (per <= 4) return 4;
  if (per <= 7) return 7;
  return -1;
}

int rows_per_stage(int cols, bool pairs) {
  int rt = 1;
  while (rt < 8 && (rt * 2) * cols * 2 <= kPSlotBytes) rt *= 2;
  if (cols * 2 * rt > kPSlotBytes) return -1;
  if (pairs && rt < 2) return -1;
  return rt;
}

}  // namespace

PersistPlan persist_plan(int dim, int q_rows, int hid, int head_dim, int gq, int n_sms) {
  PersistPlan p{};
  p.ok = false;
  p.kd = chunks_per_thread(dim);
  p.rd = rows_per_stage(dim, true);
  p.ko = chunks_per_thread(q_rows);
  p.ro = rows_per_stage(q_rows, false);
  p.kh = chunks_per_thread(hid);
  p.rh = rows_per_stage(hid, false);
  if (dim % 8 || q_rows % 8 || hid % 8 || p.kd < 0 || p.ko < 0 || p.kh < 0 || p.rd < 0 || p.ro < 0 || p.rh < 0)
    return p;
  if (head_dim * kPAttnSub * 2 * 2 > kPSlotBytes) return p;
  for (const Inst& in : kInsts) {
    if (in.kd == p.kd && in.rd == p.rd && in.ko == p.ko && in.ro == p.ro && in.kh == p.kh && in.rh == p.rh &&
        in.hd == head_dim && in.gq == gq) {
      p.fn = in.fn;
      p.grid = n_sms;
      p.ok = true;
      return p;
    }
  }
  return p;
}

int persist_max_local(int rows, int rt, int grid, int static_pct) {
  const int T = (rows + rt - 1) / rt;
  if (static_pct >= 100) return (T + grid - 1) / grid;
  int q = (int)((long long)T * static_pct / (100ll * grid));
  if (q * grid > T) q = T / grid;
  const int R = T - grid * q;
  return q + 2 * ((R + grid - 1) / grid) + 1;
}

size_t persist_smem_bytes(int red_floats, int max_local) {
  return (size_t)kPSlots * kPSlotBytes + (size_t)red_floats * 4 + 2 * 8 * kPAttnSub * 4 + 256 * 4 + 2 * kPSlots * 8 +
         (size_t)max_local * 4;
}

cudaError_t persist_prepare(const PersistPlan& p) { return raise_smem_cap(p.fn); }

cudaError_t persist_launch(const PersistPlan& p, const PArgs& a, cudaStream_t stream) {
  PArgs args = a;
  void* params[] = {&args};
  return cudaLaunchCooperativeKernel(p.fn, dim3(p.grid), dim3(kPThreads), params,
                                     persist_smem_bytes(a.red_floats, a.max_local), stream);
}

}  // namespace yb
