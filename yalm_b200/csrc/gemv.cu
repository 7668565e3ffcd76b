// Weight-streaming GEMV kernels (see gemv.cuh for the design).
#include "gemv.cuh"
#include "launch.h"

#include <cstdio>
#include <cstdlib>
#include <string>

namespace yb {

// IN: 0 = x as given, 1 = RMS-normalised x, 2 = RMS-normalised x plus the tensor-parallel partial
// sums of the previous row-parallel matvec (GemvArgs::tp_ll).  Only IN == 2 instances carry the
// exchange-read code, so the others keep their registers for the stream loop.
// WT: weight type, 0 = fp16, 1 = fp8 E5M2 (the top byte of an fp16) on the CUDA cores, 2 = fp8 E5M2
// on the tensor cores.  A 16-byte chunk of a row holds EPC = 8 or 16 weights; thread t owns the
// chunks t, t + NT, ... and the matching EPC values of x for the input prologue.
//
// WT = 2 reads the matrix in the grouped layout fp8_group_layout writes at upload: 16-row groups,
// each stored as [16-column chunk][row][16 bytes], so that a stage (a group's chunk of up to
// kMmaCols columns) is one contiguous bulk copy and the 8 rows an ldmatrix reads are 128 consecutive
// bytes (no bank conflicts).  Warp w takes the chunk's columns [w kMmaCols / NW, ...).  The input x
// is staged in shared memory as fp16 value and remainder planes; per 16 columns one
// mma.sync.m16n8k16 (fp32 accumulate) takes A = the 16 weight rows, whose e5m2 bytes become fp16
// exactly by a byte permute, and B = x with column 0 its values and column 1 its remainders
// (columns 2-7 zero).  The k order inside each 16 columns is permuted the same way in A and B (lane
// c holds columns 4c .. 4c + 3, the 4 bytes one ldmatrix lane receives), which leaves every dot
// product unchanged.  Products are exact (value + remainder carry ~22 bits of x); value and
// remainder sums meet at the group's last chunk and go to the cross-warp reduction as the CUDA-core
// path's do.
constexpr int kMmaCols = 1024;  // fp8 columns (bytes) of a row per stage, WT = 2
constexpr int kMmaRows = 16;    // rows per group (the mma's M), WT = 2
template <int NW, int KPT, int RT, int EPI, int IN, int WT>
__global__ void __launch_bounds__((NW + 1) * 32, 2) yb_stream_matvec(const GemvArgs a) {
  constexpr bool NORM = IN >= 1;
  constexpr bool TPIN = IN == 2;
  constexpr int EPC = WT ? 16 : 8;  // weights (and x values) per 16-byte chunk
  constexpr int V = EPC / 4;        // float4 of x per chunk
  extern __shared__ __align__(128) unsigned char smem[];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  constexpr int NT = NW * 32;  // consumer threads

  pdl_trigger();
  if (threadIdx.x == 0) timeline_stamp(a.trace, a.trace_stride, 0);

  constexpr bool MMA = WT == 2;
  const int C = a.cols;
  // units of RT rows: one stage each, or (tensor cores) NC column-chunk stages each
  const int NC = MMA ? (C + kMmaCols - 1) / kMmaCols : 1;
  const int T = (a.rows + RT - 1) / RT;
  const int G = gridDim.x;
  const int s_begin = (int)((long long)T * blockIdx.x / G);
  const int s_end = (int)((long long)T * (blockIdx.x + 1) / G);
  const int n_units = s_end - s_begin;
  const int n_st = n_units * NC;
  const int row_begin = s_begin * RT;
  const int NS = a.n_slots;
  const unsigned SB = a.stage_bytes;
  const unsigned row_bytes = (unsigned)C * (WT ? 1u : 2u);

  unsigned char* ring = smem;
  float* red = reinterpret_cast<float*>(smem + (size_t)NS * SB);
  float* scratch = red + a.red_floats;                    // NW floats for the norm reduction
  uint64_t* full = reinterpret_cast<uint64_t*>(scratch + 32);
  uint64_t* empty = full + NS;
  // WT = 2: x as fp16 value and remainder planes, C each, 16-byte aligned after the barriers
  __half* xs_hi = reinterpret_cast<__half*>((reinterpret_cast<uintptr_t>(empty + NS) + 15) & ~uintptr_t(15));
  __half* xs_lo = xs_hi + C;
  __shared__ int s_abort;

  if (threadIdx.x == 0) {
    s_abort = 0;
    for (int i = 0; i < NS; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], NW);
    }
    mbar_fence_init();
  }
  __syncthreads();

  if (warp == NW) {
    // ------------------------------------------------------------------ producer
    if (lane != 0 || n_st <= 0) return;
    const uint64_t pol = l2_evict_first_policy();
    const unsigned char* wbase = reinterpret_cast<const unsigned char*>(a.w);
    const bool contiguous = (a.ldw == (long long)C);
    // Warm L2 with the stages just beyond the ring: weights are static, so this (like the ring
    // fill below) may run before the previous kernel of the step has finished.
    if (!MMA && contiguous && a.l2_prefetch_stages > 0) {
      int pf_end = min(n_st, NS + a.l2_prefetch_stages);
      for (int i = NS; i < pf_end; ++i) {
        int row0 = row_begin + i * RT;
        int nr = min(RT, a.rows - row0);
        bulk_prefetch_l2(wbase + (size_t)row0 * row_bytes, (unsigned)nr * row_bytes);
      }
    }
    int issued = 0;
    for (int i = 0; i < n_st; ++i) {
      const int slot = i % NS;
      if (i >= NS) {
        if (!mbar_wait(&empty[slot], ((i / NS) - 1) & 1, a.status)) {
          s_abort = 1;
          break;
        }
      }
      unsigned char* dst = ring + (size_t)slot * SB;
      if (MMA) {
        // group s_begin + i / NC, column chunk i % NC: contiguous in the grouped layout (groups
        // ldw * 16 bytes apart, 16-column chunks 256 bytes apart)
        const int j = i % NC;
        const int ccb = min(kMmaCols, C - j * kMmaCols);
        const unsigned char* src =
            wbase + (size_t)(s_begin + i / NC) * (size_t)a.ldw * kMmaRows + (size_t)j * kMmaCols * kMmaRows;
        mbar_arrive_expect_tx(&full[slot], (unsigned)(kMmaRows * ccb));
        bulk_g2s(dst, src, (unsigned)(kMmaRows * ccb), &full[slot], pol);
      } else {
        const int row0 = row_begin + i * RT;
        const int nr = min(RT, a.rows - row0);
        mbar_arrive_expect_tx(&full[slot], (unsigned)nr * row_bytes);
        if (contiguous) {
          bulk_g2s(dst, wbase + (size_t)row0 * row_bytes, (unsigned)nr * row_bytes, &full[slot], pol);
        } else {
          for (int r = 0; r < nr; ++r)
            bulk_g2s(dst + (size_t)r * row_bytes, wbase + (size_t)(row0 + r) * (size_t)a.ldw * (WT ? 1u : 2u),
                     row_bytes, &full[slot], pol);
        }
      }
      issued = i + 1;
      if (EPI == kEpiQKV && a.kv_prefetch && a.step && i + 1 == min(NS, n_st)) {
        // this CTA's share of the K/V cache rows the attention kernel will read; the step state
        // may still be the previous step's (a prefetch only)
        int hl = *reinterpret_cast<const volatile int*>(&a.step->kv_len);
        hl = hl < 1 ? 1 : (hl > a.max_seq_len ? a.max_seq_len : hl);
        const long long per = (long long)hl * a.head_dim * 2;  // bytes per head, K or V
        const int n_kv = a.kv_rows / a.head_dim;
        const long long total = 2ll * n_kv * per;
        long long o = (total * blockIdx.x / G) & ~15ll;
        const long long end = (blockIdx.x + 1 == G) ? total : ((total * (blockIdx.x + 1) / G) & ~15ll);
        while (o < end) {
          const long long seg = o / per, off = o - seg * per;
          const __half* base = (seg < n_kv ? a.k_cache : a.v_cache) + (size_t)(seg % n_kv) * a.max_seq_len * a.head_dim;
          long long n = per - off < end - o ? per - off : end - o;
          if (n > 65536) n = 65536;
          bulk_prefetch_l2(reinterpret_cast<const unsigned char*>(base) + off, (unsigned)n);
          o += n;
        }
      }
      if (i + 1 == NS && a.pf_src) {
        // this CTA's share of the L2 warm-up, after its own ring is in flight
        long long p0 = a.pf_bytes * blockIdx.x / G, p1 = a.pf_bytes * (blockIdx.x + 1) / G;
        p0 &= ~15ll;
        p1 = (blockIdx.x + 1 == G) ? a.pf_bytes : (p1 & ~15ll);
        for (long long o = p0; o < p1; o += 65536) {
          const long long n = (p1 - o) < 65536 ? (p1 - o) : 65536;
          bulk_prefetch_l2(a.pf_src + o, (unsigned)n);
        }
      }
    }
    // Drain: never leave the CTA while a bulk copy into its shared memory may be in flight.
    for (int i = max(0, issued - NS); i < issued; ++i) mbar_wait(&full[i % NS], (i / NS) & 1, a.status);
    return;
  }

  // -------------------------------------------------------------------- consumers
  const int t = threadIdx.x;  // 0 .. NT-1
  const int n_chunks = C / EPC;
  float4 xr[KPT][V];
  float4 nw[NORM ? KPT : 1][V];
  if (NORM) {
#pragma unroll
    for (int k = 0; k < KPT; ++k) {
      const int c = k * NT + t;
      if (c < n_chunks) {
#pragma unroll
        for (int v = 0; v < V; ++v) nw[k][v] = __ldg(reinterpret_cast<const float4*>(a.norm_w) + V * c + v);
      }
    }
  }

  pdl_wait();  // activations below are produced by the previous kernel of the step

  const float* xin = a.x;
  if (TPIN && a.tp_ll) {
    // Tensor-parallel all-reduce of the previous row-parallel matvec, in two parts.
    // (1) This CTA's share of x (chunks [w_begin, w_end)): the residual plus every rank's partial,
    //     added in rank order (the same order on every rank, so all ranks hold bit-identical x),
    //     each partial read once its exchange word carries this step's epoch; written to x_out.
    // (2) A barrier over this kernel's CTAs (all resident: the grid is at most one CTA per slot),
    //     after which every CTA reads the whole new x from x_out.  Each CTA so reads P words per
    //     element of its share instead of P words per element of x.
    const unsigned ep = a.step->epoch;
    const int w_begin = (int)((long long)n_chunks * blockIdx.x / G);
    const int w_end = (int)((long long)n_chunks * (blockIdx.x + 1) / G);
    bool ok = true;
    for (int e = w_begin * EPC + t; e < w_end * EPC; e += NT) {
      float v = a.x[e];
      for (int r0 = 0; r0 < a.tp_size && ok; r0 += 8) {
        const int nr = min(8, a.tp_size - r0);
        unsigned long long w[8];
        long long t0 = 0;
        for (bool first = true;; first = false) {
          bool ready = true;
#pragma unroll
          for (int j = 0; j < 8; ++j)
            if (j < nr)
              asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(w[j]) : "l"(a.tp_ll + (size_t)(r0 + j) * C + e) : "memory");
#pragma unroll
          for (int j = 0; j < 8; ++j)
            if (j < nr) ready = ready && (unsigned)(w[j] >> 32) == ep;
          if (ready) break;
          if (first) {
            t0 = clock64();
          } else if (clock64() - t0 > kWaitBudgetCycles) {
            atomicOr(a.status, kStatusPeerTimeout);
            ok = false;
            break;
          }
          __nanosleep(100);
        }
        if (ok) {
#pragma unroll
          for (int j = 0; j < 8; ++j)
            if (j < nr) v += __uint_as_float((unsigned)w[j]);
        }
      }
      a.x_out[e] = v;
    }
    if (!ok) s_abort = 1;
    named_sync(1, NT);
    if (t == 0) {
      // release this CTA's share, then wait (bounded) for every CTA's
      asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(a.tp_bar) : "memory");
      long long t0 = clock64();
      unsigned seen;
      do {
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(seen) : "l"(a.tp_bar) : "memory");
        if ((int)(seen - (unsigned)G) >= 0) break;
        if (clock64() - t0 > kWaitBudgetCycles) {
          atomicOr(a.status, kStatusPeerTimeout);
          s_abort = 1;
          break;
        }
        __nanosleep(64);
      } while (true);
    }
    named_sync(1, NT);
    xin = a.x_out;
    if (t == 0) timeline_stamp(a.trace, a.trace_stride, 2);
  }
#pragma unroll
  for (int k = 0; k < KPT; ++k) {
    const int c = k * NT + t;
#pragma unroll
    for (int v = 0; v < V; ++v) {
      if (c < n_chunks) {
        if (TPIN && a.tp_ll)  // written by other CTAs of this kernel: read through L2
          xr[k][v] = __ldcg(reinterpret_cast<const float4*>(xin) + V * c + v);
        else
          xr[k][v] = reinterpret_cast<const float4*>(xin)[V * c + v];
      } else {
        xr[k][v] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
  }
  if (t == 0) timeline_stamp(a.trace, a.trace_stride, 1);
  if (NORM) {
    // RMSNorm (yalm src/infer.cpp:136-146): scale = 1 / sqrt(mean(x^2) + eps); x * scale * w
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < KPT; ++k)
#pragma unroll
      for (int v = 0; v < V; ++v)
        ss += xr[k][v].x * xr[k][v].x + xr[k][v].y * xr[k][v].y + xr[k][v].z * xr[k][v].z + xr[k][v].w * xr[k][v].w;
    ss = warp_sum(ss);
    if (lane == 0) scratch[warp] = ss;
    named_sync(1, NT);
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) tot += scratch[w];
    const float rms = sqrtf(tot / (float)C + a.eps);
    const float scale = 1.0f / rms;
#pragma unroll
    for (int k = 0; k < KPT; ++k) {
      const int c = k * NT + t;
      if (c < n_chunks) {
#pragma unroll
        for (int v = 0; v < V; ++v) {
          xr[k][v].x = xr[k][v].x * scale * nw[k][v].x;
          xr[k][v].y = xr[k][v].y * scale * nw[k][v].y;
          xr[k][v].z = xr[k][v].z * scale * nw[k][v].z;
          xr[k][v].w = xr[k][v].w * scale * nw[k][v].w;
        }
      }
    }
  }

  constexpr int LOG_RT = (RT == 1) ? 0 : (RT == 2) ? 1 : (RT == 4) ? 2 : 3;
  if constexpr (MMA) {
    static_assert(RT == kMmaRows, "the tensor-core path folds 16-row groups (the mma's M)");
    // x -> fp16 value and remainder planes in shared memory (this thread's chunks)
#pragma unroll
    for (int k = 0; k < KPT; ++k) {
      const int c = k * NT + t;
      if (c < n_chunks) {
        uint32_t hv[8], lv[8];
#pragma unroll
        for (int v = 0; v < V; ++v) {
          split_f16x2(xr[k][v].x, xr[k][v].y, hv[2 * v], lv[2 * v]);
          split_f16x2(xr[k][v].z, xr[k][v].w, hv[2 * v + 1], lv[2 * v + 1]);
        }
        uint4* ph = reinterpret_cast<uint4*>(xs_hi + (size_t)c * EPC);
        uint4* pl = reinterpret_cast<uint4*>(xs_lo + (size_t)c * EPC);
        ph[0] = make_uint4(hv[0], hv[1], hv[2], hv[3]);
        ph[1] = make_uint4(hv[4], hv[5], hv[6], hv[7]);
        pl[0] = make_uint4(lv[0], lv[1], lv[2], lv[3]);
        pl[1] = make_uint4(lv[4], lv[5], lv[6], lv[7]);
      }
    }
    named_sync(1, NT);
    // B: lanes 0-3 hold column 0 (values of x), lanes 4-7 column 1 (remainders); the rest is zero
    const int g = lane >> 2, c4 = lane & 3;
    const uint32_t xsrc = smem_u32(g == 0 ? xs_hi : xs_lo) + 8u * (uint32_t)c4;
    constexpr int WCOLS = kMmaCols / NW;  // columns of a chunk per warp
    float d[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    for (int i = 0; i < n_st; ++i) {
      const int slot = i % NS;
      if (!mbar_wait(&full[slot], (i / NS) & 1, a.status)) {
        s_abort = 1;
        break;
      }
      if (*(volatile int*)&s_abort) break;
      const int j = i % NC;
      const int ccb = min(kMmaCols, C - j * kMmaCols);
      const uint32_t st = smem_u32(ring + (size_t)slot * SB);
#pragma unroll
      for (int q = 0; q < WCOLS / 32; ++q) {
        const int kb = warp * WCOLS + q * 32;  // 2 k-steps of 16 columns
        if (kb < ccb) {
          uint32_t r[4];
          // matrix m = lane / 8: rows 8 (m & 1) .., k-step kb / 16 + (m >> 1); its row lane % 8
          ldsm_x4(r, st + (uint32_t)((kb / 16 + (lane >> 4)) * 256 + (8 * ((lane >> 3) & 1) + (lane & 7)) * 16));
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            if (kb + 16 * h < ccb) {
              uint32_t A[4];
              A[0] = __byte_perm(r[2 * h], 0u, 0x1404u);      // row g, columns 4c, 4c + 1
              A[1] = __byte_perm(r[2 * h + 1], 0u, 0x1404u);  // row g + 8
              A[2] = __byte_perm(r[2 * h], 0u, 0x3424u);      // row g, columns 4c + 2, 4c + 3
              A[3] = __byte_perm(r[2 * h + 1], 0u, 0x3424u);  // row g + 8
              uint32_t b0 = 0u, b1 = 0u;
              if (g < 2) {
                const uint32_t xa = xsrc + 2u * (uint32_t)(j * kMmaCols + kb + 16 * h);
                asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(b0), "=r"(b1) : "r"(xa));
              }
              mma_16816(d[h], A, b0, b1);
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
      if (j == NC - 1) {
        // the group is complete: lanes c4 = 0 hold rows g and g + 8, value (column 0) and
        // remainder (column 1) sums
        const int u = i / NC;
        if (c4 == 0) {
          red[(u * RT + g) * NW + warp] = (d[0][0] + d[1][0]) + (d[0][1] + d[1][1]);
          red[(u * RT + g + 8) * NW + warp] = (d[0][2] + d[1][2]) + (d[0][3] + d[1][3]);
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) d[h][0] = d[h][1] = d[h][2] = d[h][3] = 0.f;
      }
    }
  } else
  for (int i = 0; i < n_st; ++i) {
    const int slot = i % NS;
    if (!mbar_wait(&full[slot], (i / NS) & 1, a.status)) {
      s_abort = 1;
      break;
    }
    if (*(volatile int*)&s_abort) break;
    const unsigned char* st = ring + (size_t)slot * SB;
    const int nr = min(RT, a.rows - (row_begin + i * RT));
    // all shared-memory loads of the stage first, then independent per-chunk dot products
    float acc[RT];
#pragma unroll
    for (int r = 0; r < RT; ++r) {
      uint4 wv[KPT];
#pragma unroll
      for (int k = 0; k < KPT; ++k) {
        const int c = k * NT + t;
        wv[k] = (r < nr && c < n_chunks) ? lds128(st + (size_t)r * row_bytes + (size_t)c * 16) : make_uint4(0, 0, 0, 0);
      }
      float part[KPT];
#pragma unroll
      for (int k = 0; k < KPT; ++k) {
        if (WT)
          part[k] = dot16_e5m2(wv[k], xr[k][0], xr[k][1], xr[k][V > 2 ? 2 : 0], xr[k][V > 2 ? 3 : 1]);
        else
          part[k] = dot8(wv[k], xr[k][0], xr[k][1]);
      }
      float s = part[0];
#pragma unroll
      for (int k = 1; k < KPT; ++k) s += part[k];
      acc[r] = s;
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
    const float v = warp_reduce_scatter<RT>(acc, lane);
    const int rr = lane >> (5 - LOG_RT);
    if ((lane & ((32 >> LOG_RT) - 1)) == 0 && rr < nr) red[(i * RT + rr) * NW + warp] = v;
  }
  named_sync(1, NT);
  if (s_abort) return;
  if (t == 0) timeline_stamp(a.trace, a.trace_stride, 3);

  // -------------------------------------------------------------------- epilogue
  const int n_rows = min(n_units * RT, a.rows - row_begin);
  if (EPI == kEpiStore || EPI == kEpiResid || EPI == kEpiResidTP || EPI == kEpiStoreTP) {
    for (int lr = t; lr < n_rows; lr += NT) {
      float s = 0.f;
#pragma unroll
      for (int w = 0; w < NW; ++w) s += red[lr * NW + w];
      const int row = row_begin + lr;
      if (EPI == kEpiStore) {
        a.y[row] = s;
      } else if (EPI == kEpiResid) {
        a.y[row] += s;
      } else if (EPI == kEpiResidTP) {
        // tensor parallel: this rank's partial for `row`, tagged with the epoch, to every rank
        const unsigned ep = a.step->epoch;
        for (int p = 0; p < a.tp_size; ++p) st_ll(a.peer_ll[p] + row, s, ep);
      } else {
        // tensor-parallel logits: this rank's rows go to every rank's buffer
        for (int p = 0; p < a.tp_size; ++p) a.peer_slots[p][a.row_offset + row] = s;
      }
    }
    if (EPI == kEpiStoreTP) {
      // Publish: once every consumer thread has issued its peer stores, one thread per peer bumps
      // that peer's arrival counter with a system-scope release, which orders all of the CTA's
      // stores before the counter moves.
      named_sync(1, NT);
      if (t < a.tp_size) red_release_sys_add(a.peer_counters[t], 1u);
    }
  } else if (EPI == kEpiGateUp) {
    // rows (2j, 2j+1) = (w1 row j, w3 row j); yalm src/infer.cpp:367-382
    for (int lp = t; lp < n_rows / 2; lp += NT) {
      float g = 0.f, u = 0.f;
#pragma unroll
      for (int w = 0; w < NW; ++w) {
        g += red[(2 * lp) * NW + w];
        u += red[(2 * lp + 1) * NW + w];
      }
      float act;
      if (a.act_silu) {
        act = g / (1.0f + expf(-g));
      } else {
        act = 0.5f * g * (1.0f + tanhf(0.797885f * (g + 0.044715f * g * g * g)));
      }
      a.y[row_begin / 2 + lp] = act * u;
    }
  } else if (EPI == kEpiQKV) {
    StepState st;
    if (a.step) {
      st = *a.step;
    } else {
      st.pos = a.pos;
      st.kv_pos = a.kv_pos;
      st.kv_sink = a.kv_sink;
    }
    const int hd = a.head_dim;
    for (int lp = t; lp < n_rows / 2; lp += NT) {
      float s0 = 0.f, s1 = 0.f;
#pragma unroll
      for (int w = 0; w < NW; ++w) {
        s0 += red[(2 * lp) * NW + w];
        s1 += red[(2 * lp + 1) * NW + w];
      }
      // clip (src/infer.cpp:283-290)
      s0 = s0 < -a.qkv_clip ? -a.qkv_clip : (s0 > a.qkv_clip ? a.qkv_clip : s0);
      s1 = s1 < -a.qkv_clip ? -a.qkv_clip : (s1 > a.qkv_clip ? a.qkv_clip : s1);
      const int gr = row_begin + 2 * lp;
      if (gr < a.q_rows + a.kv_rows) {
        // interleaved-pair RoPE (src/infer.cpp:202-215): angle = pos * freq_j
        const int jh = (gr < a.q_rows ? gr : gr - a.q_rows) % hd;
        float fcr = 1.f, fci = 0.f;
        if (jh < a.rotary_dim) {
          const float val = (float)st.pos * a.inv_freq[jh >> 1];
          sincosf(val, &fci, &fcr);
        }
        const float r0 = s0 * fcr - s1 * fci;
        const float r1 = s0 * fci + s1 * fcr;
        if (gr < a.q_rows) {
          a.y[gr] = r0;
          a.y[gr + 1] = r1;
        } else {
          const int kr = gr - a.q_rows;
          const int g = kr / hd;
          __half* kh = a.k_cache + (size_t)g * a.max_seq_len * hd;
          *reinterpret_cast<__half2*>(kh + (size_t)st.kv_pos * hd + jh) = __floats2half2_rn(r0, r1);
          // attention sinks: re-rotate the kept keys by one position (src/infer.cpp:307-325)
          if (st.kv_sink > 0 && jh < a.rotary_dim) {
            float c1, s1v;
            sincosf(a.inv_freq[jh >> 1], &s1v, &c1);
            for (int r = 0; r < st.kv_sink; ++r) {
              __half2* p = reinterpret_cast<__half2*>(kh + (size_t)r * hd + jh);
              const float2 kv = __half22float2(*p);
              *p = __floats2half2_rn(kv.x * c1 - kv.y * s1v, kv.x * s1v + kv.y * c1);
            }
          }
        }
      } else {
        const int vr = gr - a.q_rows - a.kv_rows;
        const int g = vr / hd, jh = vr % hd;
        __half* vh = a.v_cache + (size_t)g * a.max_seq_len * hd;
        *reinterpret_cast<__half2*>(vh + (size_t)st.kv_pos * hd + jh) = __floats2half2_rn(s0, s1);
      }
    }
  }
  if (t == 0) timeline_stamp(a.trace, a.trace_stride, 4);
}

// ---------------------------------------------------------------------------------- host side
namespace {

template <int KPT, int RT, int EPI, int IN, int WT>
const void* pick4() {
  return reinterpret_cast<const void*>(&yb_stream_matvec<kGemvWarps, KPT, RT, EPI, IN, WT>);
}
// Instantiated combinations: residual epilogues never normalise their input; the tensor-parallel
// logits epilogue always does; pair epilogues (gate/up, QKV) need at least two rows per stage; the
// tensor-parallel input (in == 2) exists for the normalised dim-wide inputs (KPT <= 4, dim <= 8192)
// of the QKV, gate/up and logits matvecs.
template <int KPT, int RT, int WT>
const void* pick2(int epi, int in) {
  constexpr int RP = RT >= 2 ? RT : 2;
  constexpr bool TPK = KPT <= 4;
  switch (epi) {
    case kEpiStore:
      return in == 0 ? pick4<KPT, RT, kEpiStore, 0, WT>() : in == 1 ? pick4<KPT, RT, kEpiStore, 1, WT>() : nullptr;
    case kEpiResid: return in == 0 ? pick4<KPT, RT, kEpiResid, 0, WT>() : nullptr;
    case kEpiGateUp:
      if (RT < 2) return nullptr;
      if (in == 2) return TPK ? pick4<KPT, RP, kEpiGateUp, TPK ? 2 : 1, WT>() : nullptr;
      return in == 1 ? pick4<KPT, RP, kEpiGateUp, 1, WT>() : pick4<KPT, RP, kEpiGateUp, 0, WT>();
    case kEpiQKV:
      if (RT < 2) return nullptr;
      if (in == 2) return TPK ? pick4<KPT, RP, kEpiQKV, TPK ? 2 : 1, WT>() : nullptr;
      return in == 1 ? pick4<KPT, RP, kEpiQKV, 1, WT>() : pick4<KPT, RP, kEpiQKV, 0, WT>();
    case kEpiResidTP: return in == 0 ? pick4<KPT, RT, kEpiResidTP, 0, WT>() : nullptr;
    case kEpiStoreTP: return in == 2 && TPK ? pick4<KPT, RT, kEpiStoreTP, TPK ? 2 : 1, WT>() : nullptr;
  }
  return nullptr;
}
template <int KPT, int WT>
const void* pick1(int rt, int epi, int in) {
  switch (rt) {
    case 1: return pick2<KPT, 1, WT>(epi, in);
    case 2: return pick2<KPT, 2, WT>(epi, in);
    case 4: return pick2<KPT, 4, WT>(epi, in);
    case 8: return pick2<KPT, 8, WT>(epi, in);
  }
  return nullptr;
}
// fp8 rows hold twice the chunks' worth of weights: KPT 7 is not instantiated for them (it would
// mean more than 28672 columns).
const void* pick(int kpt, int rt, int epi, int in, int wt) {
  if (wt == 0) {
    switch (kpt) {
      case 1: return pick1<1, 0>(rt, epi, in);
      case 2: return pick1<2, 0>(rt, epi, in);
      case 4: return pick1<4, 0>(rt, epi, in);
      case 7: return pick1<7, 0>(rt, epi, in);
    }
  } else if (wt == 1) {
    switch (kpt) {
      case 1: return pick1<1, 1>(rt, epi, in);
      case 2: return pick1<2, 1>(rt, epi, in);
      case 4: return pick1<4, 1>(rt, epi, in);
    }
  } else if (rt == kMmaRows) {
    switch (kpt) {
      case 1: return pick2<1, kMmaRows, 2>(epi, in);
      case 2: return pick2<2, kMmaRows, 2>(epi, in);
      case 4: return pick2<4, kMmaRows, 2>(epi, in);
    }
  }
  return nullptr;
}

}  // namespace

LaunchTuning LaunchTuning::from_env() {
  static const LaunchTuning cached = [] {
    LaunchTuning t;
    const char* env = std::getenv("YB_TUNE");
    if (!env) return t;
    std::string s(env);
    size_t i = 0;
    while (i < s.size()) {
      size_t j = s.find(',', i);
      if (j == std::string::npos) j = s.size();
      std::string kv = s.substr(i, j - i);
      size_t eq = kv.find('=');
      if (eq != std::string::npos) {
        const std::string k = kv.substr(0, eq);
        const int v = std::atoi(kv.c_str() + eq + 1);
        if (k == "stage" && v >= 1024) t.stage_bytes_target = v;
        else if (k == "budget" && v >= 16384) t.smem_budget = v;
        else if (k == "slots" && v >= 2) t.max_slots = v;
        else if (k == "l2pf" && v >= 0) t.l2_prefetch_stages = v;
        else if (k == "l2wo" && v >= 0) t.l2_prefetch_wo = v;
        else if (k == "l2qkv" && v >= 0) t.l2_prefetch_qkv = v;
        else if (k == "ctas" && v >= 1 && v <= 8) t.ctas_per_sm = v;
        else if (k == "pstatic" && v >= 0 && v <= 100) t.persist_static_pct = v;
        else if (k == "pfq" && v >= 0) t.prefetch_qkv = v != 0;
        else if (k == "pfo" && v >= 0) t.prefetch_wo = v != 0;
        else if (k == "pctr" && v >= 1 && v <= 64) t.persist_claim_ctrs = v;
        else if (k == "aslots" && v >= 16 && v % 16 == 0) t.attn_cta_slots = v;
        else if (k == "acslots" && v >= 16 && v % 16 == 0) t.attn_cluster_slots = v;
        else if (k == "acl" && v >= 0 && v <= 16) t.attn_cluster = v;
        else if (k == "fp8mma" && v >= 0) t.fp8_mma = v != 0;
        else if (k == "pfplanes" && v >= 0 && v <= 15) t.prefill_planes = v;
        else if (k == "acs" && v >= 0 && v <= 32) t.attn_clusters_per_head = v;
      }
      i = j + 1;
    }
    return t;
  }();
  return cached;
}

int gemv_kpt_for(int cols, int esz) {
  const int chunks = cols / (esz == 1 ? 16 : 8);
  const int per = (chunks + kGemvWarps * 32 - 1) / (kGemvWarps * 32);
  if (per <= 1) return 1;
  if (per <= 2) return 2;
  if (per <= 4) return 4;
  if (per <= 7 && esz == 2) return 7;  // fp8 rows stop at KPT 4 (the caller splits wider matrices)
  return -1;
}

GemvPlan gemv_plan(int rows, int cols, int epi, bool norm, int n_sms, const LaunchTuning& tune, bool tp_in, int esz) {
  GemvPlan p{};
  p.ok = false;
  if (esz != 1 && esz != 2) return p;
  if (cols <= 0 || rows <= 0 || (cols % (esz == 1 ? 16 : 8)) != 0) return p;
  p.kpt = gemv_kpt_for(cols, esz);
  if (p.kpt < 0) return p;
  const int row_bytes = cols * esz;
  // fp8 weights on the CUDA cores (WT = 1), or with YB_TUNE=fp8mma=1 on the tensor cores (WT = 2, the
  // grouped layout the engine then writes at upload)
  const int wt = esz == 2 ? 0 : (tune.fp8_mma ? 2 : 1);
  int rt = 1;
  while (rt < 8 && (rt * 2) * row_bytes <= tune.stage_bytes_target) rt *= 2;
  const bool pairs = (epi == kEpiGateUp || epi == kEpiQKV);
  if (pairs && rt < 2) rt = 2;
  if (pairs && (rows % 2) != 0) return p;
  if (wt == 2) rt = kMmaRows;
  p.rt = rt;
  p.wt = wt;
  const int T = (rows + rt - 1) / rt;
  const int max_grid = n_sms * tune.ctas_per_sm;
  p.grid = T < max_grid ? T : max_grid;
  const int units_per_cta = (T + p.grid - 1) / p.grid;
  // tensor-core fp8: a stage is a group's chunk of up to kMmaCols columns; x waits in shared memory
  // as two fp16 planes
  const int chunk = cols < kMmaCols ? cols : kMmaCols;
  const int nc = wt == 2 ? (cols + kMmaCols - 1) / kMmaCols : 1;
  const int stages_per_cta = units_per_cta * nc;
  const int xs_bytes = wt == 2 ? 4 * cols + 16 : 0;
  p.red_floats = units_per_cta * rt * kGemvWarps;
  p.stage_bytes = wt == 2 ? (unsigned)((rt * chunk + 127) / 128 * 128) : (unsigned)((rt * row_bytes + 127) / 128 * 128);
  const int fixed = p.red_floats * 4 + 32 * 4 + 16 * 2 * 8 + 64 + xs_bytes;
  int ns = (tune.smem_budget - fixed) / (int)p.stage_bytes;
  if (ns > tune.max_slots) ns = tune.max_slots;
  if (ns > 16) ns = 16;
  if (ns > stages_per_cta) ns = stages_per_cta < 2 ? 2 : stages_per_cta;
  if (ns < 2) ns = 2;
  p.n_slots = ns;
  p.smem = (size_t)ns * p.stage_bytes + (size_t)p.red_floats * 4 + 32 * 4 + (size_t)ns * 2 * 8 + (size_t)xs_bytes;
  if (tp_in && !norm) return p;
  p.fn = pick(p.kpt, p.rt, epi, tp_in ? 2 : norm ? 1 : 0, wt);
  p.norm = norm;
  p.ok = p.fn != nullptr && p.smem <= 226 * 1024;
  return p;
}

cudaError_t gemv_prepare(const GemvPlan& p) { return raise_smem_cap(p.fn); }

// Grouped fp8 layout (WT = 2): dst 16-byte unit u = ((group * chunks + chunk) * 16 + row) holds
// columns [16 chunk, 16 chunk + 16) of row 16 group + row of src (zeros past the last row).
__global__ void fp8_group_layout_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst, long long rows,
                                        int cols) {
  const long long chunks = cols / 16;
  const long long units = (rows + kMmaRows - 1) / kMmaRows * kMmaRows * chunks;
  for (long long u = (long long)blockIdx.x * blockDim.x + threadIdx.x; u < units; u += (long long)gridDim.x * blockDim.x) {
    const long long r = u % kMmaRows, rest = u / kMmaRows;
    const long long chunk = rest % chunks, group = rest / chunks;
    const long long row = group * kMmaRows + r;
    dst[u] = row < rows ? src[row * chunks + chunk] : make_uint4(0u, 0u, 0u, 0u);
  }
}

size_t fp8_group_bytes(long long rows, int cols) {
  return (size_t)((rows + kMmaRows - 1) / kMmaRows) * kMmaRows * (size_t)cols;
}

cudaError_t fp8_group_layout(const void* src, void* dst, long long rows, int cols, cudaStream_t stream) {
  if (cols <= 0 || cols % 16 || rows <= 0 || (reinterpret_cast<uintptr_t>(src) & 15) ||
      (reinterpret_cast<uintptr_t>(dst) & 15))
    return cudaErrorInvalidValue;
  fp8_group_layout_kernel<<<1184, 256, 0, stream>>>(static_cast<const uint4*>(src), static_cast<uint4*>(dst), rows,
                                                     cols);
  return cudaGetLastError();
}

cudaError_t gemv_launch(const GemvPlan& p, GemvArgs a, cudaStream_t stream, bool pdl, int l2_prefetch_stages) {
  a.stage_bytes = p.stage_bytes;
  a.n_slots = p.n_slots;
  a.red_floats = p.red_floats;
  a.l2_prefetch_stages = l2_prefetch_stages;
  return launch_kernel(p.fn, dim3(p.grid), dim3((kGemvWarps + 1) * 32), p.smem, stream, pdl, &a);
}

}  // namespace yb
