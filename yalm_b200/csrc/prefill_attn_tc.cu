// Causal GQA attention of a batched prompt on the 5th-generation tensor cores (sm_100a), head_dim
// 128: yalm's per-token attention (src/infer.cpp:218-250) for T queries at once, flash-attention
// style, with the scores and the output accumulated in tensor memory.
//
// CTA = (block of QB = 128 / GQ queries, kv head g): its 128 rows are the (query, head) pairs
// qi * GQ + h of the block, so every K / V tile serves the GQ query heads of the kv head.  Key tiles
// of 64 slots, over the block's causal range [0, pos0 + last query + 1):
//
//   warp 0      TMA producer: K and V tiles (64 slots x 128 dims as two 64 x 64 boxes each, 128-byte
//               swizzle, no multicast) into a 3-stage ring
//   warp 1      owns the tensor memory (256 columns: two 64-column score buffers, a 128-column output)
//               and issues the MMAs from one lane: S[b] = Q . K^T (M 128, N 64, K-major operands) for
//               tile j + 1 while the softmax works on tile j, then O += P . V (M 128, N 128; V read
//               MN-major straight from its TMA boxes)
//   warps 4-7   softmax, one row per thread (warp % 4 selects the tensor-memory lane quadrant):
//               stage Q as fp16 value + remainder planes at the start; per tile read the score row,
//               causal mask, online softmax in base 2, write P as fp16 value + remainder planes to
//               one of two shared-memory buffers (tile j's while the MMAs still read tile j - 1's,
//               so the softmax of a tile overlaps the P . V of the one before); rescale the output
//               row in tensor memory only when the row's maximum grew by more than 2^8 since the
//               last rescale (a stale maximum keeps every p <= 256, exact in fp16 value +
//               remainder, and the final O / l is the same); at the end read O, divide by l, store
//               fp16 value + remainder
//
// q and p enter the MMAs as two fp16 planes each (value, remainder), so products keep ~22 bits, as
// the fp32 loops of yalm do; each S or O step is two MMAs accumulating into the same columns.  Every
// wait is bounded: a wait that runs out sets the status word and the CTA stops.
#include "prefill.cuh"

#include "common.cuh"
#include "tmap.h"
#include "umma.cuh"

#include <math.h>

namespace yb {

namespace {

constexpr int kTcRows = 128;      // (query, head) rows per CTA = tensor-memory lanes
constexpr int kTcKeys = 64;       // keys per tile
constexpr int kTcHD = 128;        // head_dim
constexpr int kTcStages = 3;
constexpr int kTcThreads = 256;
constexpr int kTcTmemCols = 256;  // S0 [0, 64), S1 [64, 128), O [128, 256)
constexpr uint32_t kQPlane = kTcRows * kTcHD * 2;      // 32 KB: two 16 KB blocks of 64 dims
constexpr uint32_t kPPlane = kTcRows * kTcKeys * 2;    // 16 KB
constexpr uint32_t kBox = kTcKeys * 128;               // 8 KB: 64 slots x 64 dims
constexpr uint32_t kStage = 4 * kBox;                  // K box 0, K box 1, V box 0, V box 1
constexpr uint32_t kPBuf = 2 * kPPlane;  // one P buffer: value and remainder planes
constexpr uint32_t kOffQ = 0, kOffP = 2 * kQPlane, kOffRing = kOffP + 2 * kPBuf;
constexpr uint32_t kTcSmem = kOffRing + kTcStages * kStage;  // 224 KB
constexpr uint32_t kIdescS = umma_idesc_f16(kTcRows, kTcKeys, 0, 0);
constexpr uint32_t kIdescO = umma_idesc_f16(kTcRows, kTcHD, 0, 1);

// byte offset of 16-byte chunk c (of 8) in row r of a 128-byte-swizzled block (rows 128 bytes apart)
__device__ __forceinline__ uint32_t sw128(int r, int c) { return (uint32_t)r * 128u + ((uint32_t)(c ^ (r & 7)) << 4); }

// 2^x by the special-function unit (ex2.approx: relative error about 2^-22; -inf gives +0)
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void sts128(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

}  // namespace

struct PrefillAttnTcArgs {
  const float* q;  // [T][n_heads * 128] fp32 (after RoPE)
  __half* out;     // [T][n_heads * 128]
  __half* out_lo;  // optional remainder plane
  int T, pos0, n_heads, msl;
  int v_lbo, v_sbo;  // MN-major V descriptor: byte offsets between 64-dim atoms and 8-slot groups
  unsigned* status;
};

template <int GQ>
__global__ void __launch_bounds__(kTcThreads, 1)
    prefill_attn_tc_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                           const PrefillAttnTcArgs a) {
  constexpr int QB = kTcRows / GQ;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const uint32_t sb = smem_u32(smem);
  __shared__ __align__(8) uint64_t full[kTcStages], empty[kTcStages], s_full[2], s_free[2], p_full[2], o_done[2],
      q_ready;
  __shared__ uint32_t s_tmem;
  __shared__ int s_abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nqb = (a.T + QB - 1) / QB;
  const int qb = nqb - 1 - (int)blockIdx.x;  // longest blocks first
  const int g = blockIdx.y;
  const int q0 = qb * QB;
  const int kend = a.pos0 + min(q0 + QB, a.T);  // keys [0, kend)
  const int ntile = (kend + kTcKeys - 1) / kTcKeys;
  const int q_dim = a.n_heads * kTcHD;

  if (threadIdx.x == 0) {
    s_abort = 0;
    for (int s = 0; s < kTcStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&s_free[b], 4);
      mbar_init(&p_full[b], 4);
      mbar_init(&o_done[b], 1);
    }
    mbar_init(&q_ready, 4);
    mbar_fence_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 ::"r"(smem_u32(&s_tmem)), "r"(kTcTmemCols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;
  volatile int* abort_flag = &s_abort;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ TMA producer
      const int y0 = g * a.msl;
      int j = 0;
      for (; j < ntile && !*abort_flag; ++j) {
        const int s = j % kTcStages;
        if (j >= kTcStages && !mbar_wait(&empty[s], ((j / kTcStages) - 1) & 1, a.status)) {
          *abort_flag = 1;
          break;
        }
        unsigned char* st = smem + kOffRing + (size_t)s * kStage;
        mbar_arrive_expect_tx(&full[s], kStage);
        const int y = y0 + j * kTcKeys;
        tma_load_2d(st, &kmap, 0, y, &full[s]);
        tma_load_2d(st + kBox, &kmap, 64, y, &full[s]);
        tma_load_2d(st + 2 * kBox, &vmap, 0, y, &full[s]);
        tma_load_2d(st + 3 * kBox, &vmap, 64, y, &full[s]);
      }
      // never leave while a tile load issued here may still be landing
      for (int i = max(0, j - kTcStages); i < j; ++i) mbar_wait(&full[i % kTcStages], (i / kTcStages) & 1, a.status);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (waits on all lanes)
    bool ok = mbar_wait(&q_ready, 0, a.status);
    tc_fence_after();
    const uint32_t qa = sb + kOffQ, pa = sb + kOffP;
    auto issue_s = [&](int j) -> bool {
      const int s = j % kTcStages, b = j & 1;
      if (!mbar_wait(&full[s], (j / kTcStages) & 1, a.status)) return false;
      if (j >= 2 && !mbar_wait(&s_free[b], ((j >> 1) - 1) & 1, a.status)) return false;
      const uint32_t st = sb + kOffRing + (uint32_t)s * kStage;
      const int rem = kend - j * kTcKeys;
      if (rem < kTcKeys) {
        // V rows past the causal range (another slot's or head's data, possibly not finite) are
        // zeroed: their p is 0, and 0 * v must stay 0
        for (int e = lane; e < (kTcKeys - rem) * 16; e += 32) {
          const int r = rem + e / 16, c = e % 16;
          sts128(st + 2 * kBox + (uint32_t)(c / 8) * kBox + (uint32_t)r * 128u + (uint32_t)(c % 8) * 16u, 0u, 0u, 0u, 0u);
        }
        fence_proxy_async_smem();
        __syncwarp();
      }
      tc_fence_after();
      if (lane == 0) {
#pragma unroll
        for (int plane = 0; plane < 2; ++plane)
#pragma unroll
          for (int kk = 0; kk < kTcHD / 16; ++kk) {
            const uint64_t da = umma_desc_k_sw128(qa + (uint32_t)plane * kQPlane + (uint32_t)(kk / 4) * (kQPlane / 2) +
                                                  (uint32_t)(kk % 4) * 32u);
            const uint64_t db = umma_desc_k_sw128(st + (uint32_t)(kk / 4) * kBox + (uint32_t)(kk % 4) * 32u);
            umma_f16(tmem + (uint32_t)(b * kTcKeys), da, db, kIdescS, (plane | kk) ? 1u : 0u);
          }
        umma_commit(&s_full[b]);
      }
      __syncwarp();
      return true;
    };
    if (ok) ok = issue_s(0);
    for (int j = 0; j < ntile && ok && !*abort_flag; ++j) {
      if (j + 1 < ntile && !(ok = issue_s(j + 1))) break;
      const int pb = j & 1;
      if (!(ok = mbar_wait(&p_full[pb], (j >> 1) & 1, a.status))) break;
      tc_fence_after();
      const int s = j % kTcStages;
      const uint32_t vb = sb + kOffRing + (uint32_t)s * kStage + 2 * kBox;
      if (lane == 0) {
#pragma unroll
        for (int plane = 0; plane < 2; ++plane)
#pragma unroll
          for (int kk = 0; kk < kTcKeys / 16; ++kk) {
            const uint64_t da = umma_desc_k_sw128(pa + (uint32_t)pb * kPBuf + (uint32_t)plane * kPPlane + (uint32_t)kk * 32u);
            const uint64_t db = umma_desc_sw128(vb + (uint32_t)kk * 2048u, (uint32_t)a.v_lbo, (uint32_t)a.v_sbo);
            umma_f16(tmem + 128u, da, db, kIdescO, (j | plane | kk) ? 1u : 0u);
          }
        umma_commit(&o_done[pb]);
        umma_commit(&empty[s]);
      }
      __syncwarp();
    }
    if (!ok) *abort_flag = 1;
  } else if (warp >= 4) {
    // ------------------------------------------------------------ softmax, one row per thread
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const int qi = r / GQ, h = r % GQ;
    const int tq = q0 + qi;
    const bool valid = tq < a.T;
    const int qpos = a.pos0 + tq;
    const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
    // Q row -> fp16 value and remainder planes, K-major 128-byte swizzle (two blocks of 64 dims)
    {
      const float* qrow = a.q + (size_t)(valid ? tq : 0) * q_dim + (size_t)(g * GQ + h) * kTcHD;
#pragma unroll 4
      for (int c = 0; c < kTcHD / 8; ++c) {
        float4 x0 = make_float4(0.f, 0.f, 0.f, 0.f), x1 = x0;
        if (valid) {
          x0 = __ldg(reinterpret_cast<const float4*>(qrow + 8 * c));
          x1 = __ldg(reinterpret_cast<const float4*>(qrow + 8 * c + 4));
        }
        uint32_t hi[4], lo[4];
        split_f16x2(x0.x, x0.y, hi[0], lo[0]);
        split_f16x2(x0.z, x0.w, hi[1], lo[1]);
        split_f16x2(x1.x, x1.y, hi[2], lo[2]);
        split_f16x2(x1.z, x1.w, hi[3], lo[3]);
        const uint32_t off = (uint32_t)(c / 8) * (kQPlane / 2) + sw128(r, c % 8);
        sts128(sb + kOffQ + off, hi[0], hi[1], hi[2], hi[3]);
        sts128(sb + kOffQ + kQPlane + off, lo[0], lo[1], lo[2], lo[3]);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&q_ready);
    }
    // scores in base 2: t = q.k * log2(e) / sqrt(head_dim), p = 2^(t - m)
    const float sl2 = 1.4426950408889634f / sqrtf((float)kTcHD);
    float m_run = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < ntile; ++j) {
      const int b = j & 1;
      if (*abort_flag || !(ok = mbar_wait(&s_full[b], (j >> 1) & 1, a.status))) break;
      tc_fence_after();
      float s[64];
      tmem_ld64(lane_base + (uint32_t)(b * kTcKeys), s);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_free[b]);
      float mx = -INFINITY;
      const int k0 = j * kTcKeys;
      if (valid && k0 + kTcKeys - 1 <= qpos) {  // a tile wholly inside the row's causal range
#pragma unroll
        for (int k = 0; k < 64; ++k) {
          s[k] *= sl2;
          mx = fmaxf(mx, s[k]);
        }
      } else {
#pragma unroll
        for (int k = 0; k < 64; ++k) {
          const float t = (valid && k0 + k <= qpos) ? s[k] * sl2 : -INFINITY;
          s[k] = t;
          mx = fmaxf(mx, t);
        }
      }
      const bool need = mx > m_run + 8.0f;  // also the first tile with any key (m_run = -inf)
      const float m_new = need ? mx : m_run;
      const float alpha = need ? exp2f(m_run - m_new) : 1.f;  // 0 while m_run is -inf
      float ps = 0.f;
      if (m_new != -INFINITY) {
#pragma unroll
        for (int k = 0; k < 64; ++k) {
          const float p = ex2_approx(s[k] - m_new);  // 2^-inf = +0 for masked keys
          s[k] = p;
          ps += p;
        }
      } else {
#pragma unroll
        for (int k = 0; k < 64; ++k) s[k] = 0.f;
      }
      l = l * alpha + ps;
      m_run = m_new;
      const int pb = j & 1;
      // P buffer pb was last read by the P . V of tile j - 2
      if (j >= 2 && !(ok = mbar_wait(&o_done[pb], ((j - 2) >> 1) & 1, a.status))) break;
      if (j > 0 && __any_sync(0xffffffffu, need)) {
        // the output rows take the new maxima before tile j's P . V: O(j - 1) must be complete
        if (!(ok = mbar_wait(&o_done[(j - 1) & 1], ((j - 1) >> 1) & 1, a.status))) break;
        tc_fence_after();
#pragma unroll 1
        for (int c0 = 0; c0 < kTcHD; c0 += 32) {
          float v[32];
          tmem_ld32(lane_base + 128u + (uint32_t)c0, v);
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] *= alpha;
          tmem_st32(lane_base + 128u + (uint32_t)c0, v);
        }
      }
      const uint32_t pbase = sb + kOffP + (uint32_t)pb * kPBuf;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint32_t hi[4], lo[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) split_f16x2(s[8 * c + 2 * i], s[8 * c + 2 * i + 1], hi[i], lo[i]);
        const uint32_t off = sw128(r, c);
        sts128(pbase + off, hi[0], hi[1], hi[2], hi[3]);
        sts128(pbase + kPPlane + off, lo[0], lo[1], lo[2], lo[3]);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[pb]);
    }
    if (ok && !*abort_flag && mbar_wait(&o_done[(ntile - 1) & 1], ((ntile - 1) >> 1) & 1, a.status)) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __half* o = a.out + (size_t)(valid ? tq : 0) * q_dim + (size_t)(g * GQ + h) * kTcHD;
      __half* ol = a.out_lo ? a.out_lo + (o - a.out) : nullptr;
#pragma unroll 1
      for (int c0 = 0; c0 < kTcHD; c0 += 32) {
        float v[32];
        tmem_ld32(lane_base + 128u + (uint32_t)c0, v);
        if (!valid) continue;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t hi[4], lo[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) split_f16x2(v[8 * c + 2 * i] * inv, v[8 * c + 2 * i + 1] * inv, hi[i], lo[i]);
          reinterpret_cast<uint4*>(o + c0)[c] = make_uint4(hi[0], hi[1], hi[2], hi[3]);
          if (ol) reinterpret_cast<uint4*>(ol + c0)[c] = make_uint4(lo[0], lo[1], lo[2], lo[3]);
        }
      }
    } else {
      *abort_flag = 1;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTcTmemCols) : "memory");
  }
}

namespace {
const void* pick_tc(int gq) {
  switch (gq) {
    case 1: return reinterpret_cast<const void*>(&prefill_attn_tc_kernel<1>);
    case 2: return reinterpret_cast<const void*>(&prefill_attn_tc_kernel<2>);
    case 4: return reinterpret_cast<const void*>(&prefill_attn_tc_kernel<4>);
    case 8: return reinterpret_cast<const void*>(&prefill_attn_tc_kernel<8>);
  }
  return nullptr;
}
}  // namespace

bool prefill_attention_tc_supported(int head_dim, int gq) { return head_dim == kTcHD && pick_tc(gq) != nullptr; }

cudaError_t prefill_attention_tc(const float* q, const __half* k_cache, const __half* v_cache, __half* out,
                                 __half* out_lo, int T, int pos0, int n_heads, int n_kv_heads, int max_seq_len,
                                 unsigned* status, int v_desc_order, cudaStream_t s) {
  if (T <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads || pos0 + T > max_seq_len) return cudaErrorInvalidValue;
  const int gq = n_heads / n_kv_heads;
  const void* fn = pick_tc(gq);
  if (!fn || (reinterpret_cast<uintptr_t>(q) & 15) || (reinterpret_cast<uintptr_t>(out) & 15) ||
      (out_lo && (reinterpret_cast<uintptr_t>(out_lo) & 15)))
    return cudaErrorInvalidValue;
  CUtensorMap km, vm;
  const long long rows = (long long)n_kv_heads * max_seq_len;
  if (!tmap_f16_2d_sw128(&km, k_cache, rows, kTcHD, 64, kTcKeys) ||
      !tmap_f16_2d_sw128(&vm, v_cache, rows, kTcHD, 64, kTcKeys))
    return cudaErrorInvalidValue;
  const size_t smem = kTcSmem + 1024;
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  PrefillAttnTcArgs a;
  a.q = q;
  a.out = out;
  a.out_lo = out_lo;
  a.T = T;
  a.pos0 = pos0;
  a.n_heads = n_heads;
  a.msl = max_seq_len;
  // MN-major V operand: its 64-dim atoms are the two TMA boxes (kBox apart), its 8-slot groups
  // 1024 bytes apart; v_desc_order 1 swaps the two fields (layout check)
  a.v_lbo = v_desc_order == 1 ? 1024 : (int)kBox;
  a.v_sbo = v_desc_order == 1 ? (int)kBox : 1024;
  a.status = status;
  const int qb = kTcRows / gq;
  const dim3 grid((T + qb - 1) / qb, n_kv_heads);
  void* args[] = {&km, &vm, &a};
  return cudaLaunchKernel(fn, grid, dim3(kTcThreads), args, smem, s);
}

}  // namespace yb
