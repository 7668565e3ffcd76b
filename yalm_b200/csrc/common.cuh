// Device-side building blocks shared by the decode kernels (sm_100a).
//
//  * mbarrier + cp.async.bulk (1-D TMA) helpers for streaming weight rows global -> shared;
//  * programmatic dependent launch (griddepcontrol) so a kernel can start streaming its own
//    weights while the kernel before it is still finishing;
//  * bounded waits: every spin in this library gives up after a cycle budget, records an error
//    code in a status word the host reads after each step, and lets the kernel return.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace yb {

// Status bits written by kernels into the engine's status word (host-mapped memory).
enum : unsigned {
  kStatusOk = 0u,
  kStatusMbarTimeout = 1u << 0,   // a TMA stage never landed
  kStatusPeerTimeout = 1u << 1,   // a tensor-parallel peer never delivered its partial sums
  kStatusBadArgs = 1u << 2,       // device-side argument check failed (e.g. position out of range)
};

// ~2 s at the B200's 1.965 GHz boost clock; a healthy wait ends within microseconds.
constexpr long long kWaitBudgetCycles = 4000000000ll;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- programmatic dependent launch
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------- mbarrier
// The *_s forms take 32-bit shared-window addresses; the pointer forms convert with smem_u32, which
// must only see pointers derived from a __shared__ object by pointer arithmetic (a pointer rebuilt
// from an integer has no shared provenance, and its conversion is undefined).
__device__ __forceinline__ void mbar_init_s(uint32_t bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) { mbar_init_s(smem_u32(bar), count); }
// Makes barrier initialisation visible to the async (TMA) proxy before the first bulk copy.
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx_s(uint32_t bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, unsigned bytes) {
  mbar_arrive_expect_tx_s(smem_u32(bar), bytes);
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_s(uint32_t bar, unsigned parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, unsigned parity) {
  return mbar_try_wait_s(smem_u32(bar), parity);
}
// Waits for the barrier phase with the given parity.  Returns false (and records kStatusMbarTimeout)
// when the cycle budget runs out.
__device__ __forceinline__ bool mbar_wait_s(uint32_t bar, unsigned parity, unsigned* status) {
  if (mbar_try_wait_s(bar, parity)) return true;
  long long t0 = clock64();
  while (!mbar_try_wait_s(bar, parity)) {
    if (clock64() - t0 > kWaitBudgetCycles) {
      if (status) atomicOr(status, kStatusMbarTimeout);
      return false;
    }
  }
  return true;
}
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, unsigned parity, unsigned* status) {
  return mbar_wait_s(smem_u32(bar), parity, status);
}

// ---------------------------------------------------------------- bulk copies (1-D TMA)
// Evict-first L2 policy for data streamed exactly once per step (weights).
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
// global -> shared; dst, src 16-byte aligned, bytes a multiple of 16.  Completion is signalled on
// `bar` as transaction bytes.
__device__ __forceinline__ void bulk_g2s(void* dst_smem, const void* src, unsigned bytes, uint64_t* bar,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::
          "r"(smem_u32(dst_smem)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}
__device__ __forceinline__ void bulk_g2s_nohint_s(uint32_t dst, const void* src, unsigned bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}
__device__ __forceinline__ void bulk_g2s_nohint(void* dst_smem, const void* src, unsigned bytes, uint64_t* bar) {
  bulk_g2s_nohint_s(smem_u32(dst_smem), src, bytes, smem_u32(bar));
}
// Fire-and-forget prefetch of a global range into L2 (bytes a multiple of 16).
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, unsigned bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// 16-byte global -> shared copy through L2 only (cp.async, completion per thread via commit/wait
// groups); src_bytes 0 writes zeros (src must still be a valid address).
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, unsigned src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// 2-D tiled TMA load of one box of `map` at element coordinates (x inner, y outer) into shared
// memory, completing on `bar`.  x times the element size must be a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_2d_s(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(dst), "l"(map), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  tma_load_2d_s(smem_u32(dst), map, x, y, smem_u32(bar));
}

// ---------------------------------------------------------------- warp-level mma (m16n8k16, fp16)
// Fragment layouts as the PTX ISA defines them for mma.m16n8k16 with .f16 inputs: with
// g = lane / 4 and c = lane % 4, A (16 x 16, row) holds {(g, 2c..2c+1), (g+8, 2c..), (g, 2c+8..),
// (g+8, 2c+8..)}, B (16 x 8, col) holds {(k 2c..2c+1, n g), (k 2c+8.., n g)}, C/D (16 x 8, f32)
// holds {(g, 2c), (g, 2c+1), (g+8, 2c), (g+8, 2c+1)}.
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t saddr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(saddr)
               : "memory");
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t (&r)[4], uint32_t saddr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(saddr)
               : "memory");
}
// Transposes the 8 x 8 fp16 matrix whose rows the warp holds in the (g, 2c..2c+1) layout.
__device__ __forceinline__ uint32_t movm_trans(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// fp32 pair split into an fp16 pair and its fp16 remainder: x = hi + lo to about 22 bits, so a
// product with an fp16 operand keeps nearly fp32 accuracy over two mma passes.
__device__ __forceinline__ void split_f16x2(float x, float y, uint32_t& hi, uint32_t& lo) {
  const __half2 h = __floats2half2_rn(x, y);
  const __half2 l = __floats2half2_rn(x - __low2float(h), y - __high2float(h));
  hi = *reinterpret_cast<const uint32_t*>(&h);
  lo = *reinterpret_cast<const uint32_t*>(&l);
}

// ---------------------------------------------------------------- system-scope flags (peer memory)
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Adds v to *p (possibly another GPU's memory) with release semantics at system scope.  Issued by
// one thread after a CTA barrier, it publishes every write the CTA made before the barrier (the
// release is cumulative over writes ordered before it by the barrier), so only that thread pays
// for the system-scope fence.
// Counter add with acquire-release semantics at GPU scope; returns the previous value.  After a
// __syncthreads, one thread's release publishes the whole CTA's earlier writes (release is
// cumulative over what the barrier ordered before it); the acquire orders the caller's later reads.
__device__ __forceinline__ unsigned atom_add_acq_rel_gpu(unsigned* p, unsigned v) {
  unsigned old;
  asm volatile("atom.add.acq_rel.gpu.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
__device__ __forceinline__ void red_release_sys_add(unsigned* p, unsigned v) {
  asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// Stores one 8-byte exchange word {lo: fp32 bits, hi: epoch} (possibly into another GPU's memory);
// the word is written as a unit, so a reader that sees the epoch also sees the value.
__device__ __forceinline__ void st_ll(unsigned long long* p, float v, unsigned epoch) {
  const unsigned long long w = ((unsigned long long)epoch << 32) | __float_as_uint(v);
  asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
// Loads the 8 exchange words at p (16-byte aligned, 4 independent 16-byte loads).
__device__ __forceinline__ void ll_load8(const unsigned long long* p, unsigned long long* w) {
#pragma unroll
  for (int i = 0; i < 4; ++i)
    asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(w[2 * i]), "=l"(w[2 * i + 1]) : "l"(p + 2 * i) : "memory");
}
__device__ __forceinline__ bool ll_ready8(const unsigned long long* w, unsigned epoch) {
  bool all = true;
#pragma unroll
  for (int i = 0; i < 8; ++i) all = all && (unsigned)(w[i] >> 32) == epoch;
  return all;
}
// Waits until *p >= target (wrap-safe); false + kStatusPeerTimeout when the budget runs out.
__device__ __forceinline__ bool wait_counter_geq(const unsigned* p, unsigned target, unsigned* status) {
  if ((int)(ld_acquire_sys(p) - target) >= 0) return true;
  long long t0 = clock64();
  while ((int)(ld_acquire_sys(p) - target) < 0) {
    if (clock64() - t0 > kWaitBudgetCycles) {
      if (status) atomicOr(status, kStatusPeerTimeout);
      return false;
    }
    __nanosleep(64);
  }
  return true;
}

// Orders this thread's generic-proxy shared-memory writes before later async-proxy (TMA) writes
// to the same bytes (a ring slot refilled after consumers wrote into it).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------- named barrier among consumer warps
// %globaltimer in ns (timeline diagnostics).
__device__ __forceinline__ unsigned long long timeline_ns() {
  unsigned long long v;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(v));
  return v;
}
// Per-CTA timeline stamp j of one kernel launch: trace[blockIdx.x * stride + j] (trace null = off).
__device__ __forceinline__ void timeline_stamp(unsigned long long* trace, int stride, int j) {
  if (trace) trace[(size_t)blockIdx.x * stride + j] = timeline_ns();
}

__device__ __forceinline__ void named_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ---------------------------------------------------------------- numerics
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Reduce-scatter of N per-lane values across a warp (N a power of two, N <= 32): afterwards lane l
// holds in v[0] the warp-wide sum of value index (l >> (5 - log2 N)).  Uses N - 1 + (5 - log2 N)
// shuffles instead of the 5 N of N independent reductions.
template <int N>
__device__ __forceinline__ float warp_reduce_scatter(float (&v)[N], int lane) {
  static_assert(N >= 1 && N <= 32 && (N & (N - 1)) == 0, "N must be a power of two <= 32");
  int cnt = N;
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    if (cnt > 1) {
      const int half = cnt / 2;
      const bool upper = (lane & o) != 0;
#pragma unroll
      for (int i = 0; i < N / 2; ++i) {
        if (i < half) {
          float send = upper ? v[i] : v[i + half];
          float keep = upper ? v[i + half] : v[i];
          v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
        }
      }
      cnt = half;
    } else {
      v[0] += __shfl_xor_sync(0xffffffffu, v[0], o);
    }
  }
  return v[0];
}

// Packed fp32 pair arithmetic (sm_100): two IEEE fp32 operations per instruction, each rounded
// exactly as the scalar fmaf / multiply would be.
__device__ __forceinline__ unsigned long long f2_bits(float2 v) {
  unsigned long long u;
  asm("mov.b64 %0, {%1, %2};" : "=l"(u) : "f"(v.x), "f"(v.y));
  return u;
}
__device__ __forceinline__ float2 bits_f2(unsigned long long u) {
  float2 v;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(v.x), "=f"(v.y) : "l"(u));
  return v;
}
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
  unsigned long long d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(f2_bits(a)), "l"(f2_bits(b)), "l"(f2_bits(c)));
  return bits_f2(d);
}
__device__ __forceinline__ float2 mul2(float2 a, float2 b) {
  unsigned long long d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(f2_bits(a)), "l"(f2_bits(b)));
  return bits_f2(d);
}

// 16 fp8 E5M2 weights (one 16-byte vector) dotted with 16 fp32 activations.  An E5M2 value is
// the top byte of the fp16 with the same value, so a byte permute that puts each byte above a zero
// byte yields two fp16 values per 32-bit word, exactly; even and odd elements accumulate in the two
// halves of a packed fp32 pair (two FMA chains, as in dot8).
__device__ __forceinline__ float dot16_e5m2(uint4 w, const float4& x0, const float4& x1, const float4& x2,
                                            const float4& x3) {
  const unsigned q[4] = {w.x, w.y, w.z, w.w};
  const float4* xs[4] = {&x0, &x1, &x2, &x3};
  float2 acc = make_float2(0.f, 0.f);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const unsigned lo = __byte_perm(q[i], 0u, 0x1404u);  // elements 4i, 4i+1 as fp16
    const unsigned hi = __byte_perm(q[i], 0u, 0x3424u);  // elements 4i+2, 4i+3
    const float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(&lo));
    const float2 f1 = __half22float2(*reinterpret_cast<const __half2*>(&hi));
    acc = fma2(f0, make_float2(xs[i]->x, xs[i]->y), acc);
    acc = fma2(f1, make_float2(xs[i]->z, xs[i]->w), acc);
  }
  return acc.x + acc.y;
}

// 8 fp16 weights (one 16-byte vector) dotted with 8 fp32 activations: even and odd elements in the
// two halves of a packed fp32 pair (two independent 4-long FMA chains, half the FMA instructions).
__device__ __forceinline__ float dot8(uint4 w, const float4& xa, const float4& xb) {
  const __half2* h = reinterpret_cast<const __half2*>(&w);
  float2 acc = mul2(__half22float2(h[0]), make_float2(xa.x, xa.y));
  acc = fma2(__half22float2(h[1]), make_float2(xa.z, xa.w), acc);
  acc = fma2(__half22float2(h[2]), make_float2(xb.x, xb.y), acc);
  acc = fma2(__half22float2(h[3]), make_float2(xb.z, xb.w), acc);
  return acc.x + acc.y;
}

__device__ __forceinline__ uint4 lds128(const void* p) {
  uint4 r;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "r"(smem_u32(p)));
  return r;
}

// ---------------------------------------------------------------- per-step state shared by kernels
// Written once per step by the step kernel; every later kernel of the step reads it after its
// griddepcontrol.wait.  Positions follow yalm's ring-buffer/sink rule (src/infer.cpp:489-494).
struct StepState {
  int token;
  int pos;
  int kv_sink;
  int kv_pos;
  int kv_len;
  unsigned epoch;   // forward-call counter, identical on every tensor-parallel rank
  unsigned lepoch;  // counter of forward calls that produced logits
  int pad;
  // on-device sampler (yb_forward_sample / yb_forward_prob): op 0 argmax, 1 temperature sample,
  // 2 probability of `target`
  int sample_op;
  int sample_target;
  float temperature;
  float coin;
};

}  // namespace yb
