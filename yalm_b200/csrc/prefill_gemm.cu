// Tensor-core GEMM for batched prefill on sm_100a: TMA (128-byte swizzle) into a shared-memory
// ring, tcgen05.mma (kind::f16, M 128, N 256, K 16) accumulating in tensor memory, tcgen05.ld for
// the fused epilogue.  Persistent: one CTA per SM walks the output tiles (128 tokens x 256
// features) blockIdx.x, blockIdx.x + gridDim.x, ..., token blocks fastest so CTAs working at the
// same time share the weight tile through L2.  Two accumulators in tensor memory (512 columns) let
// the epilogue of one tile run while the MMAs of the next accumulate.
//
//   warp 0      TMA producer: one elected lane fills the ring with the A and B tiles of every
//               k-block of every tile of the CTA, stage after stage
//   warp 1      owns the tensor-memory allocation; one elected lane issues the MMAs of each stage
//               into accumulator (tile & 1), commits them to the stage's `empty` barrier, and after a
//               tile's last k-block to `acc_full[tile & 1]`; before reusing an accumulator it waits
//               for `acc_empty` from the epilogue of the tile two back
//   warps 2-5   epilogue: each reads the 32 tensor-memory lanes (= tile rows) of its quadrant
//               (warp % 4), 32 columns at a time, writes the fused result, then frees the
//               accumulator
//
// Operand layouts follow the canonical K-major SWIZZLE_128B form of the UMMA shared-memory
// descriptor (rows of 128 bytes, 8-row groups 1024 bytes apart); the descriptor fields are laid
// out as the PTX ISA and CUTLASS (cute/arch/mma_sm100_desc.hpp) define them.  Every wait is
// bounded; a wait that runs out sets the status word and the CTA stops issuing work.
#include "prefill_gemm.cuh"

#include "common.cuh"
#include "tmap.h"
#include "umma.cuh"

namespace yb {

namespace {

constexpr int kTileABytes = kPreBM * kPreBK * 2;  // 16 KB
constexpr int kTileBBytes = kPreBN * kPreBK * 2;  // 32 KB
constexpr int kStageBytes = kTileABytes + kTileBBytes;
constexpr int kTmemCols = 2 * kPreBN;             // two fp32 accumulators of 128 lanes x 256 columns

// Instruction descriptor: fp16 A and B, fp32 accumulator, both K-major, M 128, N 256.
constexpr uint32_t kIdesc = umma_idesc_f16(kPreBM, kPreBN, 0, 0);

}  // namespace

__device__ __forceinline__ uint32_t pack_h2(float x, float y) {
  const __half2 h = __floats2half2_rn(x, y);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// n fp32 values as fp16 at o (16-byte stores when whole and aligned); with lo set, each value's fp16
// remainder at the same index of lo.
template <int NV>
__device__ __forceinline__ void store_f16(__half* o, __half* lo, const float (&r)[NV], int valid) {
  if (valid == NV && (reinterpret_cast<uintptr_t>(o) & 15) == 0 && (!lo || (reinterpret_cast<uintptr_t>(lo) & 15) == 0)) {
#pragma unroll
    for (int i = 0; i < NV / 8; ++i) {
      uint32_t h[4], l[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const __half2 hh = __floats2half2_rn(r[8 * i + 2 * k], r[8 * i + 2 * k + 1]);
        h[k] = *reinterpret_cast<const uint32_t*>(&hh);
        l[k] = pack_h2(r[8 * i + 2 * k] - __low2float(hh), r[8 * i + 2 * k + 1] - __high2float(hh));
      }
      reinterpret_cast<uint4*>(o)[i] = make_uint4(h[0], h[1], h[2], h[3]);
      if (lo) reinterpret_cast<uint4*>(lo)[i] = make_uint4(l[0], l[1], l[2], l[3]);
    }
  } else {
#pragma unroll
    for (int i = 0; i < NV; ++i)
      if (i < valid) {
        const __half h = __float2half_rn(r[i]);
        o[i] = h;
        if (lo) lo[i] = __float2half_rn(r[i] - __half2float(h));
      }
  }
}

// Writes 32 accumulator columns (tile columns col .. col + 31) of one row with the fused epilogue.
__device__ __forceinline__ void epilogue_chunk(const PrefillGemmArgs& a, int row, int col, const float (&v)[32]) {
  const size_t lo_off = (size_t)a.M * a.ldo;
  if (a.epi == kPreSwiGLU) {
    // (gate, up) column pairs -> silu(gate) * up at column col / 2 + i
    __half* o = a.out_f16 + (size_t)row * a.ldo + col / 2;
    float r[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float g = v[2 * i], u = v[2 * i + 1];
      r[i] = g / (1.0f + expf(-g)) * u;
    }
    store_f16<16>(o, a.lo_out ? o + lo_off : nullptr, r, min(16, (a.N - col) / 2));
  } else if (a.epi == kPreStoreF16) {
    __half* o = a.out_f16 + (size_t)row * a.ldo + col;
    store_f16<32>(o, a.lo_out ? o + lo_off : nullptr, v, min(32, a.N - col));
  } else {
    float* o = a.out_f32 + (size_t)row * a.ldo + col;
    if (col + 32 <= a.N && (reinterpret_cast<uintptr_t>(o) & 15) == 0) {
#pragma unroll
      for (int i = 0; i < 32; i += 4) {
        float4 r = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
        if (a.epi == kPreAdd) {
          const float4 q = *reinterpret_cast<const float4*>(o + i);
          r.x += q.x; r.y += q.y; r.z += q.z; r.w += q.w;
        }
        *reinterpret_cast<float4*>(o + i) = r;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (col + i < a.N) o[i] = a.epi == kPreAdd ? o[i] + v[i] : v[i];
    }
  }
}

__global__ void __launch_bounds__(kPreThreads, 1)
    prefill_gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                        const PrefillGemmArgs a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // stage buffers must start on a 1024-byte boundary (swizzle atom)
  // (aligned in the shared address space; the pointer steps by the same pad and keeps its provenance)
  unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  __shared__ __align__(8) uint64_t full[kPreStages], empty[kPreStages], acc_full[2], acc_empty[2];
  __shared__ uint32_t s_tmem;
  __shared__ int s_abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles_m = (a.M + kPreBM - 1) / kPreBM;
  const int n_tiles = tiles_m * ((a.N + kPreBN - 1) / kPreBN);
  const int nk = a.K / kPreBK;
  const int nkv = nk * (a.a_planes == 2 ? 2 : 1);  // k-blocks per tile over the A planes
  const int G = gridDim.x;

  if (threadIdx.x == 0) {
    s_abort = 0;
    for (int s = 0; s < kPreStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);  // one arrival per epilogue warp
    }
    mbar_fence_init();
  }
  if (warp == 1) {
    // whole warp: allocate the accumulator columns, publish the address
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 ::"r"(smem_u32(&s_tmem)), "r"(kTmemCols) : "memory");
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
      int it = 0;  // k-blocks issued over all tiles of this CTA
      for (int t = blockIdx.x; t < n_tiles && !*abort_flag; t += G) {
        const int m0 = (t % tiles_m) * kPreBM, n0 = (t / tiles_m) * kPreBN;
        for (int kv = 0; kv < nkv; ++kv, ++it) {
          // k-block kv % nk of A plane kv / nk (rows of plane p start at p * M) against the same
          // k-block of B
          const int kb = kv % nk, plane = kv / nk;
          const int s = it % kPreStages;
          if (it >= kPreStages && !mbar_wait(&empty[s], ((it / kPreStages) - 1) & 1, a.status)) {
            *abort_flag = 1;
            break;
          }
          unsigned char* sa = smem + (size_t)s * kStageBytes;
          mbar_arrive_expect_tx(&full[s], (unsigned)kStageBytes);
          tma_load_2d(sa, &map_a, kb * kPreBK, plane * a.M + m0, &full[s]);
          tma_load_2d(sa + kTileABytes, &map_b, kb * kPreBK, n0, &full[s]);
        }
      }
      // never leave while a tile load issued here may still be landing: the last armed phase of
      // each stage must have completed (already true unless a wait gave up)
      for (int i = max(0, it - kPreStages); i < it; ++i) mbar_wait(&full[i % kPreStages], (i / kPreStages) & 1, a.status);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------ MMA issuer
      int it = 0, j = 0;
      for (int t = blockIdx.x; t < n_tiles && !*abort_flag; t += G, ++j) {
        const int b = j & 1;
        // accumulator b was last used by tile j - 2: its epilogue must have read it out
        if (j >= 2 && !mbar_wait(&acc_empty[b], ((j >> 1) - 1) & 1, a.status)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t acc = tmem + (uint32_t)(b * kPreBN);
        bool ok = true;
        for (int kb = 0; kb < nkv; ++kb, ++it) {
          const int s = it % kPreStages;
          if (!mbar_wait(&full[s], (it / kPreStages) & 1, a.status)) {
            ok = false;
            *abort_flag = 1;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + (size_t)s * kStageBytes);
          const uint32_t sb = sa + kTileABytes;
#pragma unroll
          for (int k = 0; k < kPreBK / 16; ++k)  // 16 fp16 = 32 bytes further along the swizzled row
            umma_f16(acc, umma_desc_k_sw128(sa + k * 32), umma_desc_k_sw128(sb + k * 32), kIdesc, (kb | k) ? 1u : 0u);
          umma_commit(&empty[s]);  // the stage is free once these MMAs have read it
        }
        if (!ok) break;
        umma_commit(&acc_full[b]);
      }
    }
  } else {
    // -------------------------------------------------------------- epilogue (warps 2-5)
    const int quad = warp & 3;  // tensor-memory lanes [32 quad, 32 quad + 32) = tile rows
    int j = 0;
    for (int t = blockIdx.x; t < n_tiles; t += G, ++j) {
      const int b = j & 1;
      if (*abort_flag || !mbar_wait(&acc_full[b], (j >> 1) & 1, a.status)) break;
      tc_fence_after();
      const int m0 = (t % tiles_m) * kPreBM, n0 = (t / tiles_m) * kPreBN;
      const int row = m0 + quad * 32 + lane;
      for (int c0 = 0; c0 < kPreBN; c0 += 32) {
        float v[32];
        tmem_ld32(tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(b * kPreBN + c0), v);
        if (row < a.M && n0 + c0 < a.N) epilogue_chunk(a, row, n0 + c0, v);
      }
      // the accumulator is free for tile j + 2
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

// ---------------------------------------------------------------------------------- host side
namespace {

// Row-major fp16 matrix [rows][cols] read in boxes of box_rows x 64 columns, 128-byte swizzle;
// rows beyond the matrix read as zeros.
bool make_map(CUtensorMap* m, const __half* base, long long rows, int cols, int box_rows) {
  return tmap_f16_2d_sw128(m, base, rows, cols, kPreBK, box_rows);
}

}  // namespace

cudaError_t prefill_gemm(const __half* A, const __half* B, const PrefillGemmArgs& args, cudaStream_t stream) {
  if (args.M <= 0 || args.N <= 0 || args.K <= 0 || args.K % kPreBK || args.N % 8 ||
      (reinterpret_cast<uintptr_t>(A) & 15) || (reinterpret_cast<uintptr_t>(B) & 15))
    return cudaErrorInvalidValue;
  if ((args.epi == kPreSwiGLU || args.epi == kPreStoreF16) ? !args.out_f16 : !args.out_f32) return cudaErrorInvalidValue;
  if (args.a_planes != 1 && args.a_planes != 2) return cudaErrorInvalidValue;
  CUtensorMap ma, mb;
  if (!make_map(&ma, A, (long long)args.M * args.a_planes, args.K, kPreBM) || !make_map(&mb, B, args.N, args.K, kPreBN))
    return cudaErrorInvalidValue;
  const size_t smem = (size_t)kPreStages * kStageBytes + 1024;
  static bool attr_set[64] = {};  // per device
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(prefill_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  static int n_sms[64] = {};
  if (dev >= 0 && dev < 64 && !n_sms[dev]) cudaDeviceGetAttribute(&n_sms[dev], cudaDevAttrMultiProcessorCount, dev);
  const int sms = (dev >= 0 && dev < 64 && n_sms[dev] > 0) ? n_sms[dev] : 148;
  const long long tiles = (long long)((args.N + kPreBN - 1) / kPreBN) * ((args.M + kPreBM - 1) / kPreBM);
  const dim3 grid((unsigned)(tiles < sms ? tiles : sms));  // persistent: one CTA per SM
  prefill_gemm_kernel<<<grid, kPreThreads, smem, stream>>>(ma, mb, args);
  return cudaGetLastError();
}

}  // namespace yb
