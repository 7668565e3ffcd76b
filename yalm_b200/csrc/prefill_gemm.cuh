// Tensor-core GEMM for batched prefill (see prefill_gemm.cu).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_fp16.h>

#include <cstddef>
#include <cstdint>

namespace yb {

// C[m][n] (+)= sum_k A[m][k] * B[n][k]: A fp16 [M][K] row-major (tokens x features), B fp16 [N][K]
// row-major (the weight matrix as stored), fp32 accumulation in tensor memory.
enum PrefillEpi : int {
  kPreStore = 0,   // out_f32[m][n] = c
  kPreAdd = 1,     // out_f32[m][n] += c          (residual add)
  kPreSwiGLU = 2,  // columns (2j, 2j+1) = (gate, up): out_f16[m][j] = silu(gate) * up
  kPreStoreF16 = 3,  // out_f16[m][n] = c
};

constexpr int kPreBM = 128;      // tokens per tile (UMMA M)
constexpr int kPreBN = 256;      // output features per tile (UMMA N)
constexpr int kPreBK = 64;       // K per stage: one 128-byte swizzle row of fp16
constexpr int kPreStages = 4;
constexpr int kPreThreads = 192;  // warp 0 TMA, warp 1 MMA + TMEM owner, warps 2-5 epilogue

struct PrefillGemmArgs {
  int M, N, K;
  int epi;
  int ldo;          // row stride of the output in elements
  float* out_f32;
  __half* out_f16;
  unsigned* status;
  int a_planes;     // 1, or 2: A is [2][M][K], an fp16 value plane and its fp16 remainder plane,
                    // both multiplied by B into the same accumulator (about fp32 accuracy)
  int lo_out;       // fp16 epilogues: also write each value's fp16 remainder at out_f16 + M * ldo
};

// Host: builds the two tensor maps and launches (A: a_planes * M x K, box 128 x 64; B: N x K, box
// 256 x 64).  Returns a CUDA error code (cudaErrorInvalidValue for unsupported shapes: K % 64,
// N % 8).
cudaError_t prefill_gemm(const __half* A, const __half* B, const PrefillGemmArgs& args, cudaStream_t stream);

}  // namespace yb
