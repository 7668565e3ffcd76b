// Batched prefill (see prefill.cu): the prompt's tokens through every layer at once, GEMMs on the
// tensor cores (prefill_gemm.cu), filling the KV cache for the decode steps that follow.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "common.cuh"

namespace yb {

// Row-wise RMSNorm of x fp32 [T][dim] into xn fp16 [T][dim] (yalm src/infer.cpp:136-146); with xn_lo
// non-null also each value's fp16 remainder there (xn + xn_lo = the fp32 result to ~2^-22).
cudaError_t prefill_rmsnorm(const float* x, const float* w, __half* xn, __half* xn_lo, int T, int dim, float eps,
                            cudaStream_t s);

// Per token t (position pos0 + t): clip, interleaved-pair RoPE on q and k, q -> q_out fp32
// [T][q_rows], k / v -> fp16 cache slot pos0 + t (src/infer.cpp:283-305).  qkv fp32 [T][q+2kv].
cudaError_t prefill_qkv_post(const float* qkv, int T, int pos0, int q_rows, int kv_rows, int head_dim,
                             int rotary_dim, int max_seq_len, float qkv_clip, const float* inv_freq, float* q_out,
                             __half* k_cache, __half* v_cache, cudaStream_t s);

// Causal GQA attention of T queries at positions pos0 .. pos0 + T - 1 over cache slots
// 0 .. pos0 + t (src/infer.cpp:218-250): out fp16 [T][n_heads * head_dim], and with out_lo non-null
// each value's fp16 remainder there.  head_dim 128 runs on tcgen05 (prefill_attn_tc.cu), head_dim
// 64 on mma.sync; YB_PREFILL_ATTN=mma selects the mma.sync kernel for both.  status (optional)
// records a bounded wait that ran out.
cudaError_t prefill_attention(const float* q, const __half* k_cache, const __half* v_cache, __half* out, __half* out_lo,
                              int T, int pos0, int n_heads, int n_kv_heads, int head_dim, int max_seq_len,
                              unsigned* status, cudaStream_t s);

// The tcgen05 kernel alone (head_dim 128, n_heads / n_kv_heads in 1, 2, 4, 8).  v_desc_order 0 is the
// V operand's descriptor as the kernel uses it; 1 swaps its two byte offsets (a layout check).
bool prefill_attention_tc_supported(int head_dim, int gq);
cudaError_t prefill_attention_tc(const float* q, const __half* k_cache, const __half* v_cache, __half* out,
                                 __half* out_lo, int T, int pos0, int n_heads, int n_kv_heads, int max_seq_len,
                                 unsigned* status, int v_desc_order, cudaStream_t s);

}  // namespace yb
