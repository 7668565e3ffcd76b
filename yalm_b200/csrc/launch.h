// Host-side launch helpers and kernel plans shared by the engine and the C-ABI test hooks.
#pragma once

#include <cuda_runtime.h>
#include <cstddef>

#include "common.cuh"

namespace yb {

struct GemvArgs;
struct AttnArgs;

// Tunables for the streaming kernels (host values; see the engine for defaults).
struct LaunchTuning {
  int stage_bytes_target = 16384;  // bytes of whole rows per TMA stage
  int smem_budget = 100000;        // per-CTA dynamic shared memory; two CTAs fit on one SM
  int max_slots = 8;               // ring depth cap
  int l2_prefetch_stages = 0;      // stages beyond the ring warmed into L2 before griddepcontrol.wait (measured: off is faster)
  int l2_prefetch_wo = -1;         // the same for the wo matvec alone (-1: l2_prefetch_stages)
  int l2_prefetch_qkv = -1;        // the same for the QKV matvec alone (-1: l2_prefetch_stages)
  int ctas_per_sm = 2;              // GEMV grid = min(stages, SMs * ctas_per_sm)
  bool prefetch_qkv = false;        // graph executor: W2 kernels warm L2 with the next layer's QKV rows
  bool prefetch_wo = false;         // graph executor: QKV kernels warm L2 with the layer's Wo
  int persist_static_pct = 100;     // persistent executor: statically split share of each matvec
  int persist_claim_ctrs = 8;       // persistent executor: counters for the dynamically claimed rest
  int attn_cta_slots = 128;         // decode attention: cache slots per CTA before a kv head splits further
  int attn_cluster_slots = 1024;    // decode attention: slots per CTA of one cluster before a kv head takes more clusters
  bool fp8_mma = false;             // fp8 weights: matvec on the tensor cores, grouped layout (measured slower)
  // batched prefill: GEMMs that take the activations' fp16 remainder plane besides their values (bit 0
  // QKV, 1 wo, 2 gate/up, 3 w2).  Measured (7B, 3202-token prompt): all four 94.5 ms, worst logit
  // 0.0072 against yalm's CPU path; QKV + wo (the default) 62.9 ms, 0.0107; the gate is 2e-2.
  int prefill_planes = 3;
  int attn_cluster = 0;             // decode attention: CTAs per cluster (0: chosen by attn_prepare)
  int attn_clusters_per_head = 0;   // decode attention: clusters per kv head (0: chosen by attn_prepare)

  // Defaults, overridable with YB_TUNE="stage=16384,budget=100000,slots=8,l2pf=4,l2wo=2,l2qkv=4,ctas=2,aslots=128,acslots=1024,acl=0,acs=0,fp8mma=0,pfplanes=3"
  // (read once per process) for tuning sweeps.
  static LaunchTuning from_env();
};

struct GemvPlan {
  bool ok;
  const void* fn;
  int kpt, rt, grid, n_slots, red_floats;
  int wt;  // weight mode of the kernel: 0 fp16, 1 fp8 on the CUDA cores, 2 fp8 on the tensor cores
  unsigned stage_bytes;
  size_t smem;
  bool norm;  // the kernel RMS-normalises x (GemvArgs::norm_w must then be set)
};

int gemv_kpt_for(int cols, int esz = 2);  // esz: weight bytes (2 fp16, 1 fp8 E5M2)
// tp_in: the kernel also adds the tensor-parallel partial sums of the previous row-parallel matvec
// to its (normalised) input (GemvArgs::tp_ll).
GemvPlan gemv_plan(int rows, int cols, int epi, bool norm, int n_sms, const LaunchTuning& tune, bool tp_in = false,
                   int esz = 2);
cudaError_t gemv_prepare(const GemvPlan& p);  // once per plan, outside stream capture
// fp8 matrices for the tensor-core matvec (GemvPlan::wt == 2): [rows][cols] row-major (cols a
// multiple of 16) re-laid into 16-row groups of [16-column chunk][row][16 bytes], rows padded with
// zeros to a multiple of 16; a column panel starting at column c of such a matrix begins c * 16
// bytes in, groups cols * 16 bytes apart (GemvArgs::ldw = cols).
size_t fp8_group_bytes(long long rows, int cols);
cudaError_t fp8_group_layout(const void* src, void* dst, long long rows, int cols, cudaStream_t stream);
cudaError_t gemv_launch(const GemvPlan& p, GemvArgs a, cudaStream_t stream, bool pdl, int l2_prefetch_stages);

// Raises a kernel's dynamic shared-memory cap to everything the device allows next to the kernel's
// static shared memory (a cap, not a reservation), once per kernel, outside stream capture.
inline cudaError_t raise_smem_cap(const void* fn) {
  int dev = 0, optin = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  if (e != cudaSuccess) return e;
  cudaFuncAttributes fa;
  e = cudaFuncGetAttributes(&fa, fn);
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, optin - (int)fa.sharedSizeBytes);
}

// cudaLaunchKernelEx with the programmatic-stream-serialization attribute when `pdl` is set, so the
// kernel may begin while the previous kernel in the stream is still running (it must call
// griddepcontrol.wait before reading that kernel's results).
template <typename Args>
inline cudaError_t launch_kernel(const void* fn, dim3 grid, dim3 block, size_t smem, cudaStream_t stream, bool pdl,
                                 Args* args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  void* params[] = {args};
  return cudaLaunchKernelExC(&cfg, fn, params);
}

}  // namespace yb
