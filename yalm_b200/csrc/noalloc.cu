// Decode attention without any device allocation by the library or the caller.
//
// yb_attention_dev needs a scratch buffer from the caller (the cluster records and the merge
// counters of the attention kernel, used where several clusters share a kv head).  Some callers cannot provide one at call time: a plugin running
// inside another framework whose allocator owns all device memory, or a serving loop that forbids
// device allocation after start-up so that latency and memory use stay fixed.  For them this file
// keeps the scratch in a fixed-size array in the library's own device memory (allocated by the
// CUDA runtime when it loads the library's device code on a GPU, and held until the process
// exits), and yb_attention_dev_noalloc runs the same kernel with it.
#include "attention.cuh"
#include "engine.h"

#include <cstring>
#include <mutex>
#include <string>

namespace {

// Scratch for yb_attention_dev_noalloc: cluster records first, then the per-kv-head merge counters.
// Its size is YB_ATTENTION_NOALLOC_SCRATCH_BYTES (include/yalm_b200.h).
constexpr size_t kNoAllocScratchBytes = YB_ATTENTION_NOALLOC_SCRATCH_BYTES;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch per device (host code cannot use the symbol itself: in host
// code its name only stands for the variable, it is not a device address).
constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch_addr[kMaxDevices] = {};

int scratch_address(void** out) {
  int dev = 0;
  YB_CK(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return yb::set_error(YB_E_INVALID, "device index out of range");
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);  // with device `dev` current
    if (e != cudaSuccess || !p)
      return yb::set_error(YB_E_CUDA, std::string("cudaGetSymbolAddress(scratch) failed: ") + cudaGetErrorString(e));
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return 0;
}

}  // namespace

extern "C" int yb_attention_dev_noalloc(float* out, const float* q, const uint16_t* k_cache, const uint16_t* v_cache,
                                        int n_heads, int n_kv_heads, int head_dim, int max_seq_len, int kv_len,
                                        void* stream) {
  using namespace yb;
  if (!out || !q || !k_cache || !v_cache || kv_len <= 0 || kv_len > max_seq_len)
    return set_error(YB_E_INVALID, "bad attention arguments");
  // the size check needs only the shape (host arithmetic, no CUDA call)
  const AttnPlan shape = attn_plan(n_heads, n_kv_heads, head_dim, max_seq_len);
  if (!shape.ok) return set_error(YB_E_UNSUPPORTED, "no attention configuration for this shape");
  const size_t part_bytes = (shape.part_floats * 4 + 255) / 256 * 256;
  const size_t need = part_bytes + (size_t)n_kv_heads * 4;
  if (need > kNoAllocScratchBytes)
    return set_error(YB_E_INVALID, "attention scratch of " + std::to_string(need) + " bytes exceeds the " +
                                       std::to_string(kNoAllocScratchBytes) +
                                       "-byte fixed buffer of yb_attention_dev_noalloc (n_heads * (head_dim + 2) * 4 per cluster "
                                       "of a kv head, up to min(32, ceil(max_seq_len / 128)) clusters, + n_kv_heads * 4)");
  AttnPlan p;
  int rc = cached_attn_plan(n_heads, n_kv_heads, head_dim, max_seq_len, &p);
  if (rc) return rc;
  void* base = nullptr;
  rc = scratch_address(&base);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  unsigned* counters = reinterpret_cast<unsigned*>(static_cast<char*>(base) + part_bytes);
  // The array keeps whatever the previous call left; the merge counters must start at zero.
  YB_CK(cudaMemsetAsync(counters, 0, (size_t)n_kv_heads * 4, s));
  AttnArgs a;
  std::memset(&a, 0, sizeof(a));
  a.q = q;
  a.k_cache = reinterpret_cast<const __half*>(k_cache);
  a.v_cache = reinterpret_cast<const __half*>(v_cache);
  a.out = out;
  a.part = static_cast<float*>(base);
  a.counters = counters;
  a.step = nullptr;
  a.kv_len = kv_len;
  a.max_seq_len = max_seq_len;
  a.cta_slots = LaunchTuning::from_env().attn_cta_slots;
  a.cluster_slots = LaunchTuning::from_env().attn_cluster_slots;
  AttnMaps m;
  if (!attn_maps(&m, a.k_cache, a.v_cache, n_kv_heads, max_seq_len, head_dim))
    return set_error(YB_E_CUDA, "tensor map encoding of the KV cache failed");
  YB_CK(attn_launch(p, a, m, s, false));
  return 0;
}
