// TEST INFRASTRUCTURE ONLY — linked into the CPU-only build of yalm's decode path (oracle/Makefile).
//
// Definitions for the CUDA-side symbols that src/model.cpp references but that the CPU path never
// calls (upload_cuda & co from src/infer.cu:60-91, the coop entry points from src/coop.h:5-6,
// libgemm_init from src/libgemm.h:12, and the `_block_cuda*` / `_forward_cuda*` members).  Each
// aborts: reaching one means the CPU path was not taken.  The GPU build links the reference's own
// CUDA objects instead.
#include "model.h"
#include "coop.h"
#include "libgemm.h"

#include <cstdio>
#include <cstdlib>
#include <string>

[[noreturn]] static void not_cpu(const char* what) {
  std::fprintf(stderr, "oracle/ref_driver: CUDA symbol %s reached on the CPU path\n", what);
  std::abort();
}

// ---- CUDA-side symbols referenced from src/model.cpp, unused on the CPU path ----
extern "C" void* upload_cuda(void*, size_t) { not_cpu("upload_cuda"); }
extern "C" void* download_cuda(void*, size_t, std::string) { not_cpu("download_cuda"); }
extern "C" void register_cuda_host(void*, size_t) { not_cpu("register_cuda_host"); }
extern "C" void free_cuda(void*) { not_cpu("free_cuda"); }
extern "C" void unregister_cuda_host(void*) { not_cpu("unregister_cuda_host"); }
extern "C" void set_cuda_device(int) { not_cpu("set_cuda_device"); }
extern "C" void init_cuda_stream(cudaStream_t*) { not_cpu("init_cuda_stream"); }
void yalm_coop_prepare(Model&) { not_cpu("yalm_coop_prepare"); }
void yalm_coop_forward(Model&, InferenceState&, int, int, InferenceMode) { not_cpu("yalm_coop_forward"); }
void libgemm_init(cudaStream_t, LibGemmBackend) { not_cpu("libgemm_init"); }
template <typename T>
void Block::_block_cuda(InferenceState&, int, int, int, int) const { not_cpu("Block::_block_cuda"); }
template <typename T>
void Block::_block_cuda_lib(InferenceState&, int, int, int, int) const { not_cpu("Block::_block_cuda_lib"); }
template void Block::_block_cuda<float>(InferenceState&, int, int, int, int) const;
template void Block::_block_cuda<f16_t>(InferenceState&, int, int, int, int) const;
template void Block::_block_cuda_lib<f16_t>(InferenceState&, int, int, int, int) const;
void Model::_forward_cuda(InferenceState&, int, int, InferenceMode) { not_cpu("Model::_forward_cuda"); }
void Model::_forward_cuda_lib(InferenceState&, int, int, InferenceMode) { not_cpu("Model::_forward_cuda_lib"); }
