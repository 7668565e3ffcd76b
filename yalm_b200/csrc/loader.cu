// Weight upload fast path: host rows gathered into pinned staging buffers by several threads,
// each buffer sent with cudaMemcpyAsync on a copy stream while the next one is filled.
//
// yalm uploads each tensor with a synchronous cudaMemcpy from the mmap'd .yalm pages
// (upload_cuda, src/infer.cu:50-58, called from Model::cuda, src/model.cpp:437-451); here the page
// reads run in parallel and overlap the PCIe transfers, and the tensor-parallel slicing and the
// W1/W3 row interleave are done while gathering, so each device tensor is written once.
#include "loader.h"

#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

namespace yb {

namespace {
constexpr size_t kStageBytes = (size_t)64 << 20;  // one staging buffer
constexpr int kStages = 4;

int env_threads() {
  const char* v = std::getenv("YB_LOAD_THREADS");
  int n = v ? std::atoi(v) : 0;
  if (n <= 0) {
    // twice the cores: the gather threads spend much of their time in page faults on the
    // mapped checkpoint (measured on a 16-core host: 16 threads 12.6 GB/s, 32 threads 16.4 GB/s)
    n = 2 * (int)std::thread::hardware_concurrency();
    n = std::min(std::max(n, 1), 32);
  }
  return n;
}
}  // namespace

struct Loader::Impl {
  cudaStream_t stream = nullptr;
  unsigned char* stage[kStages] = {};
  cudaEvent_t done[kStages] = {};
  bool used[kStages] = {};
  int next = 0;
  int threads = 1;
  size_t bytes = 0;
  double t_gather = 0, t_wait = 0;  // seconds spent gathering rows / waiting for a free buffer
  std::chrono::steady_clock::time_point t0 = std::chrono::steady_clock::now();
};

Loader::Loader() : p_(new Impl) {}

Loader::~Loader() {
  if (!p_) return;
  if (p_->stream) cudaStreamSynchronize(p_->stream);
  for (int i = 0; i < kStages; ++i) {
    if (p_->done[i]) cudaEventDestroy(p_->done[i]);
    if (p_->stage[i]) cudaFreeHost(p_->stage[i]);
  }
  if (p_->stream) cudaStreamDestroy(p_->stream);
  delete p_;
}

int Loader::init() {
  YB_CK(cudaStreamCreateWithFlags(&p_->stream, cudaStreamNonBlocking));
  for (int i = 0; i < kStages; ++i) {
    YB_CK(cudaHostAlloc(reinterpret_cast<void**>(&p_->stage[i]), kStageBytes, cudaHostAllocDefault));
    YB_CK(cudaEventCreateWithFlags(&p_->done[i], cudaEventDisableTiming));
  }
  p_->threads = env_threads();
  return 0;
}

int Loader::rows(void* dst, size_t n_rows, size_t row_bytes, const std::function<const void*(size_t)>& src_row) {
  if (row_bytes == 0 || n_rows == 0) return 0;
  if (row_bytes > kStageBytes) {
    // rows larger than a stage (not produced by any .yalm tensor layout here): split each row
    for (size_t r = 0; r < n_rows; ++r) {
      const unsigned char* s = static_cast<const unsigned char*>(src_row(r));
      for (size_t o = 0; o < row_bytes; o += kStageBytes) {
        const size_t n = std::min(kStageBytes, row_bytes - o);
        int rc = rows(static_cast<unsigned char*>(dst) + r * row_bytes + o, 1, n,
                      [s, o](size_t) { return static_cast<const void*>(s + o); });
        if (rc) return rc;
      }
    }
    return 0;
  }
  const size_t per_stage = kStageBytes / row_bytes;
  for (size_t r0 = 0; r0 < n_rows; r0 += per_stage) {
    const size_t r1 = std::min(n_rows, r0 + per_stage);
    const int b = p_->next;
    p_->next = (p_->next + 1) % kStages;
    using clk = std::chrono::steady_clock;
    const auto tw = clk::now();
    if (p_->used[b]) YB_CK(cudaEventSynchronize(p_->done[b]));  // the copy out of this buffer is done
    const auto tg = clk::now();
    p_->t_wait += std::chrono::duration<double>(tg - tw).count();
    unsigned char* st = p_->stage[b];
    // gather rows [r0, r1) into the staging buffer, split across threads by row ranges
    const size_t nr = r1 - r0;
    const int nt = (int)std::min<size_t>((size_t)p_->threads, std::max<size_t>(1, nr * row_bytes / ((size_t)1 << 20)));
    auto work = [&](int ti) {
      const size_t a = r0 + nr * ti / nt, z = r0 + nr * (ti + 1) / nt;
      for (size_t r = a; r < z; ++r) std::memcpy(st + (r - r0) * row_bytes, src_row(r), row_bytes);
    };
    if (nt <= 1) {
      work(0);
    } else {
      std::vector<std::thread> pool;
      pool.reserve(nt - 1);
      for (int ti = 1; ti < nt; ++ti) pool.emplace_back(work, ti);
      work(0);
      for (auto& th : pool) th.join();
    }
    p_->t_gather += std::chrono::duration<double>(clk::now() - tg).count();
    YB_CK(cudaMemcpyAsync(static_cast<unsigned char*>(dst) + r0 * row_bytes, st, nr * row_bytes,
                          cudaMemcpyHostToDevice, p_->stream));
    YB_CK(cudaEventRecord(p_->done[b], p_->stream));
    p_->used[b] = true;
    p_->bytes += nr * row_bytes;
  }
  return 0;
}

int Loader::contiguous(void* dst, const void* src, size_t bytes) {
  const size_t row = std::min(bytes, kStageBytes / 16);
  const size_t n_full = bytes / row, tail = bytes - n_full * row;
  const unsigned char* s = static_cast<const unsigned char*>(src);
  int rc = rows(dst, n_full, row, [s, row](size_t r) { return static_cast<const void*>(s + r * row); });
  if (rc || !tail) return rc;
  return rows(static_cast<unsigned char*>(dst) + n_full * row, 1, tail,
              [s, n_full, row](size_t) { return static_cast<const void*>(s + n_full * row); });
}

int Loader::finish() {
  YB_CK(cudaStreamSynchronize(p_->stream));
  const char* dbg = std::getenv("YB_LOAD_DEBUG");
  if (dbg && dbg[0] == '1') {
    const double total = std::chrono::duration<double>(std::chrono::steady_clock::now() - p_->t0).count();
    std::fprintf(stderr, "[yalm_b200 loader] %.2f GB in %.3f s (%.1f GB/s): gather %.3f s, waiting for buffers %.3f s, %d threads\n",
                 p_->bytes / 1e9, total, p_->bytes / 1e9 / total, p_->t_gather, p_->t_wait, p_->threads);
  }
  return 0;
}

size_t Loader::bytes() const { return p_->bytes; }

}  // namespace yb
