// Weight upload fast path (see loader.cu).
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <functional>

#include "engine.h"

namespace yb {

class Loader {
 public:
  Loader();
  ~Loader();
  Loader(const Loader&) = delete;
  Loader& operator=(const Loader&) = delete;
  int init();  // staging buffers, copy stream
  // Device rows [0, n_rows) of row_bytes each at dst (contiguous) from host rows src_row(r).
  int rows(void* dst, size_t n_rows, size_t row_bytes, const std::function<const void*(size_t)>& src_row);
  int contiguous(void* dst, const void* src, size_t bytes);
  int finish();  // waits for every copy
  size_t bytes() const;

 private:
  struct Impl;
  Impl* p_;
};

}  // namespace yb
