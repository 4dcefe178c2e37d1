// csn_internal.h -- error reporting shared by the library's translation units.
#pragma once

#include <cuda_runtime.h>

#include "../../include/csn_b200.h"

namespace csn {

// Record `msg` as this thread's last error and return `code`.
int set_error(int code, const char* msg);
int set_cuda_error(cudaError_t e, const char* where);
// cudaGetLastError() after a batch of launches.
int check_launch(const char* where);

}  // namespace csn

namespace csn {

// Optional per-kernel timing (off by default).  When enabled with
// csn_timing_enable(1), every library launch wrapped in a KernelTimer records a pair
// of CUDA events on its own stream; csn_timing_read() sums the elapsed times.
bool timing_on();
void timing_push(const char* name, cudaEvent_t start, cudaEvent_t stop);

struct KernelTimer {
  const char* name;
  cudaStream_t st;
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  KernelTimer(const char* n, cudaStream_t s) : name(n), st(s) {
    if (timing_on() && cudaEventCreate(&e0) == cudaSuccess && cudaEventCreate(&e1) == cudaSuccess)
      cudaEventRecord(e0, st);
    else
      e0 = e1 = nullptr;
  }
  ~KernelTimer() {
    if (e0) {
      cudaEventRecord(e1, st);
      timing_push(name, e0, e1);
    }
  }
};

}  // namespace csn
