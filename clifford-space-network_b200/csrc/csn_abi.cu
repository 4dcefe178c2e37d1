// csn_abi.cu -- library identity and error reporting for the C ABI.
#include <stdio.h>
#include <string.h>

#include <mutex>
#include <string>
#include <vector>

#include "csn_internal.h"

namespace csn {

namespace {
thread_local char g_last_error[512] = "";
}

int set_error(int code, const char* msg) {
  snprintf(g_last_error, sizeof(g_last_error), "%s", msg ? msg : "");
  return code;
}

int set_cuda_error(cudaError_t e, const char* where) {
  snprintf(g_last_error, sizeof(g_last_error), "%s: %s (%s)", where, cudaGetErrorString(e),
           cudaGetErrorName(e));
  return CSN_ERR_CUDA;
}

int check_launch(const char* where) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e, where);
  return CSN_OK;
}

namespace {
struct TimedPair {
  std::string name;
  cudaEvent_t e0, e1;
};
std::mutex g_tmu;
bool g_timing = false;
std::vector<TimedPair> g_pairs;
}  // namespace

bool timing_on() { return g_timing; }

void timing_push(const char* name, cudaEvent_t e0, cudaEvent_t e1) {
  std::lock_guard<std::mutex> lk(g_tmu);
  g_pairs.push_back({name, e0, e1});
}

}  // namespace csn

extern "C" int csn_timing_enable(int on) {
  std::lock_guard<std::mutex> lk(csn::g_tmu);
  csn::g_timing = on != 0;
  return CSN_OK;
}

extern "C" int csn_timing_reset(void) {
  std::lock_guard<std::mutex> lk(csn::g_tmu);
  for (auto& p : csn::g_pairs) {
    cudaEventSynchronize(p.e1);
    cudaEventDestroy(p.e0);
    cudaEventDestroy(p.e1);
  }
  csn::g_pairs.clear();
  return CSN_OK;
}

extern "C" int csn_timing_read(const char* name, double* total_ms, int64_t* count) {
  std::lock_guard<std::mutex> lk(csn::g_tmu);
  double tot = 0.0;
  int64_t n = 0;
  for (auto& p : csn::g_pairs) {
    if (name && strcmp(name, p.name.c_str()) != 0) continue;
    cudaError_t e = cudaEventSynchronize(p.e1);
    if (e != cudaSuccess) return csn::set_cuda_error(e, "csn_timing_read");
    float ms = 0.0f;
    e = cudaEventElapsedTime(&ms, p.e0, p.e1);
    if (e != cudaSuccess) return csn::set_cuda_error(e, "csn_timing_read");
    tot += ms;
    ++n;
  }
  if (total_ms) *total_ms = tot;
  if (count) *count = n;
  return CSN_OK;
}

#ifndef CSN_SOURCE_HASH
#define CSN_SOURCE_HASH "unknown"
#endif
// "csn_b200 <version> (sm_100a) src <hash>": the hash of the sources the library was built
// from (computed by the build script), so a caller can check which build it loaded
extern "C" const char* csn_version(void) { return "csn_b200 0.2.0 (sm_100a) src " CSN_SOURCE_HASH; }

extern "C" const char* csn_last_error(void) { return csn::g_last_error; }
