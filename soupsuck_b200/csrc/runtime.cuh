// Host runtime of the C ABI: error strings, launch counting, device queries and
// the device error word that bounded waits write.
#pragma once

#include <atomic>
#include <mutex>
#include <string>

#include "common.cuh"

namespace sb {

namespace {
thread_local std::string t_last_error;
std::atomic<int64_t> g_launches{0};
}  // namespace

void set_error(const std::string& msg) { t_last_error = msg; }

int fail(int code, const std::string& msg) {
  set_error(msg);
  return code;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    return fail(SB_ECUDA, std::string(what) + ": " + cudaGetErrorString(e));
  }
  return SB_OK;
}

void count_launch(int n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

int device_sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  static std::mutex mu;
  static int cached[64] = {0};
  std::lock_guard<std::mutex> lock(mu);
  if (dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cached[dev] = n > 0 ? n : 148;
  }
  return cached[dev];
}

int device_error_word_address(int** ptr) {
  cudaError_t e = cudaGetSymbolAddress(reinterpret_cast<void**>(ptr), g_device_error);
  if (e != cudaSuccess) return fail(SB_ECUDA, std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
  return SB_OK;
}

}  // namespace sb

extern "C" {

int sb_abi_version(void) { return 1; }

const char* sb_last_error(void) { return sb::t_last_error.c_str(); }

int64_t sb_launch_count(void) { return sb::g_launches.load(); }

int sb_take_device_error(void* stream, int* flag) {
  SB_REQUIRE(flag != nullptr, "flag must not be NULL");
  int* dptr = nullptr;
  int rc = sb::device_error_word_address(&dptr);
  if (rc) return rc;
  cudaStream_t s = sb::as_stream(stream);
  int host = 0;
  cudaError_t e = cudaMemcpyAsync(&host, dptr, sizeof(int), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaMemsetAsync(dptr, 0, sizeof(int), s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return sb::fail(SB_ECUDA, std::string("sb_take_device_error: ") + cudaGetErrorString(e));
  *flag = host;
  return SB_OK;
}

}  // extern "C"
