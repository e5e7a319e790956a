// LoRA weight-gradient reduction that allocates nothing.
//
// sb_lora_reduce needs fp32 partial sums in a caller-provided workspace.  Some
// callers cannot provide one: code that runs where device allocation is not
// allowed or not available -- a host framework whose device memory is planned
// once up front (static memory planners, embedded deployments that forbid
// allocation after start-up), foreign-language bindings that hold no CUDA
// allocator of their own, or a training step that must not grow its memory
// footprint.  For them sb_lora_reduce_static keeps the partial sums in a
// fixed device array owned by this library, declared below.
//
// Limits and sharing:
//   * kStaticPartialFloats fp32 values (8 MiB).  The row reduction is split into
//     as many slices as the array holds (at most the split count sb_lora_reduce
//     would use); r * w above kStaticPartialFloats is rejected with SB_EINVAL.
//   * Every GPU that loads the library holds the 8 MiB array until the process exits.
//   * Every call shares the array and it keeps the last call's contents; each
//     call overwrites every partial sum it reads, so nothing has to start at zero.
//     Calls whose kernels overlap on the GPU (different streams of the same
//     device, or host threads issuing concurrently) race on it: serialise them.
//   * The first call on each device looks up the array's device address with
//     that device current (cudaGetSymbolAddress) and caches it; make that first
//     call before any stream capture.
#pragma once

#include <mutex>

#include "common.cuh"
#include "lora_mma.cuh"

namespace sb {
namespace lora_static {

constexpr int64_t kStaticPartialFloats = int64_t(1) << 21;  // 8 MiB of fp32

static __device__ __align__(256) float g_static_partials[kStaticPartialFloats];

// Device address of g_static_partials for the current device (set up once per device).
inline int partials_address(float** out) {
  static std::mutex mu;
  static float* cached[64] = {nullptr};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(SB_ECUDA, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return fail(SB_EUNSUPPORTED, "device index above 63");
  std::lock_guard<std::mutex> lock(mu);
  if (!cached[dev]) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_static_partials);
    if (e != cudaSuccess || ptr == nullptr) {
      return fail(SB_ECUDA, std::string("cudaGetSymbolAddress(g_static_partials): ") + cudaGetErrorString(e));
    }
    cached[dev] = static_cast<float*>(ptr);
  }
  *out = cached[dev];
  return SB_OK;
}

}  // namespace lora_static
}  // namespace sb

extern "C" {

int sb_lora_reduce_static(const uint16_t* pt, int64_t ldp, const uint16_t* q, int64_t m,
                          int64_t w, int r, float scale, int transpose, void* out, int out_dtype,
                          void* stream) {
  using sb::lora_static::kStaticPartialFloats;
  SB_REQUIRE(m >= 0 && w > 0, "expected m >= 0 and w > 0");
  SB_REQUIRE(r == 16 || r == 32 || r == 64, "rank must be 16, 32 or 64");
  SB_REQUIRE(ldp >= m && ldp % 16 == 0, "ldp must be >= m and a multiple of 16 (zero padded)");
  SB_REQUIRE(w % 2 == 0, "w must be even");
  SB_REQUIRE(out_dtype == SB_F16 || out_dtype == SB_F32, "bad out dtype");
  SB_REQUIRE(out != nullptr, "NULL out");
  if (static_cast<int64_t>(r) * w > kStaticPartialFloats) {
    return sb::fail(SB_EINVAL, "sb_lora_reduce_static holds at most " + std::to_string(kStaticPartialFloats) +
                                   " partial sums (r * w); got r * w = " + std::to_string(static_cast<int64_t>(r) * w) +
                                   ": use sb_lora_reduce with a workspace");
  }
  cudaStream_t st = sb::as_stream(stream);
  if (m == 0) {
    cudaError_t e = cudaMemsetAsync(out, 0, static_cast<size_t>(r) * w * (out_dtype == SB_F32 ? 4 : 2), st);
    return e == cudaSuccess ? SB_OK : sb::fail(SB_ECUDA, cudaGetErrorString(e));
  }
  SB_REQUIRE(pt && q, "NULL pointer argument");
  SB_REQUIRE(sb::aligned(pt, 4) && sb::aligned(q, 4), "pt and q must be 4-byte aligned");
  float* partial = nullptr;
  if (int rc = sb::lora_static::partials_address(&partial)) return rc;
  int splits = sb::lora::reduce_splits(ldp, w);
  const int64_t fit = kStaticPartialFloats / (static_cast<int64_t>(r) * w);
  if (splits > fit) splits = static_cast<int>(fit);
  int64_t rows_per_split = (ldp + splits - 1) / splits;
  rows_per_split = (rows_per_split + 15) / 16 * 16;
  splits = static_cast<int>((ldp + rows_per_split - 1) / rows_per_split);
  dim3 grid(static_cast<unsigned>((w + 127) / 128), static_cast<unsigned>(splits));
  const __half* P = reinterpret_cast<const __half*>(pt);
  const __half* Q = reinterpret_cast<const __half*>(q);
  if (r == 16) sb::lora::reduce_partial_kernel<16><<<grid, 256, 0, st>>>(P, ldp, Q, m, w, rows_per_split, partial);
  else if (r == 32) sb::lora::reduce_partial_kernel<32><<<grid, 256, 0, st>>>(P, ldp, Q, m, w, rows_per_split, partial);
  else sb::lora::reduce_partial_kernel<64><<<grid, 256, 0, st>>>(P, ldp, Q, m, w, rows_per_split, partial);
  sb::count_launch();
  if (int rc = sb::check_launch("lora_reduce_partial_kernel (static partials)")) return rc;
  const int64_t total = w * r;
  sb::lora::reduce_finalize_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, st>>>(
      partial, splits, w, r, scale, transpose, out, out_dtype);
  sb::count_launch();
  return sb::check_launch("lora_reduce_finalize_kernel (static partials)");
}

}  // extern "C"
