// Shared helpers for the soupsuck_b200 CUDA library (sm_100a only).
//
// * host-side status / last-error plumbing for the C ABI;
// * dtype-generic scalar load/store for the row kernels;
// * PTX wrappers for mbarriers, TMA (cp.async.bulk.tensor, no multicast),
//   tcgen05 (TMEM alloc, UMMA issue/commit, TMEM loads) with BOUNDED waits:
//   every spin on an mbarrier gives up after kWaitNanos of %globaltimer time,
//   records a code in the device error word and returns false.  Nothing here
//   traps the GPU.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdio>
#include <string>

#include "../../include/soupsuck_b200.h"

namespace sb {

// ----------------------------------------------------------------- host side
void set_error(const std::string& msg);
int fail(int code, const std::string& msg);
int check_launch(const char* what);
void count_launch(int n = 1);
int device_sm_count();
int device_error_word_address(int** ptr);

#define SB_REQUIRE(cond, msg)                                  \
  do {                                                         \
    if (!(cond)) return ::sb::fail(SB_EINVAL, std::string(msg)); \
  } while (0)

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline bool aligned(const void* p, size_t a) {
  return (reinterpret_cast<uintptr_t>(p) % a) == 0;
}

// ----------------------------------------------------------------- device side
__device__ __forceinline__ float ld_as_f32(const void* p, int dt, int64_t i) {
  return dt == SB_F32 ? static_cast<const float*>(p)[i]
                      : __half2float(static_cast<const __half*>(p)[i]);
}

__device__ __forceinline__ void st_from_f32(void* p, int dt, int64_t i, float v) {
  if (dt == SB_F32) {
    static_cast<float*>(p)[i] = v;
  } else {
    static_cast<__half*>(p)[i] = __float2half_rn(v);
  }
}

// Round an fp32 value to the given storage dtype and return it as fp32.
__device__ __forceinline__ float round_to(float v, int dt) {
  return dt == SB_F32 ? v : __half2float(__float2half_rn(v));
}

__host__ __device__ __forceinline__ int promote(int a, int b) {
  return (a == SB_F32 || b == SB_F32) ? SB_F32 : SB_F16;
}

// Device error word: set by kernels whose bounded waits expire.  Defined here
// because the library is one translation unit (soupsuck_b200.cu).
__device__ int g_device_error = 0;

enum DeviceError : int {
  kErrWaitFull = 1 << 0,
  kErrWaitEmpty = 1 << 1,
  kErrWaitDecoded = 1 << 2,
  kErrWaitAccFull = 1 << 3,
  kErrWaitAccEmpty = 1 << 4,
  kErrWaitDrain = 1 << 5,
  kErrTmemAlloc = 1 << 6,
};

// 2 seconds: far above any legitimate wait in these kernels.
constexpr uint64_t kWaitNanos = 2000000000ull;

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// --------------------------------------------------------------- mbarriers
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
          smem_addr(bar)),
      "r"(bytes)
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t addr, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(addr), "r"(parity)
      : "memory");
  return ok != 0;
}

// Same, letting the hardware suspend the thread until the phase completes or
// `hint_ns` elapse: a waiting warp then takes no issue slots from the warps
// that share its scheduler (a polling loop measurably slowed the UMMA issuer).
__device__ __forceinline__ bool mbar_try_wait_suspend(uint32_t addr, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(addr), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

// Suspension bound of one wait round: the abort flag and the time limit are
// checked at least this often.
constexpr uint32_t kSuspendHintNanos = 100000;

// Bounded wait for the phase with the given parity to complete.  Returns false
// (and records `err`) once kWaitNanos elapse, or at once if `abort` is set.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int err,
                                          volatile int* abort) {
  const uint32_t addr = smem_addr(bar);
  if (mbar_try_wait(addr, parity)) return true;
  const uint64_t start = global_timer_ns();
  while (true) {
    if (mbar_try_wait_suspend(addr, parity, kSuspendHintNanos)) return true;
    if (*abort) return false;
    if (global_timer_ns() - start > kWaitNanos) {
      atomicOr(&g_device_error, err);
      *abort = 1;
      return false;
    }
  }
}

// ------------------------------------------------ programmatic dependent launch
// Wait until the preceding kernel of the stream (launched before this one with
// programmatic stream serialisation allowed) has completed and its memory
// operations are visible; a no-op for an ordinary launch.
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Let the next kernel of the stream be scheduled once every CTA of this grid has
// reached this point (it still waits for this grid's completion before touching
// memory).
__device__ __forceinline__ void launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" :::); }

// ---------------------------------------------------------------- TMA loads
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2-D tiled bulk tensor load into this CTA's shared memory; completes bytes on `bar`.
// Coordinates: x = innermost (element index along the contiguous dimension), y = row.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_addr(dst_smem)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16 (fp16 x fp16 -> fp32).
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive (once) on an mbarrier when all previously issued UMMAs of this thread complete.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_addr(bar))
      : "memory");
}

// 32 lanes x 32 consecutive fp32 columns per warp (lane i <- TMEM lane base+i).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ------------------------------------------------------------ UMMA descriptors
// Shared-memory matrix descriptor (sm_100 format): start address, leading and
// stride byte offsets (all >> 4), version 1, swizzle layout in bits 61-63.
enum SmemLayout : uint32_t { kSwizzleNone = 0, kSwizzle128B = 2, kSwizzle64B = 4, kSwizzle32B = 6 };

__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo_bytes,
                                              uint32_t sbo_bytes, uint32_t layout) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;  // version for sm_100
  d |= static_cast<uint64_t>(layout & 0x7u) << 61;
  return d;
}

// Instruction descriptor, kind::f16 with fp16 A/B and fp32 accumulate.
// a_mn / b_mn: operand is MN-major (1) or K-major (0).
__host__ __device__ constexpr uint32_t idesc_f16_f32(uint32_t m, uint32_t n, uint32_t a_mn,
                                                     uint32_t b_mn) {
  return (1u << 4)                 // D format: f32
         | (0u << 7)               // A format: f16
         | (0u << 10)              // B format: f16
         | (a_mn << 15) | (b_mn << 16) | ((n >> 3) << 17) | ((m >> 4) << 24);
}

}  // namespace sb
