// NF4 linear entry points (forward / input gradient).
//
// Path selection for the NF4 linear:
//   * tcgen05 path (gemm_sm100.cuh): k_in % 64 == 0, 16-byte aligned operands and,
//     for dX, n_out % 8 == 0.  Covers every Qwen2.5 projection.
//   * otherwise: standalone NF4 decode into the caller's workspace, then a tiled
//     CUDA-core GEMM (fp32 accumulation) -- odd shapes from the reference's
//     tests such as (7, 13) or (17, 127).
// Both paths compute D = A.B^T + LA.LB^T + bias in fp32 and round once to fp16.
#pragma once

#include "common.cuh"
#include "gemm_host.cuh"
#include "nf4_smallm.cuh"
#include "nf4_lut.cuh"
#include "nf4_dequant.cuh"

namespace sb {

// ------------------------------------------------------------ CUDA-core fallback
// out[m, n] = sum_k A[m, k] * B(n, k) (+ LoRA, + bias); B(n, k) = W[n, k] (fwd) or W[k, n] (dx).
constexpr int kFbTile = 32;

template <bool TRANS>
__global__ void __launch_bounds__(256) fallback_gemm_kernel(
    const __half* __restrict__ A, int64_t M, int64_t N, int64_t K, const __half* __restrict__ W,
    int64_t ldw, const __half* __restrict__ LA, const __half* __restrict__ LB, int r,
    const __half* __restrict__ bias, __half* __restrict__ out) {
  __shared__ float As[kFbTile][kFbTile + 1];
  __shared__ float Bs[kFbTile][kFbTile + 1];
  const int tx = threadIdx.x % kFbTile, ty = threadIdx.x / kFbTile;  // 32 x 8
  const int64_t m0 = static_cast<int64_t>(blockIdx.y) * kFbTile, n0 = static_cast<int64_t>(blockIdx.x) * kFbTile;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int64_t k0 = 0; k0 < K; k0 += kFbTile) {
    for (int i = ty; i < kFbTile; i += 8) {
      const int64_t m = m0 + i, k = k0 + tx;
      As[i][tx] = (m < M && k < K) ? __half2float(A[m * K + k]) : 0.0f;
      const int64_t n = n0 + i;
      float b = 0.0f;
      if (n < N && k < K) b = __half2float(TRANS ? W[k * ldw + n] : W[n * ldw + k]);
      Bs[i][tx] = b;
    }
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < kFbTile; ++kk) {
      const float b = Bs[tx][kk];
#pragma unroll
      for (int q = 0; q < 4; ++q) acc[q] = fmaf(As[ty + 8 * q][kk], b, acc[q]);
    }
    __syncthreads();
  }
  const int64_t n = n0 + tx;
  if (n >= N) return;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int64_t m = m0 + ty + 8 * q;
    if (m >= M) continue;
    float v = acc[q];
    for (int j = 0; j < r; ++j) v = fmaf(__half2float(LA[m * r + j]), __half2float(LB[n * r + j]), v);
    if (bias) v += __half2float(bias[n]);
    out[m * N + n] = __float2half_rn(v);
  }
}

inline int nf4_linear_fallback(bool dx, const uint16_t* act, int64_t m, const sb_nf4_weight& w,
                               const uint16_t* bias, const uint16_t* lora_a,
                               const uint16_t* lora_b, int r, uint16_t* out, void* workspace,
                               size_t workspace_bytes, cudaStream_t stream) {
  const size_t need = static_cast<size_t>(w.n_out) * w.k_in * 2;
  if (!workspace || workspace_bytes < need) {
    return fail(SB_EWORKSPACE, "NF4 linear fallback needs " + std::to_string(need) + " workspace bytes");
  }
  uint16_t* dense = static_cast<uint16_t*>(workspace);
  ScaleSource src{w.qabs, w.absmax2, w.code2, w.offset, nullptr};
  if (int rc = launch_nf4_dequant(w.packed, src, dense, w.n_out * w.k_in, stream)) return rc;
  const int64_t N = dx ? w.k_in : w.n_out, K = dx ? w.n_out : w.k_in;
  dim3 grid(static_cast<unsigned>((N + kFbTile - 1) / kFbTile), static_cast<unsigned>((m + kFbTile - 1) / kFbTile));
  const __half* A = reinterpret_cast<const __half*>(act);
  const __half* W = reinterpret_cast<const __half*>(dense);
  if (dx) {
    fallback_gemm_kernel<true><<<grid, 256, 0, stream>>>(A, m, N, K, W, w.k_in,
        reinterpret_cast<const __half*>(lora_a), reinterpret_cast<const __half*>(lora_b), r,
        reinterpret_cast<const __half*>(bias), reinterpret_cast<__half*>(out));
  } else {
    fallback_gemm_kernel<false><<<grid, 256, 0, stream>>>(A, m, N, K, W, w.k_in,
        reinterpret_cast<const __half*>(lora_a), reinterpret_cast<const __half*>(lora_b), r,
        reinterpret_cast<const __half*>(bias), reinterpret_cast<__half*>(out));
  }
  count_launch();
  return check_launch("fallback_gemm_kernel");
}

// Small-M kernel choice, read per call: SB_SMALLM=mma takes the decode-to-shared
// mma.sync kernel (nf4_smallm.cuh) for the forward and dX, "lut" the
// unscaled-table lookup mode of nf4_lut.cuh for the forward (reductions <= 9216),
// "exact" its exact-decode mode; unset takes the exact mode.  Except under "mma",
// dX takes nf4_lut.cuh's warp-staged dX kernel.
enum SmallmKernel { kSmallmExact = 0, kSmallmLut = 1, kSmallmMma = 2 };
inline int smallm_kernel() {
  const char* e = std::getenv("SB_SMALLM");
  if (!e || !*e) return kSmallmExact;
  const std::string v(e);
  return v == "mma" ? kSmallmMma : (v == "lut" ? kSmallmLut : kSmallmExact);
}

// Activations of at most 16 rows take the streaming small-M kernel (weight-read bound).
inline bool smallm_ok(int64_t m, int64_t n_out, int64_t k_in, bool dx) {
  return m >= 1 && m <= smallm::kRows && k_in % 64 == 0 && (!dx || n_out % 8 == 0) &&
         n_out * k_in < (int64_t(1) << 32);  // byte and block offsets fit 32 bits
}

inline int nf4_linear(bool dx, const uint16_t* act, int64_t m, const sb_nf4_weight* w,
                      const uint16_t* bias, const uint16_t* lora_a, const uint16_t* lora_b, int r,
                      uint16_t* out, void* workspace, size_t workspace_bytes, void* stream) {
  SB_REQUIRE(w != nullptr, "NULL weight descriptor");
  SB_REQUIRE(m >= 0 && w->n_out > 0 && w->k_in > 0, "expected m >= 0 and a non-empty weight");
  SB_REQUIRE(r >= 0 && r <= 64, "LoRA rank must be in [0, 64]");
  SB_REQUIRE(!dx || bias == nullptr, "bias applies to the forward only");
  if (m == 0) return SB_OK;
  SB_REQUIRE(act && out && w->packed && w->qabs && w->absmax2 && w->code2 && w->offset, "NULL pointer argument");
  SB_REQUIRE(r == 0 || (lora_a && lora_b), "LoRA factors missing");
  cudaStream_t st = as_stream(stream);
  const bool tc_rank = (r == 0 || r == 16 || r == 32 || r == 64);
  const bool ptrs_ok = aligned(act, 16) && aligned(w->packed, 16) &&
                       (r == 0 || (aligned(lora_a, 16) && aligned(lora_b, 16)));
  if (smallm_ok(m, w->n_out, w->k_in, dx) && aligned(act, 16) && aligned(w->packed, 16) &&
      (r == 0 || (aligned(lora_a, 2) && aligned(lora_b, 2)))) {
    const int kind = smallm_kernel();
    if (!dx && kind != kSmallmMma && lut::fwd_ok(m, w->n_out, w->k_in, kind == kSmallmExact)) {
      return lut::run_fwd(act, m, *w, bias, lora_a, lora_b, r, out, kind == kSmallmExact, st);
    }
    if (dx && kind != kSmallmMma && lut::dx_ok(m, w->n_out, w->k_in)) {
      return lut::run_dx(act, m, *w, lora_a, lora_b, r, out, st);
    }
    return smallm::run(dx, act, m, *w, bias, lora_a, lora_b, r, out, workspace, workspace_bytes, st);
  }
  if (tc_rank && ptrs_ok && gemm::nf4_tc_shape_ok(m, w->n_out, w->k_in, dx)) {
    return gemm::nf4_linear_tc(dx, act, m, *w, bias, lora_a, lora_b, r, out, workspace,
                               workspace_bytes, st);
  }
  return nf4_linear_fallback(dx, act, m, *w, bias, lora_a, lora_b, r, out, workspace,
                             workspace_bytes, st);
}

}  // namespace sb

extern "C" {

size_t sb_nf4_linear_workspace_bytes(int64_t m, int64_t n_out, int64_t k_in, int dx) {
  if (m <= 0 || n_out <= 0 || k_in <= 0) return 0;
  if (sb::smallm_ok(m, n_out, k_in, dx != 0)) {
    return sb::smallm::plan(dx ? n_out : k_in, dx ? k_in : n_out).workspace;
  }
  // Shapes the tcgen05 path takes (with 16-byte aligned operands, which the
  // caller guarantees) need only its stream-K scratch; others the decoded weight.
  if (!sb::gemm::nf4_tc_shape_ok(m, n_out, k_in, dx != 0)) return static_cast<size_t>(n_out) * k_in * 2;
  return sb::gemm::nf4_plan(m, n_out, k_in, dx != 0).workspace;
}

int sb_nf4_linear_fwd(const uint16_t* x, int64_t m, const sb_nf4_weight* w, const uint16_t* bias,
                      const uint16_t* lora_a, const uint16_t* lora_b, int r, uint16_t* y,
                      void* workspace, size_t workspace_bytes, void* stream) {
  return sb::nf4_linear(false, x, m, w, bias, lora_a, lora_b, r, y, workspace, workspace_bytes, stream);
}

int sb_nf4_linear_dx(const uint16_t* dy, int64_t m, const sb_nf4_weight* w, const uint16_t* lora_a,
                     const uint16_t* lora_b, int r, uint16_t* dx, void* workspace,
                     size_t workspace_bytes, void* stream) {
  return sb::nf4_linear(true, dy, m, w, nullptr, lora_a, lora_b, r, dx, workspace, workspace_bytes, stream);
}

}  // extern "C"
