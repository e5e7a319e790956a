// NF4 linear entry points (forward / input gradient) and the LoRA low-rank kernels.
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
  if (tc_rank && ptrs_ok && gemm::nf4_tc_shape_ok(m, w->n_out, w->k_in, dx)) {
    return gemm::nf4_linear_tc(dx, act, m, *w, bias, lora_a, lora_b, r, out, st);
  }
  return nf4_linear_fallback(dx, act, m, *w, bias, lora_a, lora_b, r, out, workspace,
                             workspace_bytes, st);
}

// ------------------------------------------------------------ LoRA factors
// Row dot products against r <= 64 rank vectors: one warp per activation row,
// 8 halves per lane per step (16-byte loads when the row pitch allows).
template <int R>
__global__ void __launch_bounds__(256) lora_rowdot_kernel(const __half* __restrict__ X, int64_t M,
                                                          int64_t K, const __half* __restrict__ V,
                                                          int64_t v_row, int64_t v_col, int r,
                                                          float scale, __half* __restrict__ out16,
                                                          __half* __restrict__ outs16,
                                                          float* __restrict__ out32) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * 8 + warp;
  if (row >= M) return;
  float acc[R];
#pragma unroll
  for (int j = 0; j < R; ++j) acc[j] = 0.0f;
  const __half* x = X + row * K;
  for (int64_t k = lane; k < K; k += 32) {
    const float xv = __half2float(x[k]);
#pragma unroll
    for (int j = 0; j < R; ++j) {
      if (j < r) acc[j] = fmaf(xv, __half2float(V[j * v_row + k * v_col]), acc[j]);
    }
  }
#pragma unroll
  for (int j = 0; j < R; ++j) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc[j] += __shfl_xor_sync(0xffffffffu, acc[j], o);
  }
  if (lane == 0) {
    for (int j = 0; j < r; ++j) {
      if (out16) out16[row * r + j] = __float2half_rn(acc[j]);
      if (outs16) outs16[row * r + j] = __float2half_rn(acc[j] * scale);
      if (out32) out32[row * r + j] = acc[j] * scale;
    }
  }
}

template <int R>
int launch_rowdot(const uint16_t* x, int64_t m, int64_t k, const uint16_t* v, int64_t v_row,
                  int64_t v_col, int r, float scale, uint16_t* o16, uint16_t* os16, float* o32,
                  cudaStream_t st) {
  const unsigned grid = static_cast<unsigned>((m + 7) / 8);
  lora_rowdot_kernel<R><<<grid, 256, 0, st>>>(reinterpret_cast<const __half*>(x), m, k,
                                             reinterpret_cast<const __half*>(v), v_row, v_col, r,
                                             scale, reinterpret_cast<__half*>(o16),
                                             reinterpret_cast<__half*>(os16), o32);
  count_launch();
  return check_launch("lora_rowdot_kernel");
}

inline int rowdot(const uint16_t* x, int64_t m, int64_t k, const uint16_t* v, int64_t v_row,
                  int64_t v_col, int r, float scale, uint16_t* o16, uint16_t* os16, float* o32,
                  cudaStream_t st) {
  if (r <= 16) return launch_rowdot<16>(x, m, k, v, v_row, v_col, r, scale, o16, os16, o32, st);
  if (r <= 32) return launch_rowdot<32>(x, m, k, v, v_row, v_col, r, scale, o16, os16, o32, st);
  return launch_rowdot<64>(x, m, k, v, v_row, v_col, r, scale, o16, os16, o32, st);
}

// C[j, c] = scale * sum_i P[i, j] * Q[i, c]: split over rows into partial sums
// (deterministic two-stage reduction), one thread per column c.
constexpr int kTnCols = 128, kTnRows = 32;

template <int R, typename PT>
__global__ void __launch_bounds__(kTnCols) lora_tn_partial_kernel(
    const PT* __restrict__ P, const __half* __restrict__ Q, int64_t M, int64_t W, int r,
    int64_t rows_per_split, float* __restrict__ partial) {
  __shared__ float ps[kTnRows][R];
  const int64_t c = static_cast<int64_t>(blockIdx.x) * kTnCols + threadIdx.x;
  const int64_t r0 = static_cast<int64_t>(blockIdx.y) * rows_per_split;
  const int64_t r1 = r0 + rows_per_split < M ? r0 + rows_per_split : M;
  float acc[R];
#pragma unroll
  for (int j = 0; j < R; ++j) acc[j] = 0.0f;
  for (int64_t i0 = r0; i0 < r1; i0 += kTnRows) {
    __syncthreads();
    for (int t = threadIdx.x; t < kTnRows * R; t += kTnCols) {
      const int ii = t / R, j = t % R;
      const int64_t i = i0 + ii;
      float v = 0.0f;
      if (i < r1 && j < r) {
        if constexpr (sizeof(PT) == 4) v = P[i * r + j]; else v = __half2float(P[i * r + j]);
      }
      ps[ii][j] = v;
    }
    __syncthreads();
    if (c < W) {
      const int64_t lim = (r1 - i0) < kTnRows ? (r1 - i0) : kTnRows;
      for (int ii = 0; ii < lim; ++ii) {
        const float q = __half2float(Q[(i0 + ii) * W + c]);
#pragma unroll
        for (int j = 0; j < R; ++j) acc[j] = fmaf(ps[ii][j], q, acc[j]);
      }
    }
  }
  if (c < W) {
    for (int j = 0; j < r; ++j) partial[(static_cast<int64_t>(blockIdx.y) * r + j) * W + c] = acc[j];
  }
}

__global__ void lora_tn_finalize_kernel(const float* __restrict__ partial, int splits, int64_t W,
                                        int r, float scale, int transpose, float* __restrict__ out) {
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= W * r) return;
  const int64_t j = idx / W, c = idx % W;
  float acc = 0.0f;
  for (int s = 0; s < splits; ++s) acc += partial[(static_cast<int64_t>(s) * r + j) * W + c];
  acc *= scale;
  if (transpose) out[c * r + j] = acc; else out[j * W + c] = acc;
}

inline int tn_splits(int64_t m, int64_t w) {
  const int64_t col_blocks = (w + kTnCols - 1) / kTnCols;
  int64_t s = (2 * device_sm_count() + col_blocks - 1) / col_blocks;
  const int64_t max_s = (m + 63) / 64;
  if (s > max_s) s = max_s;
  if (s < 1) s = 1;
  if (s > 1024) s = 1024;
  return static_cast<int>(s);
}

template <typename PT>
int lora_tn(const PT* P, const uint16_t* Q, int64_t m, int64_t w, int r, float scale, int transpose,
            float* out, void* workspace, size_t workspace_bytes, cudaStream_t st) {
  const int splits = tn_splits(m, w);
  const size_t need = static_cast<size_t>(splits) * r * w * sizeof(float);
  if (!workspace || workspace_bytes < need) return fail(SB_EWORKSPACE, "LoRA gradient workspace too small");
  const int64_t rows_per_split = (m + splits - 1) / splits;
  dim3 grid(static_cast<unsigned>((w + kTnCols - 1) / kTnCols), static_cast<unsigned>(splits));
  float* partial = static_cast<float*>(workspace);
  const __half* q = reinterpret_cast<const __half*>(Q);
  if (r <= 16) lora_tn_partial_kernel<16, PT><<<grid, kTnCols, 0, st>>>(P, q, m, w, r, rows_per_split, partial);
  else if (r <= 32) lora_tn_partial_kernel<32, PT><<<grid, kTnCols, 0, st>>>(P, q, m, w, r, rows_per_split, partial);
  else lora_tn_partial_kernel<64, PT><<<grid, kTnCols, 0, st>>>(P, q, m, w, r, rows_per_split, partial);
  count_launch();
  if (int rc = check_launch("lora_tn_partial_kernel")) return rc;
  const int64_t total = w * r;
  lora_tn_finalize_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, st>>>(partial, splits, w, r, scale, transpose, out);
  count_launch();
  return check_launch("lora_tn_finalize_kernel");
}

__global__ void lora_transpose_kernel(const __half* __restrict__ a, int r, int64_t k, __half* __restrict__ at) {
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= k * r) return;
  const int64_t kk = idx / r, j = idx % r;
  at[idx] = a[j * k + kk];
}

}  // namespace sb

extern "C" {

size_t sb_nf4_linear_workspace_bytes(int64_t m, int64_t n_out, int64_t k_in, int dx) {
  if (m <= 0 || n_out <= 0 || k_in <= 0) return 0;
  if (sb::gemm::nf4_tc_shape_ok(m, n_out, k_in, dx != 0)) return 0;
  return static_cast<size_t>(n_out) * k_in * 2;
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

int sb_lora_down(const uint16_t* x, int64_t m, int64_t k, const uint16_t* a, int r, float scale,
                 uint16_t* z, uint16_t* zs, void* stream) {
  SB_REQUIRE(m >= 0 && k > 0 && r > 0 && r <= 64, "expected m >= 0, k > 0, 0 < r <= 64");
  if (m == 0) return SB_OK;
  SB_REQUIRE(x && a && (z || zs), "NULL pointer argument");
  return sb::rowdot(x, m, k, a, k, 1, r, scale, z, zs, nullptr, sb::as_stream(stream));
}

int sb_lora_up_grad(const uint16_t* dy, int64_t m, int64_t n, const uint16_t* b, int r,
                    float scale, uint16_t* u, float* u32, void* stream) {
  SB_REQUIRE(m >= 0 && n > 0 && r > 0 && r <= 64, "expected m >= 0, n > 0, 0 < r <= 64");
  if (m == 0) return SB_OK;
  SB_REQUIRE(dy && b && (u || u32), "NULL pointer argument");
  // u = fp16(scale * dY . B): B is [n, r], so rank vector j has element stride r.
  return sb::rowdot(dy, m, n, b, 1, r, r, scale, nullptr, u, u32, sb::as_stream(stream));
}

size_t sb_lora_grad_workspace_bytes(int64_t m, int64_t width, int r) {
  if (m <= 0 || width <= 0 || r <= 0) return 0;
  return static_cast<size_t>(sb::tn_splits(m, width)) * r * width * sizeof(float);
}

int sb_lora_grad_a(const float* u32, const uint16_t* x, int64_t m, int64_t k, int r, float* da,
                   void* workspace, size_t workspace_bytes, void* stream) {
  SB_REQUIRE(m >= 0 && k > 0 && r > 0 && r <= 64, "expected m >= 0, k > 0, 0 < r <= 64");
  SB_REQUIRE(da != nullptr, "NULL da");
  cudaStream_t st = sb::as_stream(stream);
  if (m == 0) {
    cudaError_t e = cudaMemsetAsync(da, 0, static_cast<size_t>(r) * k * 4, st);
    return e == cudaSuccess ? SB_OK : sb::fail(SB_ECUDA, cudaGetErrorString(e));
  }
  SB_REQUIRE(u32 && x, "NULL pointer argument");
  return sb::lora_tn<float>(u32, x, m, k, r, 1.0f, 0, da, workspace, workspace_bytes, st);
}

int sb_lora_grad_b(const uint16_t* dy, const uint16_t* z, int64_t m, int64_t n, int r, float scale,
                   float* db, void* workspace, size_t workspace_bytes, void* stream) {
  SB_REQUIRE(m >= 0 && n > 0 && r > 0 && r <= 64, "expected m >= 0, n > 0, 0 < r <= 64");
  SB_REQUIRE(db != nullptr, "NULL db");
  cudaStream_t st = sb::as_stream(stream);
  if (m == 0) {
    cudaError_t e = cudaMemsetAsync(db, 0, static_cast<size_t>(r) * n * 4, st);
    return e == cudaSuccess ? SB_OK : sb::fail(SB_ECUDA, cudaGetErrorString(e));
  }
  SB_REQUIRE(dy && z, "NULL pointer argument");
  return sb::lora_tn<__half>(reinterpret_cast<const __half*>(z), dy, m, n, r, scale, 1, db,
                             workspace, workspace_bytes, st);
}

int sb_lora_transpose_a(const uint16_t* a, int r, int64_t k, uint16_t* at, void* stream) {
  SB_REQUIRE(r > 0 && k > 0, "expected r > 0 and k > 0");
  SB_REQUIRE(a && at, "NULL pointer argument");
  const int64_t total = k * r;
  sb::lora_transpose_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, sb::as_stream(stream)>>>(
      reinterpret_cast<const __half*>(a), r, k, reinterpret_cast<__half*>(at));
  sb::count_launch();
  return sb::check_launch("lora_transpose_kernel");
}

}  // extern "C"
