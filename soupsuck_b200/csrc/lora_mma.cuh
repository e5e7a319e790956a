// LoRA low-rank kernels on the legacy tensor-core path (mma.sync m16n8k16, fp32 accumulate).
//
// These products are skinny (rank r = 16..64) and HBM-bound: each streams one
// activation-sized matrix once, so they use register-fragment MMAs fed by wide
// coalesced loads rather than the tcgen05 pipeline.
//
//   project  out[M, R] = X[M, K] . W[R, K]^T          (Z = X.A^T, U = dY.B)
//            writes scale_rows * out as fp16 [M, rp] (row-major, the GEMM's
//            LoRA operand) and/or scale_t * out^T as fp16 [R, ldt] (for the
//            weight-gradient reductions).
//   reduce   out[R, W] = scale * Pt[R, M] . Q[M, W]    (dA = U^T.X, dB^T = Z^T.dY)
//            split over M across CTAs into fp32 partials, summed in a fixed
//            order by a second kernel (deterministic); optional transposed output.
//   prepare  fp32/fp16 lora_A [r, K] and lora_B [N, r] -> fp16 A, A^T, B, B^T.
//
// Fragment layouts follow the PTX ISA for mma.m16n8k16 (g = lane/4, t = lane%4).
// The reduction index inside one MMA may be permuted freely as long as the A
// and B fragments use the same permutation; both kernels use that to feed the
// fragments from 16-byte (project) or 4-byte (reduce) vector loads.
#pragma once

#include "common.cuh"

namespace sb {
namespace lora {

__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint4 ldg16_or_zero(const __half* p, bool ok) {
  return ok ? __ldg(reinterpret_cast<const uint4*>(p)) : make_uint4(0, 0, 0, 0);
}

// ------------------------------------------------------------------ project
// One CTA = 4 warps = one 16-row tile of X; warp w reduces the w-th quarter of K
// in 32-element chunks; the four partial tiles are summed through shared memory.
template <int R>
__global__ void __launch_bounds__(128) project_kernel(
    const __half* __restrict__ X, int64_t M, int64_t K, const __half* __restrict__ W,
    float scale_rows, __half* __restrict__ out_rows, int ld_rows, float scale_t,
    __half* __restrict__ out_t, int64_t ldt) {
  constexpr int NT = R / 8;
  __shared__ float red[4][16][R];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int64_t m0 = static_cast<int64_t>(blockIdx.x) * 16;
  const int64_t chunks = K / 32;
  const int64_t c_begin = chunks * warp / 4, c_end = chunks * (warp + 1) / 4;
  float acc[NT][4];
#pragma unroll
  for (int j = 0; j < NT; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.0f;
  const bool r0ok = m0 + g < M, r1ok = m0 + g + 8 < M;
  const __half* x0 = X + (m0 + g) * K + 8 * t;
  const __half* x1 = X + (m0 + g + 8) * K + 8 * t;
  const __half* wrow = W + static_cast<int64_t>(g) * K + 8 * t;
#pragma unroll 2
  for (int64_t c = c_begin; c < c_end; ++c) {
    const int64_t k0 = c * 32;
    const uint4 xa = ldg16_or_zero(x0 + k0, r0ok);
    const uint4 xb = ldg16_or_zero(x1 + k0, r1ok);
    const uint32_t a_lo[4] = {xa.x, xb.x, xa.y, xb.y};
    const uint32_t a_hi[4] = {xa.z, xb.z, xa.w, xb.w};
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      const uint4 w = __ldg(reinterpret_cast<const uint4*>(wrow + static_cast<int64_t>(8 * j) * K + k0));
      mma16816(acc[j], a_lo, w.x, w.y);
      mma16816(acc[j], a_hi, w.z, w.w);
    }
  }
#pragma unroll
  for (int j = 0; j < NT; ++j) {
    red[warp][g][8 * j + 2 * t] = acc[j][0];
    red[warp][g][8 * j + 2 * t + 1] = acc[j][1];
    red[warp][g + 8][8 * j + 2 * t] = acc[j][2];
    red[warp][g + 8][8 * j + 2 * t + 1] = acc[j][3];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 16 * R; i += 128) {
    const int row = i / R, col = i % R;
    const float v = red[0][row][col] + red[1][row][col] + red[2][row][col] + red[3][row][col];
    const int64_t m = m0 + row;
    if (m < M) {
      if (out_rows) out_rows[m * ld_rows + col] = __float2half_rn(v * scale_rows);
      if (out_t) out_t[static_cast<int64_t>(col) * ldt + m] = __float2half_rn(v * scale_t);
    } else if (out_t && m < ldt) {
      out_t[static_cast<int64_t>(col) * ldt + m] = __float2half_rn(0.0f);  // zero pad for the reduction
    }
  }
}

// ------------------------------------------------------------------ reduce
// Warp = 16 output columns (two interleaved n8 tiles: physical column c0 + 2n + j),
// R/16 row tiles; CTA = 8 warps = 128 columns; blockIdx.y = slice of M.
template <int R>
__global__ void __launch_bounds__(256) reduce_partial_kernel(
    const __half* __restrict__ Pt, int64_t ldp, const __half* __restrict__ Q, int64_t M,
    int64_t Wd, int64_t rows_per_split, float* __restrict__ partial) {
  constexpr int MT = R / 16;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int64_t c0 = static_cast<int64_t>(blockIdx.x) * 128 + warp * 16;
  const int64_t mb = static_cast<int64_t>(blockIdx.y) * rows_per_split;
  const int64_t me = mb + rows_per_split < ldp ? mb + rows_per_split : ldp;
  float acc[MT][2][4];
#pragma unroll
  for (int i = 0; i < MT; ++i)
#pragma unroll
    for (int j = 0; j < 2; ++j) acc[i][j][0] = acc[i][j][1] = acc[i][j][2] = acc[i][j][3] = 0.0f;
  const int64_t col = c0 + 2 * g;
  const bool col_ok = col + 1 < Wd;
  for (int64_t m = mb; m < me; m += 16) {
    uint32_t q[4];
    const int64_t rows[4] = {m + 2 * t, m + 2 * t + 1, m + 2 * t + 8, m + 2 * t + 9};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      q[i] = (col_ok && rows[i] < M) ? __ldg(reinterpret_cast<const uint32_t*>(Q + rows[i] * Wd + col)) : 0u;
    }
    uint32_t b0[2], b1[2];
    asm("prmt.b32 %0, %1, %2, 0x5410;" : "=r"(b0[0]) : "r"(q[0]), "r"(q[1]));
    asm("prmt.b32 %0, %1, %2, 0x7632;" : "=r"(b0[1]) : "r"(q[0]), "r"(q[1]));
    asm("prmt.b32 %0, %1, %2, 0x5410;" : "=r"(b1[0]) : "r"(q[2]), "r"(q[3]));
    asm("prmt.b32 %0, %1, %2, 0x7632;" : "=r"(b1[1]) : "r"(q[2]), "r"(q[3]));
#pragma unroll
    for (int i = 0; i < MT; ++i) {
      const __half* p0 = Pt + static_cast<int64_t>(16 * i + g) * ldp + m + 2 * t;
      const __half* p1 = p0 + 8 * ldp;
      const uint32_t a[4] = {__ldg(reinterpret_cast<const uint32_t*>(p0)), __ldg(reinterpret_cast<const uint32_t*>(p1)),
                             __ldg(reinterpret_cast<const uint32_t*>(p0 + 8)), __ldg(reinterpret_cast<const uint32_t*>(p1 + 8))};
#pragma unroll
      for (int j = 0; j < 2; ++j) mma16816(acc[i][j], a, b0[j], b1[j]);
    }
  }
  float* out = partial + static_cast<int64_t>(blockIdx.y) * R * Wd;
#pragma unroll
  for (int i = 0; i < MT; ++i) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int64_t ca = c0 + 4 * t + j, cb = ca + 2;
      const int64_t ra = 16 * i + g, rb = ra + 8;
      if (ca < Wd) { out[ra * Wd + ca] = acc[i][j][0]; out[rb * Wd + ca] = acc[i][j][2]; }
      if (cb < Wd) { out[ra * Wd + cb] = acc[i][j][1]; out[rb * Wd + cb] = acc[i][j][3]; }
    }
  }
}

__global__ void reduce_finalize_kernel(const float* __restrict__ partial, int splits, int64_t Wd,
                                       int r, float scale, int transpose, void* __restrict__ out,
                                       int odt) {
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= Wd * r) return;
  const int64_t j = idx / Wd, c = idx % Wd;
  float acc = 0.0f;
  for (int s = 0; s < splits; ++s) acc += partial[(static_cast<int64_t>(s) * r + j) * Wd + c];
  acc *= scale;
  st_from_f32(out, odt, transpose ? c * r + j : j * Wd + c, acc);
}

// ------------------------------------------------------------------ prepare
// a [r, K] (dtype adt) -> a16 [r, K], at16 [K, r]; b [N, r] (bdt) -> b16 [N, r], bt16 [r, N].
__global__ void prepare_kernel(const void* __restrict__ a, int adt, const void* __restrict__ b,
                               int bdt, int r, int64_t K, int64_t N, __half* __restrict__ a16,
                               __half* __restrict__ at16, __half* __restrict__ b16,
                               __half* __restrict__ bt16) {
  const int64_t na = static_cast<int64_t>(r) * K;
  const int64_t total = na + static_cast<int64_t>(r) * N;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += stride) {
    if (i < na) {
      const int64_t j = i / K, k = i % K;
      const __half v = __float2half_rn(ld_as_f32(a, adt, i));
      if (a16) a16[i] = v;
      if (at16) at16[k * r + j] = v;
    } else {
      const int64_t ib = i - na;
      const int64_t n = ib / r, j = ib % r;
      const __half v = __float2half_rn(ld_as_f32(b, bdt, ib));
      if (b16) b16[ib] = v;
      if (bt16) bt16[j * N + n] = v;
    }
  }
}

inline int reduce_splits(int64_t m, int64_t w) {
  const int64_t col_blocks = (w + 127) / 128;
  int64_t s = (2 * device_sm_count() + col_blocks - 1) / col_blocks;
  const int64_t max_s = (m + 127) / 128;
  if (s > max_s) s = max_s;
  if (s < 1) s = 1;
  if (s > 4096) s = 4096;
  return static_cast<int>(s);
}

}  // namespace lora
}  // namespace sb

extern "C" {

int sb_lora_project(const uint16_t* x, int64_t m, int64_t k, const uint16_t* w, int r,
                    float scale_rows, uint16_t* out_rows, int ld_rows, float scale_t,
                    uint16_t* out_t, int64_t ldt, void* stream) {
  SB_REQUIRE(m >= 0 && k > 0, "expected m >= 0 and k > 0");
  SB_REQUIRE(r == 16 || r == 32 || r == 64, "rank must be 16, 32 or 64 (pad smaller ranks with zeros)");
  SB_REQUIRE(k % 32 == 0, "k must be a multiple of 32");
  SB_REQUIRE(!out_rows || ld_rows >= r, "ld_rows must be >= r");
  SB_REQUIRE(!out_t || ldt >= m, "ldt must be >= m");
  if (m == 0) return SB_OK;
  SB_REQUIRE(x && w && (out_rows || out_t), "NULL pointer argument");
  SB_REQUIRE(sb::aligned(x, 16) && sb::aligned(w, 16), "x and w must be 16-byte aligned");
  cudaStream_t st = sb::as_stream(stream);
  const unsigned grid = static_cast<unsigned>((m + 15) / 16);
  const __half* X = reinterpret_cast<const __half*>(x);
  const __half* W = reinterpret_cast<const __half*>(w);
  __half* orow = reinterpret_cast<__half*>(out_rows);
  __half* ot = reinterpret_cast<__half*>(out_t);
  if (r == 16) sb::lora::project_kernel<16><<<grid, 128, 0, st>>>(X, m, k, W, scale_rows, orow, ld_rows, scale_t, ot, ldt);
  else if (r == 32) sb::lora::project_kernel<32><<<grid, 128, 0, st>>>(X, m, k, W, scale_rows, orow, ld_rows, scale_t, ot, ldt);
  else sb::lora::project_kernel<64><<<grid, 128, 0, st>>>(X, m, k, W, scale_rows, orow, ld_rows, scale_t, ot, ldt);
  sb::count_launch();
  return sb::check_launch("lora_project_kernel");
}

size_t sb_lora_reduce_workspace_bytes(int64_t m, int64_t w, int r) {
  if (m <= 0 || w <= 0 || r <= 0) return 0;
  const int64_t ldp = (m + 15) / 16 * 16;  // the zero-padded row count the reduction runs over
  return static_cast<size_t>(sb::lora::reduce_splits(ldp, w)) * r * w * sizeof(float);
}

int sb_lora_reduce(const uint16_t* pt, int64_t ldp, const uint16_t* q, int64_t m, int64_t w, int r,
                   float scale, int transpose, void* out, int out_dtype, void* workspace,
                   size_t workspace_bytes, void* stream) {
  SB_REQUIRE(m >= 0 && w > 0, "expected m >= 0 and w > 0");
  SB_REQUIRE(r == 16 || r == 32 || r == 64, "rank must be 16, 32 or 64");
  SB_REQUIRE(ldp >= m && ldp % 16 == 0, "ldp must be >= m and a multiple of 16 (zero padded)");
  SB_REQUIRE(w % 2 == 0, "w must be even");
  SB_REQUIRE(out_dtype == SB_F16 || out_dtype == SB_F32, "bad out dtype");
  SB_REQUIRE(out != nullptr, "NULL out");
  cudaStream_t st = sb::as_stream(stream);
  if (m == 0) {
    cudaError_t e = cudaMemsetAsync(out, 0, static_cast<size_t>(r) * w * (out_dtype == SB_F32 ? 4 : 2), st);
    return e == cudaSuccess ? SB_OK : sb::fail(SB_ECUDA, cudaGetErrorString(e));
  }
  SB_REQUIRE(pt && q, "NULL pointer argument");
  SB_REQUIRE(sb::aligned(pt, 4) && sb::aligned(q, 4), "pt and q must be 4-byte aligned");
  const int splits = sb::lora::reduce_splits(ldp, w);
  const size_t need = static_cast<size_t>(splits) * r * w * sizeof(float);
  if (!workspace || workspace_bytes < need) return sb::fail(SB_EWORKSPACE, "LoRA reduce workspace too small");
  int64_t rows_per_split = (ldp + splits - 1) / splits;
  rows_per_split = (rows_per_split + 15) / 16 * 16;
  dim3 grid(static_cast<unsigned>((w + 127) / 128), static_cast<unsigned>(splits));
  float* partial = static_cast<float*>(workspace);
  const __half* P = reinterpret_cast<const __half*>(pt);
  const __half* Q = reinterpret_cast<const __half*>(q);
  if (r == 16) sb::lora::reduce_partial_kernel<16><<<grid, 256, 0, st>>>(P, ldp, Q, m, w, rows_per_split, partial);
  else if (r == 32) sb::lora::reduce_partial_kernel<32><<<grid, 256, 0, st>>>(P, ldp, Q, m, w, rows_per_split, partial);
  else sb::lora::reduce_partial_kernel<64><<<grid, 256, 0, st>>>(P, ldp, Q, m, w, rows_per_split, partial);
  sb::count_launch();
  if (int rc = sb::check_launch("lora_reduce_partial_kernel")) return rc;
  const int64_t total = w * r;
  sb::lora::reduce_finalize_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, st>>>(
      partial, splits, w, r, scale, transpose, out, out_dtype);
  sb::count_launch();
  return sb::check_launch("lora_reduce_finalize_kernel");
}

int sb_lora_prepare(const void* a, int a_dtype, const void* b, int b_dtype, int r, int64_t k,
                    int64_t n, uint16_t* a16, uint16_t* at16, uint16_t* b16, uint16_t* bt16,
                    void* stream) {
  SB_REQUIRE(r > 0 && k > 0 && n > 0, "expected positive sizes");
  SB_REQUIRE((a_dtype == SB_F16 || a_dtype == SB_F32) && (b_dtype == SB_F16 || b_dtype == SB_F32), "bad dtype");
  SB_REQUIRE(a && b, "NULL pointer argument");
  const int64_t total = static_cast<int64_t>(r) * (k + n);
  const int64_t blocks = (total + 255) / 256;
  const int grid = static_cast<int>(blocks < 4096 ? blocks : 4096);
  sb::lora::prepare_kernel<<<grid, 256, 0, sb::as_stream(stream)>>>(
      a, a_dtype, b, b_dtype, r, k, n, reinterpret_cast<__half*>(a16), reinterpret_cast<__half*>(at16),
      reinterpret_cast<__half*>(b16), reinterpret_cast<__half*>(bt16));
  sb::count_launch();
  return sb::check_launch("lora_prepare_kernel");
}

}  // extern "C"
