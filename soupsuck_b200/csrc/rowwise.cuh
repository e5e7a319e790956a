// Elementwise and row kernels: LoRA scale/add epilogue, residual add + RMSNorm,
// standalone RMSNorm and its two-stage weight gradient.
//
// All arithmetic keeps the reference's cast order (values are rounded to the
// storage dtype exactly where the Triton source casts) and never contracts a
// multiply into an add (__fmul_rn / __fadd_rn), as enable_fp_fusion=False does
// in the reference launches.  Row statistics are fp32 block reductions.
//
// Roofline: HBM-bound; per row of H features the forward add-RMSNorm moves
// H*(|r| + |d| + |s| + |y|) + 4 bytes (12,292 B at H = 1536, fp16 I/O).
#pragma once

#include "common.cuh"

namespace sb {

// ------------------------------------------------------------- LoRA epilogue
// lora_scale_add_kernel (solution/kernels/lora_epilogue.py:24-34).
__global__ void lora_scale_add_kernel(const void* __restrict__ base, int bdt,
                                      const void* __restrict__ adapter, int adt,
                                      void* __restrict__ out, int odt, int64_t count,
                                      float scale, int cast_to_base) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count;
       i += stride) {
    const float b = ld_as_f32(base, bdt, i);
    float scaled = round_to(__fmul_rn(ld_as_f32(adapter, adt, i), scale), adt);
    if (cast_to_base) scaled = round_to(scaled, bdt);
    st_from_f32(out, odt, i, __fadd_rn(b, scaled));
  }
}

// lora_scale_gradient_kernel (solution/kernels/lora_epilogue.py:37-43).
__global__ void lora_scale_grad_kernel(const void* __restrict__ grad, int gdt,
                                       void* __restrict__ dadapter, int adt, int64_t count,
                                       float scale) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count;
       i += stride) {
    const float g = round_to(ld_as_f32(grad, gdt, i), adt);
    st_from_f32(dadapter, adt, i, __fmul_rn(g, scale));
  }
}

// --------------------------------------------------------------- reductions
template <int THREADS>
__device__ __forceinline__ float block_sum(float v, float* scratch) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();  // scratch may still be read by a previous reduction
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  float total = 0.0f;
#pragma unroll
  for (int w = 0; w < THREADS / 32; ++w) total += scratch[w];
  return total;
}

constexpr int kRowThreads = 256;

// ------------------------------------------------------------ add + RMSNorm
// add_rmsnorm_forward_kernel (solution/kernels/add_rmsnorm.py:37-51).
__global__ void __launch_bounds__(kRowThreads) add_rmsnorm_fwd_kernel(
    const void* __restrict__ R, int rdt, const void* __restrict__ D, int ddt,
    const void* __restrict__ W, int wdt, int64_t w_stride, void* __restrict__ S,
    void* __restrict__ Y, int ydt, float* __restrict__ rstd_out, int64_t h, float eps) {
  extern __shared__ float srow[];
  __shared__ float scratch[kRowThreads / 32];
  const int sdt = promote(rdt, ddt);
  const int64_t row = blockIdx.x;
  const int64_t base = row * h;
  float acc = 0.0f;
  for (int64_t c = threadIdx.x; c < h; c += kRowThreads) {
    const float s = round_to(__fadd_rn(ld_as_f32(R, rdt, base + c), ld_as_f32(D, ddt, base + c)), sdt);
    srow[c] = s;
    st_from_f32(S, sdt, base + c, s);
    acc = __fadd_rn(acc, __fmul_rn(s, s));
  }
  const float total = block_sum<kRowThreads>(acc, scratch);
  const float r = rsqrtf(__fadd_rn(__fdiv_rn(total, static_cast<float>(h)), eps));
  for (int64_t c = threadIdx.x; c < h; c += kRowThreads) {
    const float q = round_to(__fmul_rn(srow[c], r), sdt);
    st_from_f32(Y, ydt, base + c, __fmul_rn(q, ld_as_f32(W, wdt, c * w_stride)));
  }
  if (threadIdx.x == 0) rstd_out[row] = r;
}

// ------------------------------------------- fp16 fast path of add + RMSNorm
// The training configuration (fp16 residual, delta, gamma, s and y; contiguous
// rows; H % 8 == 0) reads and writes every row as 16-byte vectors and keeps the
// row in registers: thread t of the row's CTA owns the 8-element pieces t,
// t + T, ... (V of them).  The cast order is the reference's, as above; only the
// order of the fp32 sum of squares differs (per-thread pieces, then the block).
__device__ __forceinline__ void h8_to_f32(const uint4& v, float (&f)[8]) {
  const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __half22float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}
__device__ __forceinline__ uint4 f32_to_h8(const float (&f)[8]) {
  uint4 v;
  __half2* h = reinterpret_cast<__half2*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
  return v;
}
__device__ __forceinline__ float f16_round(float v) { return __half2float(__float2half_rn(v)); }

template <int T>
__device__ __forceinline__ float block_sum_t(float v, float* scratch) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  float total = 0.0f;
#pragma unroll
  for (int w = 0; w < T / 32; ++w) total += scratch[w];
  return total;
}

template <int T, int V>
__global__ void __launch_bounds__(T) add_rmsnorm_fwd_h8_kernel(const uint4* __restrict__ R,
                                                               const uint4* __restrict__ D,
                                                               const uint4* __restrict__ W, uint4* __restrict__ S,
                                                               uint4* __restrict__ Y, float* __restrict__ rstd_out,
                                                               int64_t h, float eps) {
  __shared__ float scratch[T / 32];
  const int64_t h8 = h / 8;
  const int64_t base = static_cast<int64_t>(blockIdx.x) * h8;
  float s[V][8];
  float acc = 0.0f;
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const int64_t c = threadIdx.x + static_cast<int64_t>(i) * T;
    if (c < h8) {
      float r8[8], d8[8];
      h8_to_f32(__ldcs(R + base + c), r8);
      h8_to_f32(__ldcs(D + base + c), d8);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        s[i][e] = f16_round(__fadd_rn(r8[e], d8[e]));
        acc = __fadd_rn(acc, __fmul_rn(s[i][e], s[i][e]));
      }
      S[base + c] = f32_to_h8(s[i]);
    }
  }
  const float total = block_sum_t<T>(acc, scratch);
  const float r = rsqrtf(__fadd_rn(__fdiv_rn(total, static_cast<float>(h)), eps));
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const int64_t c = threadIdx.x + static_cast<int64_t>(i) * T;
    if (c < h8) {
      float w8[8], y8[8];
      h8_to_f32(__ldg(W + c), w8);
#pragma unroll
      for (int e = 0; e < 8; ++e) y8[e] = __fmul_rn(f16_round(__fmul_rn(s[i][e], r)), w8[e]);
      Y[base + c] = f32_to_h8(y8);
    }
  }
  if (threadIdx.x == 0) rstd_out[blockIdx.x] = r;
}

template <int T, int V>
__global__ void __launch_bounds__(T) add_rmsnorm_bwd_h8_kernel(const uint4* __restrict__ Sv,
                                                               const uint4* __restrict__ W,
                                                               const float* __restrict__ rstd,
                                                               const uint4* __restrict__ Gs, int64_t gs_row8,
                                                               const uint4* __restrict__ Gy, int64_t gy_row8,
                                                               uint4* __restrict__ Dr, uint4* __restrict__ Dd,
                                                               int64_t h) {
  __shared__ float scratch[T / 32];
  const int64_t h8 = h / 8;
  const int64_t row = blockIdx.x;
  const int64_t base = row * h8;
  float u[V][8], a[V][8];
  float proj = 0.0f, r = 0.0f;
  if (Gy != nullptr) {
    r = rstd[row];
    float acc = 0.0f;
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const int64_t c = threadIdx.x + static_cast<int64_t>(i) * T;
      if (c < h8) {
        float s8[8], g8[8], w8[8];
        h8_to_f32(__ldcs(Sv + base + c), s8);
        h8_to_f32(__ldcs(Gy + row * gy_row8 + c), g8);
        h8_to_f32(__ldg(W + c), w8);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          a[i][e] = __fmul_rn(s8[e], r);
          u[i][e] = f16_round(__fmul_rn(g8[e], w8[e]));
          acc = __fadd_rn(acc, __fmul_rn(u[i][e], a[i][e]));
        }
      }
    }
    proj = __fdiv_rn(block_sum_t<T>(acc, scratch), static_cast<float>(h));
  }
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const int64_t c = threadIdx.x + static_cast<int64_t>(i) * T;
    if (c < h8) {
      float gs8[8], ds[8];
      if (Gs != nullptr) h8_to_f32(__ldcs(Gs + row * gs_row8 + c), gs8);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        float d = 0.0f;
        if (Gy != nullptr) d = f16_round(__fmul_rn(r, __fsub_rn(u[i][e], __fmul_rn(a[i][e], proj))));
        if (Gs != nullptr) d = __fadd_rn(d, gs8[e]);
        ds[e] = f16_round(d);
      }
      const uint4 o = f32_to_h8(ds);
      if (Dr != nullptr) Dr[base + c] = o;
      if (Dd != nullptr) Dd[base + c] = o;
    }
  }
}

// 16-byte pieces per thread of the fast path (256 threads per row), 0 if H does
// not qualify (H % 8 != 0 or H > 8192).
constexpr int kH8Threads = 256;
inline int h8_pieces(int64_t h) {
  if (h % 8 != 0) return 0;
  const int64_t h8 = h / 8;
  for (int v : {1, 2, 4}) {
    if (h8 <= static_cast<int64_t>(v) * kH8Threads) return v;
  }
  return 0;
}

// add_rmsnorm_backward_kernel (solution/kernels/add_rmsnorm.py:54-81).
__global__ void __launch_bounds__(kRowThreads) add_rmsnorm_bwd_kernel(
    const void* __restrict__ S, int sdt, const void* __restrict__ W, int wdt, int64_t w_stride,
    const float* __restrict__ rstd, const void* __restrict__ Gs, int gsdt, int64_t gs_row,
    int64_t gs_col, const void* __restrict__ Gy, int gydt, int64_t gy_row, int64_t gy_col,
    void* __restrict__ Dr, int drdt, void* __restrict__ Dd, int dddt, int64_t h) {
  extern __shared__ float smem[];
  float* su = smem;
  float* sa = smem + h;
  __shared__ float scratch[kRowThreads / 32];
  const int64_t row = blockIdx.x;
  const int64_t base = row * h;
  float proj = 0.0f, r = 0.0f;
  if (Gy != nullptr) {
    r = rstd[row];
    float acc = 0.0f;
    for (int64_t c = threadIdx.x; c < h; c += kRowThreads) {
      const float a = __fmul_rn(ld_as_f32(S, sdt, base + c), r);
      const float g = ld_as_f32(Gy, gydt, row * gy_row + c * gy_col);
      const float u = round_to(__fmul_rn(g, ld_as_f32(W, wdt, c * w_stride)), sdt);
      su[c] = u;
      sa[c] = a;
      acc = __fadd_rn(acc, __fmul_rn(u, a));
    }
    proj = __fdiv_rn(block_sum<kRowThreads>(acc, scratch), static_cast<float>(h));
  }
  for (int64_t c = threadIdx.x; c < h; c += kRowThreads) {
    float ds = 0.0f;
    if (Gy != nullptr) {
      ds = round_to(__fmul_rn(r, __fsub_rn(su[c], __fmul_rn(sa[c], proj))), sdt);
    }
    if (Gs != nullptr) ds = __fadd_rn(ds, ld_as_f32(Gs, gsdt, row * gs_row + c * gs_col));
    ds = round_to(ds, sdt);
    if (Dr != nullptr) st_from_f32(Dr, drdt, base + c, ds);
    if (Dd != nullptr) st_from_f32(Dd, dddt, base + c, ds);
  }
}

// ------------------------------------------------------------ RMSNorm alone
// rmsnorm_forward_kernel (solution/kernels/rmsnorm.py:42-52).
__global__ void __launch_bounds__(kRowThreads) rmsnorm_fwd_kernel(
    const void* __restrict__ X, int xdt, int64_t x_row, const void* __restrict__ W, int wdt,
    int64_t w_stride, void* __restrict__ Y, int ydt, float* __restrict__ rstd_out, int64_t h,
    float eps) {
  __shared__ float scratch[kRowThreads / 32];
  const int64_t row = blockIdx.x;
  float acc = 0.0f;
  for (int64_t c = threadIdx.x; c < h; c += kRowThreads) {
    const float x = ld_as_f32(X, xdt, row * x_row + c);
    acc = __fadd_rn(acc, __fmul_rn(x, x));
  }
  const float r = rsqrtf(__fadd_rn(__fdiv_rn(block_sum<kRowThreads>(acc, scratch), static_cast<float>(h)), eps));
  for (int64_t c = threadIdx.x; c < h; c += kRowThreads) {
    const float q = round_to(__fmul_rn(ld_as_f32(X, xdt, row * x_row + c), r), xdt);
    st_from_f32(Y, ydt, row * h + c, __fmul_rn(q, ld_as_f32(W, wdt, c * w_stride)));
  }
  if (threadIdx.x == 0) rstd_out[row] = r;
}

// rmsnorm_input_gradient_kernel (solution/kernels/rmsnorm.py:55-70).
__global__ void __launch_bounds__(kRowThreads) rmsnorm_input_grad_kernel(
    const void* __restrict__ X, int xdt, int64_t x_row, const void* __restrict__ W, int wdt,
    int64_t w_stride, const void* __restrict__ G, int gdt, int64_t g_row, int64_t g_col,
    const float* __restrict__ rstd, void* __restrict__ Dx, int64_t h) {
  extern __shared__ float smem[];
  float* su = smem;
  float* sa = smem + h;
  __shared__ float scratch[kRowThreads / 32];
  const int64_t row = blockIdx.x;
  const float r = rstd[row];
  float acc = 0.0f;
  for (int64_t c = threadIdx.x; c < h; c += kRowThreads) {
    const float a = __fmul_rn(ld_as_f32(X, xdt, row * x_row + c), r);
    const float g = ld_as_f32(G, gdt, row * g_row + c * g_col);
    const float u = round_to(__fmul_rn(g, ld_as_f32(W, wdt, c * w_stride)), xdt);
    su[c] = u;
    sa[c] = a;
    acc = __fadd_rn(acc, __fmul_rn(u, a));
  }
  const float proj = __fdiv_rn(block_sum<kRowThreads>(acc, scratch), static_cast<float>(h));
  for (int64_t c = threadIdx.x; c < h; c += kRowThreads) {
    st_from_f32(Dx, xdt, row * h + c, __fmul_rn(r, __fsub_rn(su[c], __fmul_rn(sa[c], proj))));
  }
}

// rmsnorm_weight_partials_kernel / _finalize_kernel (solution/kernels/rmsnorm.py:73-102):
// 32-row x 128-feature partial sums, then a per-feature sum over the partials.
constexpr int kDgRows = 32, kDgCols = 128;

__global__ void __launch_bounds__(kDgCols) rmsnorm_dgamma_partial_kernel(
    const void* __restrict__ X, int xdt, int64_t x_row, const void* __restrict__ G, int gdt,
    int64_t g_row, int64_t g_col, const float* __restrict__ rstd, float* __restrict__ partial,
    int64_t rows, int64_t h, int exact_half) {
  const int64_t group = blockIdx.x;
  const int64_t c = static_cast<int64_t>(blockIdx.y) * kDgCols + threadIdx.x;
  if (c >= h) return;
  float acc = 0.0f;
  for (int i = 0; i < kDgRows; ++i) {
    const int64_t row = group * kDgRows + i;
    if (row >= rows) break;
    const float q = round_to(__fmul_rn(ld_as_f32(X, xdt, row * x_row + c), rstd[row]), xdt);
    float p = __fmul_rn(ld_as_f32(G, gdt, row * g_row + c * g_col), q);
    if (exact_half) p = round_to(p, SB_F16);
    acc = __fadd_rn(acc, p);
  }
  partial[group * h + c] = acc;
}

__global__ void rmsnorm_dgamma_finalize_kernel(const float* __restrict__ partial, int64_t groups,
                                               void* __restrict__ dw, int dwdt, int64_t h) {
  const int64_t c = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (c >= h) return;
  float acc = 0.0f;
  for (int64_t g = 0; g < groups; ++g) acc = __fadd_rn(acc, partial[g * h + c]);
  st_from_f32(dw, dwdt, c, acc);
}

inline int elementwise_grid(int64_t count) {
  const int64_t blocks = (count + 255) / 256;
  const int64_t cap = static_cast<int64_t>(device_sm_count()) * 8;
  return static_cast<int>(blocks < cap ? blocks : cap);
}

inline bool dtype_ok(int dt) { return dt == SB_F16 || dt == SB_F32; }

constexpr int64_t kMaxRowSmemFloats = 48 * 1024 / 4 / 2;  // two fp32 rows in 48 KB

}  // namespace sb

extern "C" {

int sb_lora_scale_add(const void* base, int base_dtype, const void* adapter, int adapter_dtype,
                      void* out, int out_dtype, int64_t count, float scale, int cast_to_base,
                      void* stream) {
  SB_REQUIRE(count >= 0, "count must be non-negative");
  SB_REQUIRE(sb::dtype_ok(base_dtype) && sb::dtype_ok(adapter_dtype) && sb::dtype_ok(out_dtype),
             "dtype must be SB_F16 or SB_F32");
  if (count == 0) return SB_OK;
  SB_REQUIRE(base && adapter && out, "NULL pointer argument");
  sb::lora_scale_add_kernel<<<sb::elementwise_grid(count), 256, 0, sb::as_stream(stream)>>>(
      base, base_dtype, adapter, adapter_dtype, out, out_dtype, count, scale, cast_to_base);
  sb::count_launch();
  return sb::check_launch("lora_scale_add_kernel");
}

int sb_lora_scale_grad(const void* grad, int grad_dtype, void* dadapter, int adapter_dtype,
                       int64_t count, float scale, void* stream) {
  SB_REQUIRE(count >= 0, "count must be non-negative");
  SB_REQUIRE(sb::dtype_ok(grad_dtype) && sb::dtype_ok(adapter_dtype), "dtype must be SB_F16 or SB_F32");
  if (count == 0) return SB_OK;
  SB_REQUIRE(grad && dadapter, "NULL pointer argument");
  sb::lora_scale_grad_kernel<<<sb::elementwise_grid(count), 256, 0, sb::as_stream(stream)>>>(
      grad, grad_dtype, dadapter, adapter_dtype, count, scale);
  sb::count_launch();
  return sb::check_launch("lora_scale_grad_kernel");
}

int sb_add_rmsnorm_fwd(const void* residual, int r_dtype, const void* delta, int d_dtype,
                       const void* weight, int w_dtype, int64_t w_stride, void* s, void* y,
                       int y_dtype, float* rstd, int64_t rows, int64_t h, float eps,
                       void* stream) {
  SB_REQUIRE(rows >= 0 && h > 0, "expected rows >= 0 and h > 0");
  SB_REQUIRE(h <= sb::kMaxRowSmemFloats * 2, "h too large for the row kernel");
  SB_REQUIRE(sb::dtype_ok(r_dtype) && sb::dtype_ok(d_dtype) && sb::dtype_ok(w_dtype) &&
                 sb::dtype_ok(y_dtype),
             "dtype must be SB_F16 or SB_F32");
  if (rows == 0) return SB_OK;
  SB_REQUIRE(residual && delta && weight && s && y && rstd, "NULL pointer argument");
  SB_REQUIRE(rows <= 0x7fffffff, "too many rows");
  const int pieces = sb::h8_pieces(h);
  if (pieces && r_dtype == SB_F16 && d_dtype == SB_F16 && w_dtype == SB_F16 && y_dtype == SB_F16 &&
      w_stride == 1 && sb::aligned(residual, 16) && sb::aligned(delta, 16) && sb::aligned(weight, 16) &&
      sb::aligned(s, 16) && sb::aligned(y, 16)) {
    const uint4* R = static_cast<const uint4*>(residual);
    const uint4* D = static_cast<const uint4*>(delta);
    const uint4* W = static_cast<const uint4*>(weight);
    uint4* S = static_cast<uint4*>(s);
    uint4* Y = static_cast<uint4*>(y);
    constexpr int T = sb::kH8Threads;
    const unsigned grid = static_cast<unsigned>(rows);
    cudaStream_t st = sb::as_stream(stream);
    if (pieces == 1) sb::add_rmsnorm_fwd_h8_kernel<T, 1><<<grid, T, 0, st>>>(R, D, W, S, Y, rstd, h, eps);
    else if (pieces == 2) sb::add_rmsnorm_fwd_h8_kernel<T, 2><<<grid, T, 0, st>>>(R, D, W, S, Y, rstd, h, eps);
    else sb::add_rmsnorm_fwd_h8_kernel<T, 4><<<grid, T, 0, st>>>(R, D, W, S, Y, rstd, h, eps);
    sb::count_launch();
    return sb::check_launch("add_rmsnorm_fwd_h8_kernel");
  }
  sb::add_rmsnorm_fwd_kernel<<<static_cast<unsigned>(rows), sb::kRowThreads, h * sizeof(float),
                               sb::as_stream(stream)>>>(residual, r_dtype, delta, d_dtype, weight,
                                                        w_dtype, w_stride, s, y, y_dtype, rstd,
                                                        h, eps);
  sb::count_launch();
  return sb::check_launch("add_rmsnorm_fwd_kernel");
}

int sb_add_rmsnorm_bwd(const void* s, int s_dtype, const void* weight, int w_dtype,
                       int64_t w_stride, const float* rstd, const void* gs, int gs_dtype,
                       int64_t gs_row, int64_t gs_col, const void* gy, int gy_dtype,
                       int64_t gy_row, int64_t gy_col, void* dr, int dr_dtype, void* dd,
                       int dd_dtype, int64_t rows, int64_t h, void* stream) {
  SB_REQUIRE(rows >= 0 && h > 0, "expected rows >= 0 and h > 0");
  SB_REQUIRE(h <= sb::kMaxRowSmemFloats, "h too large for the row kernel");
  SB_REQUIRE(sb::dtype_ok(s_dtype) && sb::dtype_ok(w_dtype), "dtype must be SB_F16 or SB_F32");
  SB_REQUIRE(!gs || sb::dtype_ok(gs_dtype), "bad gs dtype");
  SB_REQUIRE(!gy || sb::dtype_ok(gy_dtype), "bad gy dtype");
  SB_REQUIRE(!dr || sb::dtype_ok(dr_dtype), "bad dr dtype");
  SB_REQUIRE(!dd || sb::dtype_ok(dd_dtype), "bad dd dtype");
  if (rows == 0 || (!dr && !dd)) return SB_OK;
  SB_REQUIRE(s && weight && (rstd || !gy), "NULL pointer argument");
  SB_REQUIRE(rows <= 0x7fffffff, "too many rows");
  const int pieces = sb::h8_pieces(h);
  const bool gs_ok = !gs || (gs_dtype == SB_F16 && gs_col == 1 && gs_row % 8 == 0 && sb::aligned(gs, 16));
  const bool gy_ok = !gy || (gy_dtype == SB_F16 && gy_col == 1 && gy_row % 8 == 0 && sb::aligned(gy, 16));
  const bool out_ok = (!dr || (dr_dtype == SB_F16 && sb::aligned(dr, 16))) &&
                      (!dd || (dd_dtype == SB_F16 && sb::aligned(dd, 16)));
  if (pieces && s_dtype == SB_F16 && w_dtype == SB_F16 && w_stride == 1 && sb::aligned(s, 16) &&
      sb::aligned(weight, 16) && gs_ok && gy_ok && out_ok) {
    const uint4* S = static_cast<const uint4*>(s);
    const uint4* W = static_cast<const uint4*>(weight);
    const uint4* GS = static_cast<const uint4*>(gs);
    const uint4* GY = static_cast<const uint4*>(gy);
    uint4* DR = static_cast<uint4*>(dr);
    uint4* DD = static_cast<uint4*>(dd);
    constexpr int T = sb::kH8Threads;
    const unsigned grid = static_cast<unsigned>(rows);
    cudaStream_t st = sb::as_stream(stream);
    const int64_t gs8 = gs_row / 8, gy8 = gy_row / 8;
    if (pieces == 1) sb::add_rmsnorm_bwd_h8_kernel<T, 1><<<grid, T, 0, st>>>(S, W, rstd, GS, gs8, GY, gy8, DR, DD, h);
    else if (pieces == 2) sb::add_rmsnorm_bwd_h8_kernel<T, 2><<<grid, T, 0, st>>>(S, W, rstd, GS, gs8, GY, gy8, DR, DD, h);
    else sb::add_rmsnorm_bwd_h8_kernel<T, 4><<<grid, T, 0, st>>>(S, W, rstd, GS, gs8, GY, gy8, DR, DD, h);
    sb::count_launch();
    return sb::check_launch("add_rmsnorm_bwd_h8_kernel");
  }
  sb::add_rmsnorm_bwd_kernel<<<static_cast<unsigned>(rows), sb::kRowThreads,
                               2 * h * sizeof(float), sb::as_stream(stream)>>>(
      s, s_dtype, weight, w_dtype, w_stride, rstd, gs, gs_dtype, gs_row, gs_col, gy, gy_dtype,
      gy_row, gy_col, dr, dr_dtype, dd, dd_dtype, h);
  sb::count_launch();
  return sb::check_launch("add_rmsnorm_bwd_kernel");
}

int sb_rmsnorm_fwd(const void* x, int x_dtype, int64_t x_row, const void* weight, int w_dtype,
                   int64_t w_stride, void* y, int y_dtype, float* rstd, int64_t rows,
                   int64_t h, float eps, void* stream) {
  SB_REQUIRE(rows >= 0 && h > 0, "expected rows >= 0 and h > 0");
  SB_REQUIRE(sb::dtype_ok(x_dtype) && sb::dtype_ok(w_dtype) && sb::dtype_ok(y_dtype),
             "dtype must be SB_F16 or SB_F32");
  if (rows == 0) return SB_OK;
  SB_REQUIRE(x && weight && y && rstd, "NULL pointer argument");
  SB_REQUIRE(rows <= 0x7fffffff, "too many rows");
  sb::rmsnorm_fwd_kernel<<<static_cast<unsigned>(rows), sb::kRowThreads, 0, sb::as_stream(stream)>>>(
      x, x_dtype, x_row, weight, w_dtype, w_stride, y, y_dtype, rstd, h, eps);
  sb::count_launch();
  return sb::check_launch("rmsnorm_fwd_kernel");
}

int sb_rmsnorm_input_grad(const void* x, int x_dtype, int64_t x_row, const void* weight,
                          int w_dtype, int64_t w_stride, const void* g, int g_dtype,
                          int64_t g_row, int64_t g_col, const float* rstd, void* dx,
                          int64_t rows, int64_t h, void* stream) {
  SB_REQUIRE(rows >= 0 && h > 0, "expected rows >= 0 and h > 0");
  SB_REQUIRE(h <= sb::kMaxRowSmemFloats, "h too large for the row kernel");
  SB_REQUIRE(sb::dtype_ok(x_dtype) && sb::dtype_ok(w_dtype) && sb::dtype_ok(g_dtype),
             "dtype must be SB_F16 or SB_F32");
  if (rows == 0) return SB_OK;
  SB_REQUIRE(x && weight && g && rstd && dx, "NULL pointer argument");
  SB_REQUIRE(rows <= 0x7fffffff, "too many rows");
  sb::rmsnorm_input_grad_kernel<<<static_cast<unsigned>(rows), sb::kRowThreads,
                                  2 * h * sizeof(float), sb::as_stream(stream)>>>(
      x, x_dtype, x_row, weight, w_dtype, w_stride, g, g_dtype, g_row, g_col, rstd, dx, h);
  sb::count_launch();
  return sb::check_launch("rmsnorm_input_grad_kernel");
}

size_t sb_rmsnorm_weight_grad_workspace_bytes(int64_t rows, int64_t h) {
  if (rows <= 0 || h <= 0) return 0;
  return static_cast<size_t>((rows + sb::kDgRows - 1) / sb::kDgRows) * h * sizeof(float);
}

int sb_rmsnorm_weight_grad(const void* x, int x_dtype, int64_t x_row, const void* g,
                           int g_dtype, int64_t g_row, int64_t g_col, const float* rstd,
                           void* dw, int dw_dtype, int64_t rows, int64_t h, int exact_half,
                           void* workspace, size_t workspace_bytes, void* stream) {
  SB_REQUIRE(rows >= 0 && h > 0, "expected rows >= 0 and h > 0");
  SB_REQUIRE(sb::dtype_ok(x_dtype) && sb::dtype_ok(g_dtype) && sb::dtype_ok(dw_dtype),
             "dtype must be SB_F16 or SB_F32");
  SB_REQUIRE(dw != nullptr, "NULL dw");
  cudaStream_t st = sb::as_stream(stream);
  if (rows == 0) {
    cudaError_t e = cudaMemsetAsync(dw, 0, h * (dw_dtype == SB_F32 ? 4 : 2), st);
    return e == cudaSuccess ? SB_OK : sb::fail(SB_ECUDA, cudaGetErrorString(e));
  }
  SB_REQUIRE(x && g && rstd, "NULL pointer argument");
  const size_t need = sb_rmsnorm_weight_grad_workspace_bytes(rows, h);
  if (workspace_bytes < need || !workspace) return sb::fail(SB_EWORKSPACE, "workspace too small");
  const int64_t groups = (rows + sb::kDgRows - 1) / sb::kDgRows;
  SB_REQUIRE(groups <= 0x7fffffff, "too many rows");
  dim3 grid(static_cast<unsigned>(groups), static_cast<unsigned>((h + sb::kDgCols - 1) / sb::kDgCols));
  sb::rmsnorm_dgamma_partial_kernel<<<grid, sb::kDgCols, 0, st>>>(
      x, x_dtype, x_row, g, g_dtype, g_row, g_col, rstd, static_cast<float*>(workspace), rows, h,
      exact_half);
  sb::count_launch();
  if (int rc = sb::check_launch("rmsnorm_dgamma_partial_kernel")) return rc;
  sb::rmsnorm_dgamma_finalize_kernel<<<static_cast<unsigned>((h + 127) / 128), 128, 0, st>>>(
      static_cast<const float*>(workspace), groups, dw, dw_dtype, h);
  sb::count_launch();
  return sb::check_launch("rmsnorm_dgamma_finalize_kernel");
}

}  // extern "C"
