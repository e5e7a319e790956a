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

#include <algorithm>
#include <mutex>

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

// Finalize with the splits spread over a CTA: 256 threads = 16 split groups x 16
// float4 columns, so a CTA covers 64 consecutive values of one partial row
// [r * Wd] and group q sums splits q, q + 16, ...; the 16 group sums are then
// added in group order.  The order is fixed, so results are deterministic, and
// every split's 64-value row segment is read by 16 threads at once (the
// one-thread-per-output kernel above serialises up to a few hundred loads).
// Requires Wd % 4 == 0 (float4 rows).
__global__ void __launch_bounds__(256) reduce_finalize2_kernel(const float* __restrict__ partial, int splits,
                                                               int64_t Wd, int r, float scale, int transpose,
                                                               void* __restrict__ out, int odt) {
  __shared__ float4 part[16][17];
  const int col4 = threadIdx.x & 15, grp = threadIdx.x >> 4;
  const int64_t total4 = Wd * r / 4;
  const int64_t e4 = static_cast<int64_t>(blockIdx.x) * 16 + col4;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  if (e4 < total4) {
    const float4* src = reinterpret_cast<const float4*>(partial) + e4;
    const int64_t split4 = total4;
#pragma unroll 4
    for (int s = grp; s < splits; s += 16) {
      const float4 v = __ldcg(src + static_cast<int64_t>(s) * split4);
      acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
    }
  }
  part[grp][col4] = acc;
  __syncthreads();
  if (grp == 0 && e4 < total4) {
    float4 t = part[0][col4];
#pragma unroll
    for (int q = 1; q < 16; ++q) {
      const float4 v = part[q][col4];
      t.x += v.x; t.y += v.y; t.z += v.z; t.w += v.w;
    }
    const float vals[4] = {t.x * scale, t.y * scale, t.z * scale, t.w * scale};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t e = e4 * 4 + i;
      const int64_t j = e / Wd, c = e % Wd;
      st_from_f32(out, odt, transpose ? c * r + j : j * Wd + c, vals[i]);
    }
  }
}

// ------------------------------------------------------------------ streamed variants
// The two kernels above keep few bytes in flight (4-byte loads in the reduction,
// one 16-row tile of 4 warps in the projection).  The streamed variants below
// are what the C entry points use for aligned shapes: they move 16-byte pieces
// with many loads in flight per thread, so both run close to HBM bandwidth.

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;  // src-size 0 zero-fills the 16 bytes
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}

// project2: one CTA = 8 warps = one 16-row tile of X; warp w reduces the w-th
// eighth of K, loading kUnroll 32-element chunks of both rows before its MMAs.
template <int R>
__global__ void __launch_bounds__(256) project2_kernel(
    const __half* __restrict__ X, int64_t M, int64_t K, const __half* __restrict__ W,
    float scale_rows, __half* __restrict__ out_rows, int ld_rows, float scale_t,
    __half* __restrict__ out_t, int64_t ldt) {
  constexpr int NT = R / 8;
  constexpr int kWarps = 8;
  constexpr int kUnroll = 4;
  __shared__ float red[kWarps][16][R + 1];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int64_t m0 = static_cast<int64_t>(blockIdx.x) * 16;
  const int64_t chunks = K / 32;
  const int64_t c_begin = chunks * warp / kWarps, c_end = chunks * (warp + 1) / kWarps;
  float acc[NT][4];
#pragma unroll
  for (int j = 0; j < NT; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.0f;
  const bool r0ok = m0 + g < M, r1ok = m0 + g + 8 < M;
  const __half* x0 = X + (m0 + g) * K + 8 * t;
  const __half* x1 = X + (m0 + g + 8) * K + 8 * t;
  const __half* wrow = W + static_cast<int64_t>(g) * K + 8 * t;
  for (int64_t c = c_begin; c < c_end; c += kUnroll) {
    uint4 xa[kUnroll], xb[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const bool in = c + u < c_end;
      const int64_t k0 = (c + u) * 32;
      xa[u] = ldg16_or_zero(x0 + k0, in && r0ok);
      xb[u] = ldg16_or_zero(x1 + k0, in && r1ok);
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      if (c + u < c_end) {
        const int64_t k0 = (c + u) * 32;
        const uint32_t a_lo[4] = {xa[u].x, xb[u].x, xa[u].y, xb[u].y};
        const uint32_t a_hi[4] = {xa[u].z, xb[u].z, xa[u].w, xb[u].w};
#pragma unroll
        for (int j = 0; j < NT; ++j) {
          const uint4 w = __ldg(reinterpret_cast<const uint4*>(wrow + static_cast<int64_t>(8 * j) * K + k0));
          mma16816(acc[j], a_lo, w.x, w.y);
          mma16816(acc[j], a_hi, w.z, w.w);
        }
      }
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
  for (int i = threadIdx.x; i < 16 * R; i += blockDim.x) {
    const int row = i / R, col = i % R;
    float v = 0.0f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) v += red[w][row][col];
    const int64_t m = m0 + row;
    if (m < M) {
      if (out_rows) out_rows[m * ld_rows + col] = __float2half_rn(v * scale_rows);
      if (out_t) out_t[static_cast<int64_t>(col) * ldt + m] = __float2half_rn(v * scale_t);
    } else if (out_t && m < ldt) {
      out_t[static_cast<int64_t>(col) * ldt + m] = __float2half_rn(0.0f);  // zero pad for the reduction
    }
  }
}

// reduce2: CTA = 256 output columns (8 warps x 32) over rows [split * rows_per_split, ...).
// 32-row tiles of Q (16 KB) and Pt (R x 64 B) are staged with cp.async in a
// kStages ring; fragments come from ldmatrix (Q transposed).  Shared layouts are
// XOR-swizzled on 16-byte chunks so every ldmatrix phase hits 32 distinct banks:
// Q row k (512 B): chunk c stored at c ^ (k & 7); Pt row j (64 B): c at c ^ ((j >> 1) & 3).
// Requires Wd % 8 == 0, 16-byte aligned Q and Pt, ldp % 16 == 0.
constexpr int kRedCols = 256, kRedRows = 32, kRedStages = 4;

template <int R>
struct Red2Smem {
  static constexpr int kQBytes = kRedRows * kRedCols * 2;  // 16 KB
  static constexpr int kPBytes = R * kRedRows * 2;         // R x 64 B
  static constexpr int kStage = kQBytes + kPBytes;
  static constexpr int kBytes = kRedStages * kStage;
};

template <int R>
__global__ void __launch_bounds__(256) reduce2_kernel(
    const __half* __restrict__ Pt, int64_t ldp, const __half* __restrict__ Q, int64_t M,
    int64_t Wd, int64_t rows_per_split, float* __restrict__ partial) {
  using S = Red2Smem<R>;
  constexpr int MT = R / 16;
  extern __shared__ __align__(128) uint8_t red_smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int64_t c0 = static_cast<int64_t>(blockIdx.x) * kRedCols;
  const int64_t mb = static_cast<int64_t>(blockIdx.y) * rows_per_split;
  int64_t me = mb + rows_per_split;
  if (me > ldp) me = ldp;
  const int ntiles = me > mb ? static_cast<int>((me - mb + kRedRows - 1) / kRedRows) : 0;
  const uint32_t sbase = smem_addr(red_smem);

  auto issue = [&](int tile) {
    const int slot = tile % kRedStages;
    const uint32_t qs = sbase + slot * S::kStage;
    const uint32_t ps = qs + S::kQBytes;
    const int64_t r0 = mb + static_cast<int64_t>(tile) * kRedRows;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int row = (tid >> 5) + 8 * u, chunk = tid & 31;
      const int64_t m = r0 + row, col = c0 + chunk * 8;
      const bool ok = m < M && col < Wd;
      cp_async16(qs + row * 512 + ((chunk ^ (row & 7)) << 4), ok ? Q + m * Wd + col : Q, ok);
    }
    for (int i = tid; i < 4 * R; i += 256) {
      const int j = i >> 2, chunk = i & 3;
      const int64_t tok = r0 + chunk * 8;
      const bool ok = tok < ldp;
      cp_async16(ps + j * 64 + ((chunk ^ ((j >> 1) & 3)) << 4), ok ? Pt + j * ldp + tok : Pt, ok);
    }
  };

  float acc[MT][4][4];
#pragma unroll
  for (int i = 0; i < MT; ++i)
#pragma unroll
    for (int n = 0; n < 4; ++n) acc[i][n][0] = acc[i][n][1] = acc[i][n][2] = acc[i][n][3] = 0.0f;

#pragma unroll
  for (int s = 0; s < kRedStages - 1; ++s) {
    if (s < ntiles) issue(s);
    cp_async_commit();
  }
  const int mat = lane >> 3, r8 = lane & 7;
  for (int tile = 0; tile < ntiles; ++tile) {
    cp_async_wait<kRedStages - 2>();
    __syncthreads();
    if (tile + kRedStages - 1 < ntiles) issue(tile + kRedStages - 1);
    cp_async_commit();
    const int slot = tile % kRedStages;
    const uint32_t qs = sbase + slot * S::kStage;
    const uint32_t ps = qs + S::kQBytes;
#pragma unroll
    for (int ks = 0; ks < 2; ++ks) {
      uint32_t a[MT][4];
#pragma unroll
      for (int i = 0; i < MT; ++i) {
        const int j = 16 * i + r8 + 8 * (mat & 1);
        const int chunk = 2 * ks + (mat >> 1);
        ldsm_x4(ps + j * 64 + ((chunk ^ ((j >> 1) & 3)) << 4), a[i]);
      }
      uint32_t b[2][4];
#pragma unroll
      for (int pr = 0; pr < 2; ++pr) {
        const int k = 16 * ks + r8 + 8 * (mat & 1);
        const int chunk = warp * 4 + 2 * pr + (mat >> 1);
        ldsm_x4_trans(qs + k * 512 + ((chunk ^ (k & 7)) << 4), b[pr]);
      }
#pragma unroll
      for (int i = 0; i < MT; ++i) {
#pragma unroll
        for (int pr = 0; pr < 2; ++pr) {
          mma16816(acc[i][2 * pr], a[i], b[pr][0], b[pr][1]);
          mma16816(acc[i][2 * pr + 1], a[i], b[pr][2], b[pr][3]);
        }
      }
    }
  }
  cp_async_wait<0>();
  float* out = partial + static_cast<int64_t>(blockIdx.y) * R * Wd;
#pragma unroll
  for (int i = 0; i < MT; ++i) {
#pragma unroll
    for (int n = 0; n < 4; ++n) {
      const int64_t col = c0 + warp * 32 + 8 * n + 2 * t;
      if (col < Wd) {
        const int64_t ra = 16 * i + g;
        *reinterpret_cast<float2*>(out + ra * Wd + col) = make_float2(acc[i][n][0], acc[i][n][1]);
        *reinterpret_cast<float2*>(out + (ra + 8) * Wd + col) = make_float2(acc[i][n][2], acc[i][n][3]);
      }
    }
  }
}

// Split count of reduce2: enough CTAs to fill the GPU twice, at least 64 rows each.
inline int reduce2_splits(int64_t ldp, int64_t w) {
  const int64_t col_blocks = (w + kRedCols - 1) / kRedCols;
  int64_t s = (2 * device_sm_count() + col_blocks - 1) / col_blocks;
  const int64_t max_s = (ldp + 63) / 64;
  if (s > max_s) s = max_s;
  if (s < 1) s = 1;
  if (s > 4096) s = 4096;
  return static_cast<int>(s);
}

inline bool reduce2_ok(const void* pt, const void* q, int64_t w) {
  return w % 8 == 0 && aligned(pt, 16) && aligned(q, 16);
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

template <int R>
inline int launch_reduce2(dim3 grid, const __half* P, int64_t ldp, const __half* Q, int64_t m, int64_t w,
                          int64_t rows_per_split, float* partial, cudaStream_t st) {
  static std::mutex mu;
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lock(mu);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
      cudaError_t e = cudaFuncSetAttribute(reduce2_kernel<R>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           Red2Smem<R>::kBytes);
      if (e != cudaSuccess) return fail(SB_ECUDA, std::string("reduce2 smem attribute: ") + cudaGetErrorString(e));
      configured[dev] = true;
    }
  }
  reduce2_kernel<R><<<grid, 256, Red2Smem<R>::kBytes, st>>>(P, ldp, Q, m, w, rows_per_split, partial);
  count_launch();
  return check_launch("lora_reduce2_kernel");
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
  if (r == 16) sb::lora::project2_kernel<16><<<grid, 256, 0, st>>>(X, m, k, W, scale_rows, orow, ld_rows, scale_t, ot, ldt);
  else if (r == 32) sb::lora::project2_kernel<32><<<grid, 256, 0, st>>>(X, m, k, W, scale_rows, orow, ld_rows, scale_t, ot, ldt);
  else sb::lora::project2_kernel<64><<<grid, 256, 0, st>>>(X, m, k, W, scale_rows, orow, ld_rows, scale_t, ot, ldt);
  sb::count_launch();
  return sb::check_launch("lora_project2_kernel");
}

size_t sb_lora_reduce_workspace_bytes(int64_t m, int64_t w, int r) {
  if (m <= 0 || w <= 0 || r <= 0) return 0;
  const int64_t ldp = (m + 15) / 16 * 16;  // the zero-padded row count the reduction runs over
  const int64_t splits = std::max(sb::lora::reduce_splits(ldp, w), sb::lora::reduce2_splits(ldp, w));
  return static_cast<size_t>(splits) * r * w * sizeof(float);
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
  float* partial = static_cast<float*>(workspace);
  const __half* P = reinterpret_cast<const __half*>(pt);
  const __half* Q = reinterpret_cast<const __half*>(q);
  int splits = 0;
  if (sb::lora::reduce2_ok(pt, q, w)) {
    splits = sb::lora::reduce2_splits(ldp, w);
    int64_t rows_per_split = (ldp + splits - 1) / splits;
    rows_per_split = (rows_per_split + sb::lora::kRedRows - 1) / sb::lora::kRedRows * sb::lora::kRedRows;
    splits = static_cast<int>((ldp + rows_per_split - 1) / rows_per_split);
    const size_t need = static_cast<size_t>(splits) * r * w * sizeof(float);
    if (!workspace || workspace_bytes < need) return sb::fail(SB_EWORKSPACE, "LoRA reduce workspace too small");
    dim3 grid(static_cast<unsigned>((w + sb::lora::kRedCols - 1) / sb::lora::kRedCols), static_cast<unsigned>(splits));
    int rc = SB_OK;
    if (r == 16) rc = sb::lora::launch_reduce2<16>(grid, P, ldp, Q, m, w, rows_per_split, partial, st);
    else if (r == 32) rc = sb::lora::launch_reduce2<32>(grid, P, ldp, Q, m, w, rows_per_split, partial, st);
    else rc = sb::lora::launch_reduce2<64>(grid, P, ldp, Q, m, w, rows_per_split, partial, st);
    if (rc) return rc;
  } else {
    splits = sb::lora::reduce_splits(ldp, w);
    const size_t need = static_cast<size_t>(splits) * r * w * sizeof(float);
    if (!workspace || workspace_bytes < need) return sb::fail(SB_EWORKSPACE, "LoRA reduce workspace too small");
    int64_t rows_per_split = (ldp + splits - 1) / splits;
    rows_per_split = (rows_per_split + 15) / 16 * 16;
    dim3 grid(static_cast<unsigned>((w + 127) / 128), static_cast<unsigned>(splits));
    if (r == 16) sb::lora::reduce_partial_kernel<16><<<grid, 256, 0, st>>>(P, ldp, Q, m, w, rows_per_split, partial);
    else if (r == 32) sb::lora::reduce_partial_kernel<32><<<grid, 256, 0, st>>>(P, ldp, Q, m, w, rows_per_split, partial);
    else sb::lora::reduce_partial_kernel<64><<<grid, 256, 0, st>>>(P, ldp, Q, m, w, rows_per_split, partial);
    sb::count_launch();
    if (int rc = sb::check_launch("lora_reduce_partial_kernel")) return rc;
  }
  const int64_t total = w * r;
  if (w % 4 == 0) {
    sb::lora::reduce_finalize2_kernel<<<static_cast<unsigned>((total / 4 + 15) / 16), 256, 0, st>>>(
        partial, splits, w, r, scale, transpose, out, out_dtype);
    sb::count_launch();
    return sb::check_launch("lora_reduce_finalize2_kernel");
  }
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
