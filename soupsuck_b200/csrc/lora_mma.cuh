// LoRA low-rank kernels on the legacy tensor-core path (mma.sync m16n8k16, fp32 accumulate).
//
// These products are skinny (rank r = 16..64) and HBM-bound: each streams one
// activation-sized matrix once, so they use register-fragment MMAs fed by wide
// coalesced loads rather than the tcgen05 pipeline.
//
//   project  out[M, R] = X[M, K] . W[R, K]^T          (Z = X.A^T, U = dY.B);
//            ranks 16 / 32 split the reduction over a cluster (project3)
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

// Finalize of the streamed reduction: one thread per four outputs adds the splits'
// fp32 partials in split order (16-byte loads, four splits in flight), scales and
// stores; enough threads for the whole output in one wave.
__global__ void __launch_bounds__(256) reduce_finalize3_kernel(const float* __restrict__ partial, int splits,
                                                               int64_t Wd, int r, float scale, int transpose,
                                                               void* __restrict__ out, int odt) {
  const int64_t total4 = Wd * r / 4;
  const int64_t e4 = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (e4 >= total4) return;
  const float4* src = reinterpret_cast<const float4*>(partial) + e4;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  int s = 0;
  for (; s + 4 <= splits; s += 4) {
    float4 v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) v[u] = __ldcg(src + static_cast<int64_t>(s + u) * total4);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      acc.x += v[u].x; acc.y += v[u].y; acc.z += v[u].z; acc.w += v[u].w;
    }
  }
  for (; s < splits; ++s) {
    const float4 v = __ldcg(src + static_cast<int64_t>(s) * total4);
    acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
  }
  const float vals[4] = {acc.x * scale, acc.y * scale, acc.z * scale, acc.w * scale};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t e = e4 * 4 + i;
    const int64_t j = e / Wd, c = e % Wd;
    st_from_f32(out, odt, transpose ? c * r + j : j * Wd + c, vals[i]);
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

// project3: the projection for ranks <= 32 with the reduction split over a
// cluster.  A cluster of S CTAs owns one block of 32 rows (two m16 tiles, so each
// W fragment feeds two MMAs); CTA `rank` reduces columns [K*rank/S, K*(rank+1)/S)
// with its 8 warps, the warps' partials meet in shared memory, and the S CTA
// partials are added in rank order through distributed shared memory, each rank
// finishing a share of the 32 x R outputs (fixed order: deterministic).  S is
// chosen so that about four CTAs run per SM whatever the row count, which keeps
// enough 16-byte loads in flight to stream X at HBM rate.
constexpr int kProj3Rows = 32;
constexpr int64_t kProj3MinK = 4096;  // rows at least this long take the cluster split

template <int R>
__global__ void __launch_bounds__(256) project3_kernel(
    const __half* __restrict__ X, int64_t M, int64_t K, const __half* __restrict__ W, int S,
    float scale_rows, __half* __restrict__ out_rows, int ld_rows, float scale_t,
    __half* __restrict__ out_t, int64_t ldt) {
  static_assert(R == 16 || R == 32, "cluster projection for ranks 16 and 32");
  constexpr int NT = R / 8, MT = 2, kWarps = 8, kUnroll = 4;
  __shared__ float red[kWarps][kProj3Rows][R + 1];
  __shared__ float part[kProj3Rows * R];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const uint32_t rank = gemm::pair::cluster_rank();
  const int64_t m0 = static_cast<int64_t>(blockIdx.x / S) * kProj3Rows;
  const int64_t chunks = K / 32;
  const int64_t cta_b = chunks * rank / S, cta_e = chunks * (rank + 1) / S;
  const int64_t c_begin = cta_b + (cta_e - cta_b) * warp / kWarps;
  const int64_t c_end = cta_b + (cta_e - cta_b) * (warp + 1) / kWarps;
  float acc[MT][NT][4];
#pragma unroll
  for (int i = 0; i < MT; ++i)
#pragma unroll
    for (int j = 0; j < NT; ++j) acc[i][j][0] = acc[i][j][1] = acc[i][j][2] = acc[i][j][3] = 0.0f;
  const __half* xr[MT][2];
  bool rok[MT][2];
#pragma unroll
  for (int i = 0; i < MT; ++i)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int64_t row = m0 + 16 * i + g + 8 * h;
      rok[i][h] = row < M;
      xr[i][h] = X + (rok[i][h] ? row : 0) * K + 8 * t;
    }
  const __half* wrow = W + static_cast<int64_t>(g) * K + 8 * t;
  for (int64_t c = c_begin; c < c_end; c += kUnroll) {
    uint4 xv[kUnroll][MT][2];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const bool in = c + u < c_end;
      const int64_t k0 = (c + u) * 32;
#pragma unroll
      for (int i = 0; i < MT; ++i)
#pragma unroll
        for (int h = 0; h < 2; ++h) xv[u][i][h] = ldg16_or_zero(xr[i][h] + k0, in && rok[i][h]);
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      if (c + u < c_end) {
        const int64_t k0 = (c + u) * 32;
#pragma unroll
        for (int j = 0; j < NT; ++j) {
          const uint4 w = __ldg(reinterpret_cast<const uint4*>(wrow + static_cast<int64_t>(8 * j) * K + k0));
#pragma unroll
          for (int i = 0; i < MT; ++i) {
            const uint32_t a_lo[4] = {xv[u][i][0].x, xv[u][i][1].x, xv[u][i][0].y, xv[u][i][1].y};
            const uint32_t a_hi[4] = {xv[u][i][0].z, xv[u][i][1].z, xv[u][i][0].w, xv[u][i][1].w};
            mma16816(acc[i][j], a_lo, w.x, w.y);
            mma16816(acc[i][j], a_hi, w.z, w.w);
          }
        }
      }
    }
  }
#pragma unroll
  for (int i = 0; i < MT; ++i)
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      red[warp][16 * i + g][8 * j + 2 * t] = acc[i][j][0];
      red[warp][16 * i + g][8 * j + 2 * t + 1] = acc[i][j][1];
      red[warp][16 * i + g + 8][8 * j + 2 * t] = acc[i][j][2];
      red[warp][16 * i + g + 8][8 * j + 2 * t + 1] = acc[i][j][3];
    }
  __syncthreads();
  for (int e = threadIdx.x; e < kProj3Rows * R; e += blockDim.x) {
    const int row = e / R, col = e % R;
    float v = 0.0f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) v += red[w][row][col];
    part[e] = v;
  }
  gemm::pair::cluster_sync_all();
  const uint32_t part_s = smem_addr(part);
  const int total = kProj3Rows * R;
  const int share = (total + S - 1) / S;
  const int e0 = static_cast<int>(rank) * share;
  const int e1 = e0 + share < total ? e0 + share : total;
  for (int e = e0 + threadIdx.x; e < e1; e += blockDim.x) {
    const int row = e / R, col = e % R;
    float v = 0.0f;
    for (int q = 0; q < S; ++q) {
      const uint32_t addr = gemm::pair::map_to_rank(part_s + static_cast<uint32_t>(e * 4), static_cast<uint32_t>(q));
      float pv;
      asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(pv) : "r"(addr) : "memory");
      v += pv;
    }
    const int64_t m = m0 + row;
    if (m < M) {
      if (out_rows) out_rows[m * ld_rows + col] = __float2half_rn(v * scale_rows);
      if (out_t) out_t[static_cast<int64_t>(col) * ldt + m] = __float2half_rn(v * scale_t);
    } else if (out_t && m < ldt) {
      out_t[static_cast<int64_t>(col) * ldt + m] = __float2half_rn(0.0f);  // zero pad for the reduction
    }
  }
  gemm::pair::cluster_sync_all();  // no CTA leaves while a peer still reads its partial
}

// Cluster size of project3 for m rows and k columns (see above).
inline int project3_split(int64_t m, int64_t k) {
  const int64_t blocks = (m + kProj3Rows - 1) / kProj3Rows;
  const int64_t want = (4 * static_cast<int64_t>(device_sm_count()) + blocks - 1) / blocks;
  int64_t s = want < 8 ? want : 8;
  const int64_t cap = k / 32 / 32;  // every warp keeps at least four 32-column chunks
  if (s > cap) s = cap;
  return static_cast<int>(s < 1 ? 1 : s);
}

template <int R>
inline int launch_project3(const __half* X, int64_t m, int64_t k, const __half* W, float scale_rows, __half* orow,
                           int ld_rows, float scale_t, __half* ot, int64_t ldt, cudaStream_t st) {
  const int S = project3_split(m, k);
  const int64_t blocks = (m + kProj3Rows - 1) / kProj3Rows;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(blocks * S), 1, 1);
  cfg.blockDim = dim3(256, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(S);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, project3_kernel<R>, X, m, k, W, S, scale_rows, orow, ld_rows, scale_t,
                                     ot, ldt);
  if (e != cudaSuccess) return fail(SB_ECUDA, std::string("lora_project3 launch: ") + cudaGetErrorString(e));
  count_launch();
  return check_launch("lora_project3_kernel");
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
  // One index range per output array, so every array is written in order
  // (coalesced); the small inputs are read through the caches.  Sizes fit 32 bits.
  const uint32_t rr = static_cast<uint32_t>(r), kk = static_cast<uint32_t>(K), nn = static_cast<uint32_t>(N);
  const uint32_t na = rr * kk, nbv = rr * nn;
  const uint32_t total = 2 * na + 2 * nbv;
  const uint32_t stride = gridDim.x * blockDim.x;
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    if (i < na) {
      if (a16) a16[i] = __float2half_rn(ld_as_f32(a, adt, i));
    } else if (i < 2 * na) {
      const uint32_t e = i - na, k = e / rr, j = e - k * rr;  // at16[k][j] = a[j][k]
      if (at16) at16[e] = __float2half_rn(ld_as_f32(a, adt, static_cast<int64_t>(j) * kk + k));
    } else if (i < 2 * na + nbv) {
      const uint32_t e = i - 2 * na;
      if (b16) b16[e] = __float2half_rn(ld_as_f32(b, bdt, e));
    } else {
      const uint32_t e = i - 2 * na - nbv, j = e / nn, n = e - j * nn;  // bt16[j][n] = b[n][j]
      if (bt16) bt16[e] = __float2half_rn(ld_as_f32(b, bdt, static_cast<int64_t>(n) * rr + j));
    }
  }
}

// Two adapters of one input as one rank-2r adapter: a1, a2 [r, K] and b1, b2 [N, r]
// (dtype adt / bdt) -> a_cat [2r, K] (a1 over a2), at_cat [K, 2r], b_bd [2N, 2r]
// = [[b1, 0], [0, b2]] and bt_bd [2r, 2N] (its transpose), fp16, zero blocks
// written too.  One index range per output array (each written in order).
__global__ void pair_prepare_kernel(const void* __restrict__ a1, const void* __restrict__ a2, int adt,
                                    const void* __restrict__ b1, const void* __restrict__ b2, int bdt, int r,
                                    int64_t K, int64_t N, __half* __restrict__ a_cat, __half* __restrict__ at_cat,
                                    __half* __restrict__ b_bd, __half* __restrict__ bt_bd) {
  const uint32_t rr = static_cast<uint32_t>(r), r2 = 2 * rr, kk = static_cast<uint32_t>(K);
  const uint32_t n2 = 2 * static_cast<uint32_t>(N), nn = static_cast<uint32_t>(N);
  const uint32_t na = r2 * kk, nbv = n2 * r2;
  const uint32_t total = 2 * na + 2 * nbv;
  const uint32_t stride = gridDim.x * blockDim.x;
  // a_cat[j][k] for j in [0, 2r); b_bd[row][c] is b1 / b2 on the diagonal blocks.
  auto a_val = [&](uint32_t j, uint32_t k) -> __half {
    const bool second = j >= rr;
    return __float2half_rn(ld_as_f32(second ? a2 : a1, adt, static_cast<int64_t>(second ? j - rr : j) * kk + k));
  };
  auto b_val = [&](uint32_t row, uint32_t c) -> __half {
    const bool row2 = row >= nn, col2 = c >= rr;
    if (row2 != col2) return __float2half_rn(0.0f);
    return __float2half_rn(ld_as_f32(row2 ? b2 : b1, bdt, static_cast<int64_t>(row2 ? row - nn : row) * rr +
                                                              (col2 ? c - rr : c)));
  };
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    if (i < na) {
      const uint32_t j = i / kk;
      a_cat[i] = a_val(j, i - j * kk);
    } else if (i < 2 * na) {
      const uint32_t e = i - na, k = e / r2;
      at_cat[e] = a_val(e - k * r2, k);
    } else if (i < 2 * na + nbv) {
      const uint32_t e = i - 2 * na, row = e / r2;
      b_bd[e] = b_val(row, e - row * r2);
    } else {
      const uint32_t e = i - 2 * na - nbv, c = e / n2;
      bt_bd[e] = b_val(e - c * n2, c);
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

// ------------------------------------------------------------------ dual
// The LoRA backward reads its upstream gradient Q = dY [M, W] for two products:
// u = Q . Bt^T [M, r] (the rank-r factor of the input gradient and of dA) and
// dB = Pt . Q [r, W] with Pt = Z^T (the forward's rank-r factor, transposed).  For
// the MLP's dgate|dup that is 118 MB per read.  dual_kernel streams every
// [32 x 256] tile of Q once, through the reduce2 ring, into both:
//   * dB: the CTA's 256 columns over its row split, as reduce2 (partials per
//     split, summed by the reduce finalize kernels);
//   * u: the tile's 32 rows over the CTA's 256 columns, from the CTA's block of Bt
//     held in shared memory; written per column block and summed by
//     dual_u_finalize_kernel.
// Block-diagonal mode (wsplit > 0: two adapters side by side, the gate/up pair):
// columns below wsplit use factor rows [0, RH) of Pt and Bt, the others rows
// [RH, 2 RH); only those diagonal blocks are computed -- u's off-diagonal blocks
// multiply zeros, and dB's are not wanted.  wsplit is a multiple of 256, so a
// column block lies on one side.
// Warps for u: (m16 tile mi, group nq of RH/16 n8 tiles, column half kh), the two
// column halves added in fixed order through shared memory.  DB = false: u only
// (the forward's Z = X.A^T for long rows), without Pt, dB or its partials.
// Three ring slots (two tiles in flight): 63 KB of shared memory at RH = 16, so
// three CTAs (24 warps) share an SM.  The kernel waits on shared-memory and MMA
// latency (ldmatrix -> mma chains) more than on bytes in flight.
constexpr int kDualStages = 3;

template <int RH>
struct DualSmem {
  static constexpr int kStage = Red2Smem<RH>::kStage;
  static constexpr int kRing = kDualStages * kStage;
  static constexpr int kBtBytes = RH * kRedCols * 2;           // the CTA's Bt block
  static constexpr int kXchBytes = 2 * 4 * 32 * (RH / 4) * 4;  // two tiles' column-half partials
  static constexpr int kBytes = kRing + kBtBytes + kXchBytes;
};

template <int RH, bool DB>
__global__ void __launch_bounds__(256) dual_kernel(
    const __half* __restrict__ Pt, int64_t ldp, const __half* __restrict__ Bt, int64_t ldb,
    const __half* __restrict__ Q, int64_t M, int64_t Wd, int64_t wsplit, int64_t rows_end,
    int64_t rows_per_split, float* __restrict__ partial, float* __restrict__ upart, int64_t ldq) {
  using S = DualSmem<RH>;
  constexpr int MT = RH / 16;  // dB: m16 tiles of factor rows
  constexpr int NPW = RH / 16; // u: n8 tiles per warp
  extern __shared__ __align__(128) uint8_t dual_smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int64_t c0 = static_cast<int64_t>(blockIdx.x) * kRedCols;
  const int64_t jbase = (wsplit > 0 && c0 >= wsplit) ? RH : 0;
  const int64_t mb = static_cast<int64_t>(blockIdx.y) * rows_per_split;
  int64_t me = mb + rows_per_split;
  if (me > rows_end) me = rows_end;
  const int ntiles = me > mb ? static_cast<int>((me - mb + kRedRows - 1) / kRedRows) : 0;
  const uint32_t sbase = smem_addr(dual_smem);
  const uint32_t bts = sbase + S::kRing;
  float* xch = reinterpret_cast<float*>(dual_smem + S::kRing + S::kBtBytes);

  auto issue = [&](int tile) {
    const int slot = tile % kDualStages;
    const uint32_t qs = sbase + slot * S::kStage;
    const uint32_t ps = qs + Red2Smem<RH>::kQBytes;
    const int64_t r0 = mb + static_cast<int64_t>(tile) * kRedRows;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int row = (tid >> 5) + 8 * u, chunk = tid & 31;
      const int64_t m = r0 + row, col = c0 + chunk * 8;
      const bool ok = m < M && col < Wd;
      cp_async16(qs + row * 512 + ((chunk ^ (row & 7)) << 4), ok ? Q + m * Wd + col : Q, ok);
    }
    if constexpr (DB) {
      for (int i = tid; i < 4 * RH; i += 256) {
        const int j = i >> 2, chunk = i & 3;
        const int64_t tok = r0 + chunk * 8;
        const bool ok = tok < ldp;
        cp_async16(ps + j * 64 + ((chunk ^ ((j >> 1) & 3)) << 4), ok ? Pt + (jbase + j) * ldp + tok : Pt, ok);
      }
    }
  };

  // The CTA's Bt block (rows jbase .. jbase + RH, its 256 columns): part of group 0.
  for (int i = tid; i < RH * 32; i += 256) {
    const int j = i >> 5, chunk = i & 31;
    const int64_t col = c0 + chunk * 8;
    const bool ok = col < Wd;
    cp_async16(bts + j * 512 + ((chunk ^ (j & 7)) << 4), ok ? Bt + (jbase + j) * ldb + col : Bt, ok);
  }

  float acc[MT][4][4];
#pragma unroll
  for (int i = 0; i < MT; ++i)
#pragma unroll
    for (int n = 0; n < 4; ++n) acc[i][n][0] = acc[i][n][1] = acc[i][n][2] = acc[i][n][3] = 0.0f;

#pragma unroll
  for (int s = 0; s < kDualStages - 1; ++s) {
    if (s < ntiles) issue(s);
    cp_async_commit();
  }
  const int mat = lane >> 3, r8 = lane & 7;
  const int mi = warp & 1, nq = (warp >> 1) & 1, kh = warp >> 2;
  const int64_t ublock = static_cast<int64_t>(blockIdx.x) * ldq;
  for (int tile = 0; tile < ntiles; ++tile) {
    cp_async_wait<kDualStages - 2>();
    __syncthreads();
    if (tile + kDualStages - 1 < ntiles) issue(tile + kDualStages - 1);
    cp_async_commit();
    const int slot = tile % kDualStages;
    const uint32_t qs = sbase + slot * S::kStage;
    const uint32_t ps = qs + Red2Smem<RH>::kQBytes;
    // dB += Pt[:, tile rows] . Q[tile rows, warp's 32 columns]
#pragma unroll
    for (int ks = 0; ks < (DB ? 2 : 0); ++ks) {
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
    // u[tile rows 16 mi .., n8 tiles of group nq] over column half kh
    float uacc[NPW][4];
#pragma unroll
    for (int n = 0; n < NPW; ++n) uacc[n][0] = uacc[n][1] = uacc[n][2] = uacc[n][3] = 0.0f;
    const int arow = 16 * mi + r8 + 8 * (mat & 1);
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const int cb = kh * 16 + kk * 4;  // first 16-byte chunk of this pair of k16 steps
      uint32_t a0[4], a1[4];
      ldsm_x4(qs + arow * 512 + (((cb + (mat >> 1)) ^ (arow & 7)) << 4), a0);
      ldsm_x4(qs + arow * 512 + (((cb + 2 + (mat >> 1)) ^ (arow & 7)) << 4), a1);
#pragma unroll
      for (int n = 0; n < NPW; ++n) {
        const int j = 8 * (nq * NPW + n) + r8;
        uint32_t bb[4];
        ldsm_x4(bts + j * 512 + (((cb + mat) ^ (j & 7)) << 4), bb);
        mma16816(uacc[n], a0, bb[0], bb[1]);
        mma16816(uacc[n], a1, bb[2], bb[3]);
      }
    }
    float* x = xch + ((tile & 1) * 4 + (warp & 3)) * 32 * (RH / 4) + lane * (RH / 4);
    if (kh == 1) {
#pragma unroll
      for (int n = 0; n < NPW; ++n)
        *reinterpret_cast<float4*>(x + 4 * n) = make_float4(uacc[n][0], uacc[n][1], uacc[n][2], uacc[n][3]);
    }
    __syncthreads();
    if (kh == 0) {
      const int64_t r0 = mb + static_cast<int64_t>(tile) * kRedRows + 16 * mi + g;
#pragma unroll
      for (int n = 0; n < NPW; ++n) {
        const float4 o = *reinterpret_cast<const float4*>(x + 4 * n);
        const int j = 8 * (nq * NPW + n) + 2 * t;
        if (r0 < ldq)
          *reinterpret_cast<float2*>(upart + (ublock + r0) * RH + j) = make_float2(uacc[n][0] + o.x, uacc[n][1] + o.y);
        if (r0 + 8 < ldq)
          *reinterpret_cast<float2*>(upart + (ublock + r0 + 8) * RH + j) =
              make_float2(uacc[n][2] + o.z, uacc[n][3] + o.w);
      }
    }
  }
  cp_async_wait<0>();
  if constexpr (DB) {
    float* out = partial + static_cast<int64_t>(blockIdx.y) * RH * Wd;
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
}

// u[m, j] = fp16(scale * sum of upart[cb][m][j mod RH] over the column blocks of
// j's side), rows m < M into out_rows [M, ld_rows], and transposed into out_t
// [rout, ldt] with zeros for rows M .. ldt.  A CTA: 8 groups x 32 float4 outputs;
// group q adds blocks q, q + 8, ... and the group sums are added in group order.
__global__ void __launch_bounds__(256) dual_u_finalize_kernel(
    const float* __restrict__ upart, int nblocks, int split_block, int64_t ldq, int rh, int rout, int64_t M,
    float scale_rows, __half* __restrict__ out_rows, int ld_rows, float scale_t, __half* __restrict__ out_t,
    int64_t ldt) {
  __shared__ float4 part[8][33];
  const int col = threadIdx.x & 31, grp = threadIdx.x >> 5;
  const int q4 = rout / 4;
  const int64_t total4 = ldq * q4;
  const int64_t e4 = static_cast<int64_t>(blockIdx.x) * 32 + col;
  const int64_t m = e4 / q4;
  const int j = static_cast<int>(e4 % q4) * 4;
  const int side = (split_block > 0 && j >= rh) ? 1 : 0;
  const int lo = side ? split_block : 0;
  const int hi = (split_block > 0 && !side) ? split_block : nblocks;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  if (e4 < total4) {
    const int jj = j - side * rh;
    for (int cb = lo + grp; cb < hi; cb += 8) {
      const float4 v = __ldcg(reinterpret_cast<const float4*>(upart + (static_cast<int64_t>(cb) * ldq + m) * rh + jj));
      acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
    }
  }
  part[grp][col] = acc;
  __syncthreads();
  if (grp != 0 || e4 >= total4) return;
  float4 s = part[0][col];
#pragma unroll
  for (int q = 1; q < 8; ++q) {
    const float4 v = part[q][col];
    s.x += v.x; s.y += v.y; s.z += v.z; s.w += v.w;
  }
  const float vals[4] = {s.x, s.y, s.z, s.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (m < M) {
      if (out_rows) out_rows[m * ld_rows + j + i] = __float2half_rn(vals[i] * scale_rows);
      if (out_t) out_t[static_cast<int64_t>(j + i) * ldt + m] = __float2half_rn(vals[i] * scale_t);
    } else if (out_t && m < ldt) {
      out_t[static_cast<int64_t>(j + i) * ldt + m] = __float2half_rn(0.0f);
    }
  }
}

template <int RH, bool DB>
inline int launch_dual(dim3 grid, const __half* P, int64_t ldp, const __half* Bt, int64_t ldb, const __half* Q,
                       int64_t m, int64_t w, int64_t wsplit, int64_t rows_end, int64_t rows_per_split,
                       float* partial, float* upart, int64_t ldq, cudaStream_t st) {
  static std::mutex mu;
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lock(mu);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
      cudaError_t e = cudaFuncSetAttribute(dual_kernel<RH, DB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           DualSmem<RH>::kBytes);
      if (e != cudaSuccess) return fail(SB_ECUDA, std::string("dual smem attribute: ") + cudaGetErrorString(e));
      configured[dev] = true;
    }
  }
  dual_kernel<RH, DB><<<grid, 256, DualSmem<RH>::kBytes, st>>>(P, ldp, Bt, ldb, Q, m, w, wsplit, rows_end,
                                                             rows_per_split, partial, upart, ldq);
  count_launch();
  return check_launch("lora_dual_kernel");
}

// Row plan of dual_kernel for m rows and w columns: (splits, rows per split), the
// splits as reduce2's, over the 16-row padded length.
struct DualPlan {
  int64_t ldq, rows_per_split;
  int splits, nblocks;
  size_t partial_bytes, upart_bytes;
};

// The split count is chosen for whole waves of dual_kernel (three CTAs per SM at
// RH = 16, two at RH = 32): cost = waves x (row tiles per CTA + one for the
// CTA's partial-sum write), fewest splits on ties.
inline DualPlan dual_plan(int64_t m, int64_t w, int rh) {
  DualPlan d{};
  d.ldq = (m + 15) / 16 * 16;
  d.nblocks = static_cast<int>((w + kRedCols - 1) / kRedCols);
  const int64_t slots = (rh == 16 ? 3 : 2) * static_cast<int64_t>(device_sm_count());
  const int64_t max_s = std::max<int64_t>(1, std::min<int64_t>(4096, (d.ldq + 63) / 64));
  int64_t best_rps = d.ldq, best_cost = INT64_MAX;
  for (int64_t s = 1; s <= max_s; ++s) {
    int64_t rps = (d.ldq + s - 1) / s;
    rps = (rps + kRedRows - 1) / kRedRows * kRedRows;
    const int64_t splits = (d.ldq + rps - 1) / rps;
    const int64_t waves = (d.nblocks * splits + slots - 1) / slots;
    const int64_t cost = waves * (rps / kRedRows + 1);
    if (cost < best_cost) {
      best_cost = cost;
      best_rps = rps;
    }
  }
  const int64_t rps = best_rps;
  d.rows_per_split = rps;
  d.splits = static_cast<int>((d.ldq + rps - 1) / rps);
  d.partial_bytes = (static_cast<size_t>(d.splits) * rh * w * sizeof(float) + 255) / 256 * 256;
  d.upart_bytes = static_cast<size_t>(d.nblocks) * d.ldq * rh * sizeof(float);
  return d;
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
  // Long rows (the MLP's act, dgate|dup) take the cluster-split kernel; short rows
  // (hidden-size inputs) keep one 16-row tile per CTA, which already yields more
  // CTAs than SMs and no cluster exchange.
  const bool split = k >= sb::lora::kProj3MinK;
  if (r == 16 && split) return sb::lora::launch_project3<16>(X, m, k, W, scale_rows, orow, ld_rows, scale_t, ot, ldt, st);
  if (r == 32 && split) return sb::lora::launch_project3<32>(X, m, k, W, scale_rows, orow, ld_rows, scale_t, ot, ldt, st);
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
  if (w % 4 == 0 && splits >= 16) {
    // Many splits over few outputs: spread the splits over 16 thread groups.
    sb::lora::reduce_finalize2_kernel<<<static_cast<unsigned>((total / 4 + 15) / 16), 256, 0, st>>>(
        partial, splits, w, r, scale, transpose, out, out_dtype);
    sb::count_launch();
    return sb::check_launch("lora_reduce_finalize2_kernel");
  }
  if (w % 4 == 0) {
    sb::lora::reduce_finalize3_kernel<<<static_cast<unsigned>((total / 4 + 255) / 256), 256, 0, st>>>(
        partial, splits, w, r, scale, transpose, out, out_dtype);
    sb::count_launch();
    return sb::check_launch("lora_reduce_finalize3_kernel");
  }
  sb::lora::reduce_finalize_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, st>>>(
      partial, splits, w, r, scale, transpose, out, out_dtype);
  sb::count_launch();
  return sb::check_launch("lora_reduce_finalize_kernel");
}

size_t sb_lora_dual_workspace_bytes(int64_t m, int64_t w, int r, int64_t wsplit) {
  if (m <= 0 || w <= 0 || r <= 0) return 0;
  const int rh = wsplit > 0 ? r / 2 : r;
  const sb::lora::DualPlan d = sb::lora::dual_plan(m, w, rh);
  return d.partial_bytes + d.upart_bytes;
}

int sb_lora_dual(const uint16_t* q, int64_t m, int64_t w, const uint16_t* pt, int64_t ldp, const uint16_t* bt,
                 int r, int64_t wsplit, float scale_b, int transpose_b, void* db_out, int db_dtype,
                 float scale_rows, uint16_t* u_rows, int ld_rows, float scale_t, uint16_t* u_t, int64_t ldt,
                 void* workspace, size_t workspace_bytes, void* stream) {
  SB_REQUIRE(m >= 0 && w > 0, "expected m >= 0 and w > 0");
  SB_REQUIRE(w % 8 == 0, "w must be a multiple of 8");
  SB_REQUIRE(wsplit >= 0 && wsplit < w, "wsplit must be in [0, w)");
  if (wsplit > 0) {
    SB_REQUIRE(wsplit % sb::lora::kRedCols == 0, "wsplit must be a multiple of 256");
    SB_REQUIRE(r == 32 || r == 64, "block-diagonal rank must be 32 or 64 (two halves of 16 or 32)");
  } else {
    SB_REQUIRE(r == 16 || r == 32, "rank must be 16 or 32 (pad smaller ranks with zeros)");
  }
  SB_REQUIRE(!pt || (ldp >= m && ldp % 16 == 0), "ldp must be >= m and a multiple of 16 (zero padded)");
  SB_REQUIRE(!pt || db_dtype == SB_F16 || db_dtype == SB_F32, "bad dB dtype");
  SB_REQUIRE(!u_rows || ld_rows >= r, "ld_rows must be >= r");
  SB_REQUIRE(!u_t || (ldt >= m && ldt <= (m + 15) / 16 * 16), "ldt must be m rounded up to at most 16");
  SB_REQUIRE(!pt || db_out != nullptr, "NULL dB output");
  const int rh = wsplit > 0 ? r / 2 : r;
  cudaStream_t st = sb::as_stream(stream);
  if (m == 0) {
    if (!pt) return SB_OK;
    cudaError_t e = cudaMemsetAsync(db_out, 0, static_cast<size_t>(rh) * w * (db_dtype == SB_F32 ? 4 : 2), st);
    return e == cudaSuccess ? SB_OK : sb::fail(SB_ECUDA, cudaGetErrorString(e));
  }
  SB_REQUIRE(q && bt && (u_rows || u_t), "NULL pointer argument");
  SB_REQUIRE(sb::aligned(q, 16) && sb::aligned(bt, 16) && (!pt || sb::aligned(pt, 16)),
             "q, pt and bt must be 16-byte aligned");
  const sb::lora::DualPlan d = sb::lora::dual_plan(m, w, rh);
  if (!workspace || workspace_bytes < d.partial_bytes + d.upart_bytes)
    return sb::fail(SB_EWORKSPACE, "LoRA dual workspace too small");
  float* partial = static_cast<float*>(workspace);
  float* upart = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + d.partial_bytes);
  const __half* P = reinterpret_cast<const __half*>(pt);
  const __half* B = reinterpret_cast<const __half*>(bt);
  const __half* Q = reinterpret_cast<const __half*>(q);
  dim3 grid(static_cast<unsigned>(d.nblocks), static_cast<unsigned>(d.splits));
  int rc;
  if (P) {
    rc = rh == 16 ? sb::lora::launch_dual<16, true>(grid, P, ldp, B, w, Q, m, w, wsplit, d.ldq, d.rows_per_split,
                                                    partial, upart, d.ldq, st)
                  : sb::lora::launch_dual<32, true>(grid, P, ldp, B, w, Q, m, w, wsplit, d.ldq, d.rows_per_split,
                                                    partial, upart, d.ldq, st);
  } else {
    rc = rh == 16 ? sb::lora::launch_dual<16, false>(grid, P, ldp, B, w, Q, m, w, wsplit, d.ldq, d.rows_per_split,
                                                     partial, upart, d.ldq, st)
                  : sb::lora::launch_dual<32, false>(grid, P, ldp, B, w, Q, m, w, wsplit, d.ldq, d.rows_per_split,
                                                     partial, upart, d.ldq, st);
  }
  if (rc) return rc;
  const int64_t total = w * rh;
  if (!P) {
    // u only
  } else if (d.splits >= 16) {
    sb::lora::reduce_finalize2_kernel<<<static_cast<unsigned>((total / 4 + 15) / 16), 256, 0, st>>>(
        partial, d.splits, w, rh, scale_b, transpose_b, db_out, db_dtype);
    sb::count_launch();
    if ((rc = sb::check_launch("lora_reduce_finalize2_kernel"))) return rc;
  } else {
    sb::lora::reduce_finalize3_kernel<<<static_cast<unsigned>((total / 4 + 255) / 256), 256, 0, st>>>(
        partial, d.splits, w, rh, scale_b, transpose_b, db_out, db_dtype);
    sb::count_launch();
    if ((rc = sb::check_launch("lora_reduce_finalize3_kernel"))) return rc;
  }
  const int64_t total4 = d.ldq * (r / 4);
  sb::lora::dual_u_finalize_kernel<<<static_cast<unsigned>((total4 + 31) / 32), 256, 0, st>>>(
      upart, d.nblocks, wsplit > 0 ? static_cast<int>(wsplit / sb::lora::kRedCols) : 0, d.ldq, rh, r, m,
      scale_rows, reinterpret_cast<__half*>(u_rows), ld_rows, scale_t, reinterpret_cast<__half*>(u_t), ldt);
  sb::count_launch();
  return sb::check_launch("lora_dual_u_finalize_kernel");
}

int sb_lora_prepare(const void* a, int a_dtype, const void* b, int b_dtype, int r, int64_t k,
                    int64_t n, uint16_t* a16, uint16_t* at16, uint16_t* b16, uint16_t* bt16,
                    void* stream) {
  SB_REQUIRE(r > 0 && k > 0 && n > 0, "expected positive sizes");
  SB_REQUIRE((a_dtype == SB_F16 || a_dtype == SB_F32) && (b_dtype == SB_F16 || b_dtype == SB_F32), "bad dtype");
  SB_REQUIRE(a && b, "NULL pointer argument");
  SB_REQUIRE(2 * static_cast<int64_t>(r) * (k + n) < (int64_t(1) << 31), "LoRA factors too large");
  const int64_t total = 2 * static_cast<int64_t>(r) * (k + n);
  const int64_t blocks = (total + 255) / 256;
  const int grid = static_cast<int>(blocks < 4096 ? blocks : 4096);
  sb::lora::prepare_kernel<<<grid, 256, 0, sb::as_stream(stream)>>>(
      a, a_dtype, b, b_dtype, r, k, n, reinterpret_cast<__half*>(a16), reinterpret_cast<__half*>(at16),
      reinterpret_cast<__half*>(b16), reinterpret_cast<__half*>(bt16));
  sb::count_launch();
  return sb::check_launch("lora_prepare_kernel");
}

int sb_lora_prepare_pair(const void* a1, const void* a2, int a_dtype, const void* b1, const void* b2,
                         int b_dtype, int r, int64_t k, int64_t n, uint16_t* a_cat, uint16_t* at_cat,
                         uint16_t* b_bd, uint16_t* bt_bd, void* stream) {
  SB_REQUIRE(r > 0 && k > 0 && n > 0, "expected positive sizes");
  SB_REQUIRE((a_dtype == SB_F16 || a_dtype == SB_F32) && (b_dtype == SB_F16 || b_dtype == SB_F32), "bad dtype");
  SB_REQUIRE(a1 && a2 && b1 && b2 && a_cat && at_cat && b_bd && bt_bd, "NULL pointer argument");
  const int64_t total = 4 * static_cast<int64_t>(r) * k + 8 * n * static_cast<int64_t>(r);
  SB_REQUIRE(total < (int64_t(1) << 31), "LoRA factors too large");
  const int64_t blocks = (total + 255) / 256;
  const int grid = static_cast<int>(blocks < 4096 ? blocks : 4096);
  sb::lora::pair_prepare_kernel<<<grid, 256, 0, sb::as_stream(stream)>>>(
      a1, a2, a_dtype, b1, b2, b_dtype, r, k, n, reinterpret_cast<__half*>(a_cat), reinterpret_cast<__half*>(at_cat),
      reinterpret_cast<__half*>(b_bd), reinterpret_cast<__half*>(bt_bd));
  sb::count_launch();
  return sb::check_launch("lora_pair_prepare_kernel");
}

}  // extern "C"
