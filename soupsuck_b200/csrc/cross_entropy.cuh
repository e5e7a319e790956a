// Fused linear cross-entropy over a frozen fp16 head (vocabulary chunks, online softmax).
//
// Reference: _FrozenLinearCrossEntropy (solution/kernels/cross_entropy.py:133-211).
//
// Forward: one persistent tcgen05 GEMM (hidden . W^T, 128 x 256 tiles) whose
// epilogue rounds each logit to fp16 and folds it into per-row tile statistics
// (max, first argmax, sum exp, sum exp*z, target logit).  Logits never reach
// memory; the statistics ([vocab tiles, rows]) are merged per row by
// ce_merge_kernel into lse = m + log s, entropy = lse - t/s, loss = lse - z_t.
//
// Backward: the labelled rows are compacted on the device (no host round trip;
// the reference's torch.nonzero sync, :173-188, disappears), then per vocabulary
// chunk of 8192:
//   dz  = fp16((exp(z - lse) - onehot) * g / gain)   tcgen05 GEMM + kCeDz epilogue,
//                                                   kept in L2 (rows x 8192 fp16)
//   acc += dz . W_chunk                               tcgen05 GEMM, fp32 accumulate
// and finally dhidden[row] = acc * gain (ignored rows exact zero), gain =
// max(|g|, 1e-30) / 1024 as in :192.
#pragma once

#include "common.cuh"
#include "gemm_host.cuh"

namespace sb {
namespace ce {

constexpr int kFwdBN = 256;
constexpr int kBwdChunk = 8192;        // smallest backward vocabulary chunk
constexpr int kBwdChunkMax = 32768;    // largest
constexpr int64_t kBwdDzBudget = int64_t(256) << 20;  // bytes of the fp16 dZ chunk [t, chunk]

// Backward vocabulary chunk for t rows: the largest power of two in
// [kBwdChunk, kBwdChunkMax] whose dZ chunk fits the budget (32768 at t = 3300,
// 8192 from t = 16384 on); larger chunks mean fewer, fuller GEMM launches
// (CE fwd+bwd at t = 3300: 4.83 ms with 8192, 4.45 ms with 32768).
inline int64_t bwd_chunk(int64_t t, int64_t v) {
  int64_t c = kBwdChunkMax;
  while (c > kBwdChunk && static_cast<int64_t>(c) * 2 * (t > 0 ? t : 1) > kBwdDzBudget) c /= 2;
  return v < c ? ((v + 63) / 64) * 64 : c;
}

__device__ unsigned long long g_bad_targets = 0;

__global__ void check_targets_kernel(const int64_t* __restrict__ t, int64_t n, int64_t v, int64_t ignore) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  unsigned long long bad = 0;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
    const int64_t x = t[i];
    if (x != ignore && (x < 0 || x >= v)) ++bad;
  }
  if (bad) atomicAdd(&g_bad_targets, bad);
}

__global__ void ce_merge_kernel(const float* __restrict__ stats, const int* __restrict__ args,
                                int64_t ld, int n_tiles, const int64_t* __restrict__ targets,
                                int64_t ignore, int64_t rows, float* __restrict__ loss,
                                float* __restrict__ entropy, int64_t* __restrict__ argmax,
                                float* __restrict__ lse_out, float* __restrict__ row_max) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= rows) return;
  float M = -INFINITY, S = 0.0f, T = 0.0f, tz = 0.0f;
  int arg = 0;
  for (int nt = 0; nt < n_tiles; ++nt) {
    const float* b = stats + static_cast<int64_t>(nt) * 4 * ld + i;
    const float mt = b[0], st = b[ld], tt = b[2 * ld];
    tz += b[3 * ld];
    if (mt > M) {
      const float r = M == -INFINITY ? 0.0f : __expf(M - mt);
      S = fmaf(S, r, st);
      T = fmaf(T, r, tt);
      M = mt;
      arg = args[static_cast<int64_t>(nt) * ld + i];
    } else if (mt != -INFINITY) {
      const float r = __expf(mt - M);
      S = fmaf(st, r, S);
      T = fmaf(tt, r, T);
    }
  }
  const float l = M + logf(S);
  lse_out[i] = l;
  entropy[i] = l - T / S;
  const int64_t tg = targets[i];
  loss[i] = tg != ignore ? l - tz : 0.0f;
  argmax[i] = arg;
  if (row_max) row_max[i] = M;
}

// The same merge spread over a CTA: 32 consecutive rows (one per lane) and 16
// warps; warp w folds tiles w, w + 16, ... in increasing order (loads coalesced
// across the rows), then warp 0 merges the 16 partial results in warp order.
// On equal maxima the smaller column wins, as in the tile-order scan above, so
// the first argmax is kept; the order is fixed, so results are deterministic.
constexpr int kMergeWarps = 16;

__device__ __forceinline__ void merge_stat(float& M, float& S, float& T, int& A, float m2, float s2, float t2,
                                           int a2) {
  if (m2 == -INFINITY) return;
  if (M == -INFINITY) {
    M = m2; S = s2; T = t2; A = a2;
    return;
  }
  if (m2 > M) {
    const float r = __expf(M - m2);
    S = fmaf(S, r, s2);
    T = fmaf(T, r, t2);
    M = m2;
    A = a2;
  } else {
    const float r = __expf(m2 - M);
    S = fmaf(s2, r, S);
    T = fmaf(t2, r, T);
    if (m2 == M && a2 < A) A = a2;
  }
}

__global__ void __launch_bounds__(32 * kMergeWarps) ce_merge2_kernel(
    const float* __restrict__ stats, const int* __restrict__ args, int64_t ld, int n_tiles,
    const int64_t* __restrict__ targets, int64_t ignore, int64_t rows, float* __restrict__ loss,
    float* __restrict__ entropy, int64_t* __restrict__ argmax, float* __restrict__ lse_out,
    float* __restrict__ row_max) {
  __shared__ float part[kMergeWarps][4][32];
  __shared__ int part_arg[kMergeWarps][32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t i = static_cast<int64_t>(blockIdx.x) * 32 + lane;
  const bool ok = i < rows;
  float M = -INFINITY, S = 0.0f, T = 0.0f, tz = 0.0f;
  int A = 0x7fffffff;
  if (ok) {
    for (int nt = warp; nt < n_tiles; nt += kMergeWarps) {
      const float* b = stats + static_cast<int64_t>(nt) * 4 * ld + i;
      const float mt = b[0], st = b[ld], tt = b[2 * ld];
      tz += b[3 * ld];
      merge_stat(M, S, T, A, mt, st, tt, args[static_cast<int64_t>(nt) * ld + i]);
    }
  }
  part[warp][0][lane] = M;
  part[warp][1][lane] = S;
  part[warp][2][lane] = T;
  part[warp][3][lane] = tz;
  part_arg[warp][lane] = A;
  __syncthreads();
  if (warp != 0 || !ok) return;
  M = part[0][0][lane]; S = part[0][1][lane]; T = part[0][2][lane]; tz = part[0][3][lane];
  A = part_arg[0][lane];
#pragma unroll 1
  for (int w = 1; w < kMergeWarps; ++w) {
    merge_stat(M, S, T, A, part[w][0][lane], part[w][1][lane], part[w][2][lane], part_arg[w][lane]);
    tz += part[w][3][lane];
  }
  const float l = M + logf(S);
  lse_out[i] = l;
  entropy[i] = l - T / S;
  const int64_t tg = targets[i];
  loss[i] = tg != ignore ? l - tz : 0.0f;
  argmax[i] = M == -INFINITY ? 0 : A;
  if (row_max) row_max[i] = M;
}

// Single-block stream compaction of labelled rows (deterministic order).
__global__ void __launch_bounds__(1024) ce_compact_kernel(const int64_t* __restrict__ targets,
                                                          int64_t n, int64_t ignore,
                                                          int* __restrict__ idx, int* __restrict__ inv,
                                                          int* __restrict__ count) {
  __shared__ int warp_tot[32];
  __shared__ int base_s;
  if (threadIdx.x == 0) base_s = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int64_t start = 0; start < n; start += 1024) {
    const int64_t i = start + threadIdx.x;
    const int valid = (i < n && targets[i] != ignore) ? 1 : 0;
    const unsigned ballot = __ballot_sync(0xffffffffu, valid);
    const int pre = __popc(ballot & ((1u << lane) - 1u));
    if (lane == 0) warp_tot[warp] = __popc(ballot);
    __syncthreads();
    int wbase = 0, total = 0;
    for (int w = 0; w < 32; ++w) {
      if (w < warp) wbase += warp_tot[w];
      total += warp_tot[w];
    }
    const int pos = base_s + wbase + pre;
    if (i < n) {
      if (valid) {
        idx[pos] = static_cast<int>(i);
        inv[i] = pos;
      } else {
        inv[i] = -1;
      }
    }
    __syncthreads();
    if (threadIdx.x == 0) base_s += total;
    __syncthreads();
  }
  if (threadIdx.x == 0) *count = base_s;
}

__global__ void ce_gather_kernel(const __half* __restrict__ hidden, int64_t h,
                                 const int64_t* __restrict__ targets, const float* __restrict__ lse,
                                 const float* __restrict__ grad, const int* __restrict__ idx,
                                 const int* __restrict__ count, __half* __restrict__ hc,
                                 int64_t* __restrict__ tc, float* __restrict__ lc,
                                 float* __restrict__ gc, float* __restrict__ gain) {
  const int64_t i = blockIdx.x;
  if (i >= *count) return;
  const int64_t src = idx[i];
  if (threadIdx.x == 0) {
    tc[i] = targets[src];
    lc[i] = lse[src];
    const float g = grad[src];
    gc[i] = g;
    gain[i] = __fdiv_rn(fmaxf(fabsf(g), 1e-30f), 1024.0f);
  }
  const uint4* s = reinterpret_cast<const uint4*>(hidden + src * h);
  uint4* d = reinterpret_cast<uint4*>(hc + i * h);
  for (int64_t c = threadIdx.x; c < h / 8; c += blockDim.x) d[c] = s[c];
}

// dHidden[row] = gain * (acc + acc2)[compacted row]: the two halves of the split
// dZ . W_chunk reduction are added here, in a fixed order.
__global__ void ce_finalize_kernel(const float* __restrict__ acc, const float* __restrict__ acc2,
                                   const float* __restrict__ gain, const int* __restrict__ inv, int64_t h,
                                   void* __restrict__ out, int odt) {
  const int64_t row = blockIdx.x;
  const int c = inv[row];
  for (int64_t col = threadIdx.x; col < h; col += blockDim.x) {
    const int64_t at = static_cast<int64_t>(c) * h + col;
    const float v = c < 0 ? 0.0f : (acc[at] + acc2[at]) * gain[c];
    st_from_f32(out, odt, row * h + col, v);
  }
}

inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

struct BwdLayout {
  size_t idx, inv, count, hc, tc, lc, gc, gain, acc, acc2, dz, total;
};

inline BwdLayout bwd_layout(int64_t t, int64_t h, int64_t v) {
  BwdLayout L{};
  size_t o = 0;
  auto take = [&](size_t bytes) { size_t at = o; o = align256(o + bytes); return at; };
  const int64_t chunk = bwd_chunk(t, v);
  L.idx = take(t * 4);
  L.inv = take(t * 4);
  L.count = take(16);
  L.hc = take(t * h * 2);
  L.tc = take(t * 8);
  L.lc = take(t * 4);
  L.gc = take(t * 4);
  L.gain = take(t * 4);
  L.acc = take(t * h * 4);
  L.acc2 = take(t * h * 4);
  L.dz = take(t * chunk * 2);
  L.total = o;
  return L;
}

}  // namespace ce
}  // namespace sb

extern "C" {

size_t sb_ce_forward_workspace_bytes(int64_t t, int64_t h, int64_t v) {
  (void)h;
  if (t <= 0 || v <= 0) return 0;
  const int64_t n_tiles = (v + sb::ce::kFwdBN - 1) / sb::ce::kFwdBN;
  return sb::ce::align256(static_cast<size_t>(n_tiles) * t * 4 * sizeof(float)) +
         sb::ce::align256(static_cast<size_t>(n_tiles) * t * sizeof(int));
}

size_t sb_ce_backward_workspace_bytes(int64_t t, int64_t h, int64_t v) {
  if (t <= 0 || v <= 0 || h <= 0) return 0;
  return sb::ce::bwd_layout(t, h, v).total;
}

int sb_ce_check_targets(const int64_t* targets, int64_t t, int64_t v, int64_t ignore_index,
                        int64_t* bad, void* stream) {
  SB_REQUIRE(bad != nullptr, "NULL bad");
  *bad = 0;
  if (t <= 0) return SB_OK;
  SB_REQUIRE(targets != nullptr, "NULL targets");
  cudaStream_t st = sb::as_stream(stream);
  void* dptr = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&dptr, sb::ce::g_bad_targets);
  if (e == cudaSuccess) e = cudaMemsetAsync(dptr, 0, sizeof(unsigned long long), st);
  if (e != cudaSuccess) return sb::fail(SB_ECUDA, cudaGetErrorString(e));
  const int64_t blocks = (t + 255) / 256;
  sb::ce::check_targets_kernel<<<static_cast<unsigned>(blocks < 1024 ? blocks : 1024), 256, 0, st>>>(targets, t, v, ignore_index);
  sb::count_launch();
  if (int rc = sb::check_launch("check_targets_kernel")) return rc;
  unsigned long long host = 0;
  e = cudaMemcpyAsync(&host, dptr, sizeof(host), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return sb::fail(SB_ECUDA, cudaGetErrorString(e));
  *bad = static_cast<int64_t>(host);
  return SB_OK;
}

static int ce_forward_impl(const uint16_t* hidden, int64_t t, int64_t h, const uint16_t* weight, int64_t v,
                           const int64_t* targets, int64_t ignore_index, float* loss, float* entropy,
                           int64_t* argmax, float* lse, float* row_max, void* workspace,
                           size_t workspace_bytes, void* stream) {
  using namespace sb::gemm;
  SB_REQUIRE(t >= 0 && h > 0 && v > 0, "expected t >= 0, h > 0, v > 0");
  if (t == 0) return SB_OK;
  SB_REQUIRE(hidden && weight && targets && loss && entropy && argmax && lse, "NULL pointer argument");
  SB_REQUIRE(h % 8 == 0, "hidden size must be a multiple of 8 (pad with zeros)");
  SB_REQUIRE(t <= 0x7fffffff && v <= 0x7fffffff && h <= 0x7fffffff, "size out of range");
  const size_t need = sb_ce_forward_workspace_bytes(t, h, v);
  if (!workspace || workspace_bytes < need) return sb::fail(SB_EWORKSPACE, "CE forward workspace too small");
  cudaStream_t st = sb::as_stream(stream);
  const int n_tiles = static_cast<int>((v + sb::ce::kFwdBN - 1) / sb::ce::kFwdBN);
  float* stats = static_cast<float*>(workspace);
  int* args = reinterpret_cast<int*>(static_cast<uint8_t*>(workspace) +
                                     sb::ce::align256(static_cast<size_t>(n_tiles) * t * 4 * sizeof(float)));
  CUtensorMap ta, tb;
  int rc = make_map(&ta, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, hidden, h, t, h * 2, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = make_map(&tb, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, weight, h, v, h * 2, 64, sb::ce::kFwdBN, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  Params p{};
  p.M = static_cast<int>(t);
  p.N = static_cast<int>(v);
  p.K = static_cast<int>(h);
  p.m_tiles = static_cast<int>((t + 127) / 128);
  p.n_tiles = n_tiles;
  p.k_blocks = static_cast<int>((h + 63) / 64);
  p.targets = targets;
  p.ignore_index = ignore_index;
  p.stats = stats;
  p.stats_arg = args;
  p.stats_ld = t;
  p.col_offset = 0;
  rc = launch<kDenseK, kCeStats, 1, sb::ce::kFwdBN, 4>(ta, tb, ta, ta, p, st, "ce_logits_stats");
  if (rc) return rc;
  sb::ce::ce_merge2_kernel<<<static_cast<unsigned>((t + 31) / 32), 32 * sb::ce::kMergeWarps, 0, st>>>(
      stats, args, t, n_tiles, targets, ignore_index, t, loss, entropy, argmax, lse, row_max);
  sb::count_launch();
  return sb::check_launch("ce_merge2_kernel");
}

int sb_ce_forward(const uint16_t* hidden, int64_t t, int64_t h, const uint16_t* weight, int64_t v,
                  const int64_t* targets, int64_t ignore_index, float* loss, float* entropy,
                  int64_t* argmax, float* lse, void* workspace, size_t workspace_bytes,
                  void* stream) {
  return ce_forward_impl(hidden, t, h, weight, v, targets, ignore_index, loss, entropy, argmax, lse,
                         nullptr, workspace, workspace_bytes, stream);
}

int sb_ce_forward_shard(const uint16_t* hidden, int64_t t, int64_t h, const uint16_t* weight, int64_t v,
                        const int64_t* targets, int64_t ignore_index, float* loss, float* entropy,
                        int64_t* argmax, float* lse, float* row_max, void* workspace,
                        size_t workspace_bytes, void* stream) {
  SB_REQUIRE(t == 0 || row_max != nullptr, "NULL row_max");
  return ce_forward_impl(hidden, t, h, weight, v, targets, ignore_index, loss, entropy, argmax, lse,
                         row_max, workspace, workspace_bytes, stream);
}

int sb_ce_backward(const uint16_t* hidden, int64_t t, int64_t h, const uint16_t* weight, int64_t v,
                   const int64_t* targets, int64_t ignore_index, const float* lse,
                   const float* grad, void* dhidden, int dh_dtype, void* workspace,
                   size_t workspace_bytes, void* stream) {
  using namespace sb::gemm;
  SB_REQUIRE(t >= 0 && h > 0 && v > 0, "expected t >= 0, h > 0, v > 0");
  SB_REQUIRE(dh_dtype == SB_F16 || dh_dtype == SB_F32, "dhidden dtype must be SB_F16 or SB_F32");
  if (t == 0) return SB_OK;
  SB_REQUIRE(hidden && weight && targets && lse && grad && dhidden, "NULL pointer argument");
  SB_REQUIRE(h % 8 == 0, "hidden size must be a multiple of 8 (pad with zeros)");
  SB_REQUIRE(sb::aligned(hidden, 16) && sb::aligned(weight, 16), "operands must be 16-byte aligned");
  SB_REQUIRE(t <= 0x7fffffff && v <= 0x7fffffff && h <= 0x7fffffff, "size out of range");
  const sb::ce::BwdLayout L = sb::ce::bwd_layout(t, h, v);
  if (!workspace || workspace_bytes < L.total) return sb::fail(SB_EWORKSPACE, "CE backward workspace too small");
  cudaStream_t st = sb::as_stream(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int* idx = reinterpret_cast<int*>(ws + L.idx);
  int* inv = reinterpret_cast<int*>(ws + L.inv);
  int* count = reinterpret_cast<int*>(ws + L.count);
  __half* hc = reinterpret_cast<__half*>(ws + L.hc);
  int64_t* tc = reinterpret_cast<int64_t*>(ws + L.tc);
  float* lc = reinterpret_cast<float*>(ws + L.lc);
  float* gc = reinterpret_cast<float*>(ws + L.gc);
  float* gain = reinterpret_cast<float*>(ws + L.gain);
  float* acc = reinterpret_cast<float*>(ws + L.acc);
  float* acc2 = reinterpret_cast<float*>(ws + L.acc2);
  __half* dz = reinterpret_cast<__half*>(ws + L.dz);
  const int64_t chunk = sb::ce::bwd_chunk(t, v);

  sb::ce::ce_compact_kernel<<<1, 1024, 0, st>>>(targets, t, ignore_index, idx, inv, count);
  sb::count_launch();
  if (int rc = sb::check_launch("ce_compact_kernel")) return rc;
  sb::ce::ce_gather_kernel<<<static_cast<unsigned>(t), 128, 0, st>>>(
      reinterpret_cast<const __half*>(hidden), h, targets, lse, grad, idx, count, hc, tc, lc, gc, gain);
  sb::count_launch();
  if (int rc = sb::check_launch("ce_gather_kernel")) return rc;
  // acc and acc2 are adjacent in the workspace (one clear for both).
  cudaError_t e = cudaMemsetAsync(acc, 0, L.dz - L.acc, st);
  if (e != cudaSuccess) return sb::fail(SB_ECUDA, cudaGetErrorString(e));

  CUtensorMap t_hc, t_dz;
  int rc = make_map(&t_hc, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, hc, h, t, h * 2, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  for (int64_t v0 = 0; v0 < v; v0 += chunk) {
    const int64_t vc = (v - v0) < chunk ? (v - v0) : chunk;
    const uint16_t* wc = weight + v0 * h;
    CUtensorMap t_wk, t_wmn;
    rc = make_map(&t_wk, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, wc, h, vc, h * 2, 64, 256, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    rc = make_map(&t_dz, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, dz, vc, t, chunk * 2, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    rc = make_map(&t_wmn, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, wc, h, vc, h * 2, 64, 64, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    Params p1{};
    p1.M = static_cast<int>(t);
    p1.N = static_cast<int>(vc);
    p1.K = static_cast<int>(h);
    p1.m_tiles = static_cast<int>((t + 127) / 128);
    p1.n_tiles = static_cast<int>((vc + 255) / 256);
    p1.k_blocks = static_cast<int>((h + 63) / 64);
    p1.m_dev = count;
    p1.vec_ok = 1;  // chunk pitch is a multiple of 64 elements
    p1.out = dz;
    p1.ldo = chunk;
    p1.targets = tc;
    p1.ignore_index = ignore_index;
    p1.lse = lc;
    p1.grad = gc;
    p1.gain = gain;
    p1.col_offset = v0;
    rc = launch<kDenseK, kCeDz, 1, 256, 4>(t_hc, t_wk, t_hc, t_hc, p1, st, "ce_logits_dz");
    if (rc) return rc;
    Params p2{};
    p2.M = static_cast<int>(t);
    p2.N = static_cast<int>(h);
    p2.K = static_cast<int>(vc);
    p2.m_tiles = static_cast<int>((t + 127) / 128);
    // 128 x 256 tiles with each tile's reduction split in two halves (the second
    // accumulating into acc2): as many CTAs as 128 x 128 tiles, but UMMAs that
    // read 12 KB of shared memory per 128 cycles instead of 8 KB per 64.
    p2.n_tiles = static_cast<int>((h + 255) / 256);
    p2.ksplit = 2;
    p2.out_split = acc2;
    p2.k_blocks = static_cast<int>((vc + 63) / 64);
    p2.m_dev = count;
    p2.vec_ok = (h % 4 == 0);
    p2.out = acc;
    p2.ldo = h;
    rc = launch<kDenseMN, kAccF32, 1, 256, 4>(t_dz, t_wmn, t_dz, t_dz, p2, st, "ce_dz_weight");
    if (rc) return rc;
  }
  sb::ce::ce_finalize_kernel<<<static_cast<unsigned>(t), 256, 0, st>>>(acc, acc2, gain, inv, h, dhidden, dh_dtype);
  sb::count_launch();
  return sb::check_launch("ce_finalize_kernel");
}

}  // extern "C"
