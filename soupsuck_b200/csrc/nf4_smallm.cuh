// Small-M NF4 linear (M <= 16 activation rows): forward Y = X . deq(W)^T and dX = dY . deq(W).
//
// With at most 16 rows the product is bound by reading the packed weight
// (0.5 byte per weight), not by arithmetic, so this path drops the tcgen05
// pipeline (whose 128-row tiles would be almost empty) for a streaming design:
// every CTA owns 256 output columns and a slice of the reduction; per 64-wide
// step its 256 threads each decode one (row, 64-block) of the weight into a
// 128B-swizzled shared tile (the exact table decode of the tcgen05 kernel:
// fp16_rn(NF4[i] * scale), bit-identical to the reference's decoder), and the 8
// warps multiply it with the activation tile on mma.sync m16n8k16 (fp32
// accumulate).  Packed bytes and activation chunks stream in with cp.async,
// kAhead steps ahead of the decode (kStages-deep shared rings; every thread reads
// back only the packed bytes it copied itself), the absmax byte and absmax2 value
// two steps ahead in registers; decoded tiles are double-buffered with one barrier
// per step.  Reduction slices write fp32 partials; a second kernel sums them in a
// fixed order and adds bias and the LoRA term.
//
//   forward: output column c = weight row, reduction = k_in; step tile = 256 rows x 64 k.
//   dX:      output column c = k_in index, reduction = n_out; step tile = 64 weight rows
//            x 256 columns, stored as four 64-column panels.
#pragma once

#include "common.cuh"
#include "gemm_sm100.cuh"
#include "lora_mma.cuh"

namespace sb {
namespace smallm {

constexpr int kCols = 256;     // output columns per CTA
constexpr int kStep = 64;      // reduction elements per step
constexpr int kRows = 16;      // activation rows (M <= 16)
constexpr int kStages = 4, kAhead = kStages - 2;  // see the buffer-reuse argument in the kernel
constexpr int kWTile = kCols * kStep * 2;   // 32 KB decoded weight tile (double-buffered)
constexpr int kRawTile = kCols * kStep / 2; // 8 KB packed bytes per step
constexpr int kATile = kRows * kStep * 2;   // 2 KB activation tile
constexpr int kRawOff = 2 * kWTile;
constexpr int kAOff = kRawOff + kStages * kRawTile;
constexpr int kCodeOff = kAOff + kStages * kATile;
constexpr int kSmem = kCodeOff + 1024 + 1024;  // + code2 table + alignment

struct Args {
  const __half* act;       // [M, red] row-major
  int M;
  int64_t red, width;      // reduction length, output columns
  const uint8_t* packed;
  const uint8_t* qabs;
  const float* absmax2;
  const float* code2;
  const float* offset;
  int64_t n_out, k_in;     // weight shape
  int steps_per_split;
  float* partial;          // [splits][16][width]
};

template <bool DX>
__global__ void __launch_bounds__(256, 2) nf4_smallm_kernel(const Args a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* code2_s = reinterpret_cast<float*>(smem + kCodeOff);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t c0 = static_cast<int64_t>(blockIdx.x) * kCols;
  const int64_t total_steps = (a.red + kStep - 1) / kStep;
  const int64_t s0 = static_cast<int64_t>(blockIdx.y) * a.steps_per_split;
  int64_t s1 = s0 + a.steps_per_split;
  if (s1 > total_steps) s1 = total_steps;
  for (int i = tid; i < 256; i += blockDim.x) code2_s[i] = __ldg(a.code2 + i);
  const float off = __ldg(a.offset);
  const int64_t bpr = a.k_in / 64;
  const int64_t row_bytes = a.k_in / 2;

  // This thread's decode task: one (weight row, 64-block) per step.  Forward: row
  // c0 + tid, block s (the pointers advance by one block per step); dX: row
  // s * 64 + tid % 64, block (c0 + 64 * (tid / 64)) / 64 (they advance by 64 rows).
  // Offsets inside the weight fit 32 bits (checked by the host).
  const uint8_t* pk;
  const uint8_t* qk;
  uint32_t pk_step, qk_step;
  int64_t row_first;       // weight row of step s0 for this thread
  bool col_ok;
  if constexpr (!DX) {
    row_first = c0 + tid;
    col_ok = row_first < a.n_out;
    pk = a.packed + static_cast<uint32_t>(row_first * row_bytes + s0 * (kStep / 2));
    qk = a.qabs + static_cast<uint32_t>(row_first * bpr + s0);
    pk_step = kStep / 2;
    qk_step = 1;
  } else {
    row_first = s0 * kStep + (tid & 63);
    const int64_t col = c0 + 64 * (tid >> 6);
    col_ok = col < a.k_in;
    pk = a.packed + static_cast<uint32_t>(row_first * row_bytes + col / 2);
    qk = a.qabs + static_cast<uint32_t>(row_first * bpr + col / 64);
    pk_step = static_cast<uint32_t>(kStep * row_bytes);
    qk_step = static_cast<uint32_t>(kStep * bpr);
  }
  auto valid_at = [&](int64_t s) -> bool {
    if constexpr (!DX) return col_ok;
    else return col_ok && row_first + (s - s0) * kStep < a.n_out;
  };
  // Issue the cp.async copies of step s: this thread's 32 packed bytes, and for
  // threads 0..127 one 16-byte activation chunk (zero-filled outside the operands).
  const int ar = tid >> 3, ac = tid & 7;
  auto issue = [&](int64_t s) {
    const int st = static_cast<int>((s - s0) % kStages);
    const bool ok = valid_at(s);
    const uint8_t* src = ok ? pk + static_cast<uint32_t>(s - s0) * pk_step : a.packed;
    const uint32_t dst = smem_addr(smem + kRawOff + st * kRawTile + tid * 32);
    lora::cp_async16(dst, src, ok);
    lora::cp_async16(dst + 16, ok ? src + 16 : src, ok);
    if (tid < kRows * 8) {
      const int64_t col = s * kStep + ac * 8;
      const bool aok = ar < a.M && col < a.red;
      const __half* asrc = aok ? a.act + ar * a.red + col : a.act;
      lora::cp_async16(smem_addr(smem + kAOff + st * kATile + ar * 128 + ((ac ^ (ar & 7)) << 4)), asrc, aok);
    }
  };
  // Scale inputs of step s (absmax byte, absmax2 value), kept two steps ahead in registers.
  const uint32_t q_base = static_cast<uint32_t>(qk - a.qabs);
  auto scale_in = [&](int64_t s, uint32_t& q, float& a2) {
    if (s < s1 && valid_at(s)) {
      const uint32_t blk = q_base + static_cast<uint32_t>(s - s0) * qk_step;
      q = __ldg(a.qabs + blk);
      a2 = __ldg(a.absmax2 + (blk >> 8));
    } else {
      q = 0;
      a2 = 0.0f;
    }
  };

  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.0f;

  // Prologue: steps s0 .. s0 + kAhead - 1 in flight (one commit group per step, empty
  // groups past the end keep the group count uniform for wait_group).
  for (int j = 0; j < kAhead; ++j) {
    if (s0 + j < s1) issue(s0 + j);
    lora::cp_async_commit();
  }
  uint32_t q0, q1;
  float a20, a21;
  scale_in(s0, q0, a20);
  scale_in(s0 + 1, q1, a21);
  const int mat = lane >> 3, r8 = lane & 7;
  for (int64_t s = s0; s < s1; ++s) {
    // Step s + kAhead reuses ring slot (s + kAhead - s0) % kStages, last read by the
    // MMAs of step s + kAhead - kStages = s - 2, which finished before the barrier
    // of step s - 1: safe to overwrite here, before this step's barrier.
    if (s + kAhead < s1) issue(s + kAhead);
    lora::cp_async_commit();
    lora::cp_async_wait<kAhead>();   // this thread's copies of step s have landed
    const int st = static_cast<int>((s - s0) % kStages);
    const int buf = static_cast<int>((s - s0) & 1);
    uint8_t* wt = smem + buf * kWTile;
    const bool valid = valid_at(s);
    const uint4 w0 = *reinterpret_cast<const uint4*>(smem + kRawOff + st * kRawTile + tid * 32);
    const uint4 w1 = *reinterpret_cast<const uint4*>(smem + kRawOff + st * kRawTile + tid * 32 + 16);
    const float scale = valid ? __fadd_rn(__fmul_rn(code2_s[q0], a20), off) : 0.0f;
    q0 = q1;
    a20 = a21;
    scale_in(s + 2, q1, a21);
    if constexpr (!DX) {
      gemm::nf4_decode_words(w0, w1, wt + tid * 128, tid, scale, valid);
    } else {
      const int row = tid & 63, j = tid >> 6;
      gemm::nf4_decode_words(w0, w1, wt + j * 8192 + row * 128, row, scale, valid);
    }
    __syncthreads();  // decoded tile and activation tile of step s are complete for every warp
    const uint32_t wts = smem_addr(wt), ats = smem_addr(smem + kAOff + st * kATile);
#pragma unroll
    for (int kk = 0; kk < kStep / 16; ++kk) {
      uint32_t af[4];
      {
        const int r = r8 + 8 * (mat & 1), c = 2 * kk + (mat >> 1);
        lora::ldsm_x4(ats + r * 128 + ((c ^ (r & 7)) << 4), af);
      }
#pragma unroll
      for (int pr = 0; pr < 2; ++pr) {
        uint32_t bf[4];
        if constexpr (!DX) {
          // rows = weight rows (output columns), 16-byte chunks along k
          const int n = warp * 32 + pr * 16 + r8 + 8 * (mat >> 1);
          const int c = 2 * kk + (mat & 1);
          lora::ldsm_x4(wts + n * 128 + ((c ^ (n & 7)) << 4), bf);
        } else {
          // rows = weight rows (reduction), columns = output columns in 64-wide panels
          const int k = 16 * kk + r8 + 8 * (mat & 1);
          const int col = warp * 32 + pr * 16 + 8 * (mat >> 1);
          const int j = col >> 6, c = (col & 63) >> 3;
          lora::ldsm_x4_trans(wts + j * 8192 + k * 128 + ((c ^ (k & 7)) << 4), bf);
        }
        lora::mma16816(acc[2 * pr], af, bf[0], bf[1]);
        lora::mma16816(acc[2 * pr + 1], af, bf[2], bf[3]);
      }
    }
  }
  lora::cp_async_wait<0>();
  // Partial sums: D fragment rows m = g, g + 8; columns 2t, 2t + 1 of each n8 tile.
  const int g = lane >> 2, t = lane & 3;
  float* out = a.partial + static_cast<int64_t>(blockIdx.y) * kRows * a.width;
#pragma unroll
  for (int nt = 0; nt < 4; ++nt) {
    const int64_t col = c0 + warp * 32 + nt * 8 + 2 * t;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int m = g + 8 * h;
      if (m < a.M) {
        if (col < a.width) out[m * a.width + col] = acc[nt][2 * h];
        if (col + 1 < a.width) out[m * a.width + col + 1] = acc[nt][2 * h + 1];
      }
    }
  }
}

// out[m, c] = fp16(sum_s partial[s][m][c] + bias[c] + sum_j la[m][j] lb[c][j]).
__global__ void nf4_smallm_finalize(const float* __restrict__ partial, int splits, int M, int64_t width,
                                    const __half* __restrict__ bias, const __half* __restrict__ la,
                                    const __half* __restrict__ lb, int r, __half* __restrict__ out) {
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= static_cast<int64_t>(M) * width) return;
  const int m = static_cast<int>(idx / width);
  const int64_t c = idx % width;
  float v = 0.0f;
  for (int s = 0; s < splits; ++s) v += partial[(static_cast<int64_t>(s) * kRows + m) * width + c];
  if (r > 0) {
    float l = 0.0f;
    for (int j = 0; j < r; ++j) l = fmaf(__half2float(la[m * r + j]), __half2float(lb[c * r + j]), l);
    v += l;
  }
  if (bias) v = __fadd_rn(v, __half2float(bias[c]));
  out[idx] = __float2half_rn(v);
}

struct Plan {
  int64_t col_tiles, steps, splits, steps_per_split;
  size_t workspace;
};

inline Plan plan(int64_t red, int64_t width) {
  Plan p{};
  p.col_tiles = (width + kCols - 1) / kCols;
  p.steps = (red + kStep - 1) / kStep;
  // Two CTAs per SM in total (short slices win: parallelism matters more here than
  // the per-CTA prologue).
  int64_t splits = (2 * device_sm_count() + p.col_tiles - 1) / p.col_tiles;
  if (splits > p.steps) splits = p.steps;
  if (splits < 1) splits = 1;
  p.steps_per_split = (p.steps + splits - 1) / splits;
  p.splits = (p.steps + p.steps_per_split - 1) / p.steps_per_split;
  p.workspace = static_cast<size_t>(p.splits) * kRows * width * sizeof(float);
  return p;
}

inline bool eligible(int64_t m, int64_t n_out, int64_t k_in, const void* act, const void* packed) {
  return m >= 1 && m <= kRows && k_in % 64 == 0 && aligned(act, 16) && aligned(packed, 16);
}

inline int run(bool dx, const uint16_t* act, int64_t m, const sb_nf4_weight& w, const uint16_t* bias,
               const uint16_t* lora_a, const uint16_t* lora_b, int r, uint16_t* out, void* workspace,
               size_t workspace_bytes, cudaStream_t st) {
  const int64_t red = dx ? w.n_out : w.k_in, width = dx ? w.k_in : w.n_out;
  if (dx && red % 8 != 0) return fail(SB_EINVAL, "small-M dX needs n_out % 8 == 0");
  const Plan pl = plan(red, width);
  if (!workspace || workspace_bytes < pl.workspace) return fail(SB_EWORKSPACE, "small-M NF4 workspace too small");
  static std::mutex mu;
  static bool configured[2][64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lock(mu);
    if (dev >= 0 && dev < 64 && !configured[dx][dev]) {
      cudaError_t e = dx ? cudaFuncSetAttribute(nf4_smallm_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem)
                         : cudaFuncSetAttribute(nf4_smallm_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
      if (e != cudaSuccess) return fail(SB_ECUDA, std::string("small-M smem attribute: ") + cudaGetErrorString(e));
      configured[dx][dev] = true;
    }
  }
  Args a{};
  a.act = reinterpret_cast<const __half*>(act);
  a.M = static_cast<int>(m);
  a.red = red;
  a.width = width;
  a.packed = w.packed;
  a.qabs = w.qabs;
  a.absmax2 = w.absmax2;
  a.code2 = w.code2;
  a.offset = w.offset;
  a.n_out = w.n_out;
  a.k_in = w.k_in;
  a.steps_per_split = static_cast<int>(pl.steps_per_split);
  a.partial = static_cast<float*>(workspace);
  dim3 grid(static_cast<unsigned>(pl.col_tiles), static_cast<unsigned>(pl.splits));
  if (dx) nf4_smallm_kernel<true><<<grid, 256, kSmem, st>>>(a);
  else nf4_smallm_kernel<false><<<grid, 256, kSmem, st>>>(a);
  count_launch();
  if (int rc = check_launch("nf4_smallm_kernel")) return rc;
  const int64_t total = m * width;
  nf4_smallm_finalize<<<static_cast<unsigned>((total + 255) / 256), 256, 0, st>>>(
      a.partial, static_cast<int>(pl.splits), static_cast<int>(m), width, reinterpret_cast<const __half*>(bias),
      reinterpret_cast<const __half*>(lora_a), reinterpret_cast<const __half*>(lora_b), r,
      reinterpret_cast<__half*>(out));
  count_launch();
  return check_launch("nf4_smallm_finalize");
}

}  // namespace smallm
}  // namespace sb
