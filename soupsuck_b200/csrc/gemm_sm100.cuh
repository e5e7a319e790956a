// Warp-specialised persistent tcgen05 GEMM for sm_100a with an in-SMEM NF4 decoder.
//
//   D[M, N] = A[M, K] . B[N, K]^T  (+ LA[M, r] . LB[N, r]^T)   fp16 x fp16 -> fp32 (TMEM)
//
// B comes from one of four sources:
//   kNF4Fwd   packed NF4 weight W[N, K] (forward Y = X . deq(W)^T): K-major operand;
//   kNF4Dx    packed NF4 weight W[K_red, N_out] (dX = dY . deq(W)):  MN-major operand;
//   kDenseK   fp16 B[N, K] row-major (CE logits = hidden . W_head^T);
//   kDenseMN  fp16 B[K, N] row-major (CE dX = dZ . W_head_chunk).
// For the NF4 modes the producer TMA-loads the packed bytes (no swizzle) and
// decoder warps expand them, 64 elements per thread, into the 128B-swizzled fp16
// layout the UMMA descriptor expects.  The decoded values are bit-identical to
// the standalone decoder (reference solution/kernels/nf4.py:41-59): per 64-block
// the thread builds the 16-entry table fp16_rn(NF4[i] * scale) with separate
// fp32 multiply/add, then expands 8 nibbles at a time with byte permutes.
//
// Roles (one CTA per SM; > 114 KB of shared memory so no two tcgen05 kernels
// share an SM and TMEM allocation never waits on another CTA):
//   warp 0       TMA producer (A tiles, packed B or dense B, LoRA factors)
//   warp 1       TMEM allocator + single-thread UMMA issuer
//   warps 4..7   epilogue (TMEM lanes 32*(warp%4) ..), double-buffered accumulators
//   warps 8..15  NF4 decoders, two groups of 4 warps alternating k-steps
// Every mbarrier wait is bounded (common.cuh); on expiry the CTA records an error
// word, stops issuing, waits (bounded) for its in-flight TMA and UMMA work and
// frees TMEM before returning.
//
// The multiple-of-64 k_in requirement of the NF4 modes keeps each 64-element
// quantization block inside one weight row, so a tile's block index is
// row * (k_in / 64) + column / 64; absmax2 is indexed by the global block id.
#pragma once

#include "common.cuh"
#include "nf4_dequant.cuh"

namespace sb {
namespace gemm {

enum BMode : int { kNF4Fwd = 0, kNF4Dx = 1, kDenseK = 2, kDenseMN = 3 };
enum EMode : int { kStoreF16 = 0, kStoreF32 = 1, kAccF32 = 2, kCeStats = 3, kCeDz = 4,
                   // 2-SM pair kernel only (gemm_pair.cuh): the Qwen2 MLP's SwiGLU fused into
                   // the gate/up forward and into the down projection's dX
                   kSwiGLUFwd = 5, kSwiGLUBwd = 6 };

constexpr int kBK = 64;        // reduction elements per pipeline stage (one 128 B swizzle row)
constexpr int kTileRows = 128; // rows per UMMA (M = 128, cta_group::1)

struct Params {
  int M, N, K;            // logical problem: D[M, N], reduction K
  int m_tiles, n_tiles, k_blocks;
  int lora_r;             // 0, 16, 32 or 64: extra LoRA step(s) after the main loop
  const int* m_dev;       // optional runtime row count (CE backward compaction)
  int vec_ok;             // output rows are 16-byte aligned
  int store_tma;          // 2-SM pair kernel: fp16 output written by bulk tensor stores
  int streamk;            // 1: stream-K schedule (equal k-iteration shares per CTA)
  int nfast;              // 2-SM pair kernel: tiles numbered n-fastest (see tile_m / tile_n)
  int ksplit;             // whole-tile schedule: 2 splits every tile's reduction in two halves,
                          // the second half accumulating into out_split (0 or 1: no split)
  void* out_split;        // kAccF32 / kStoreF32 output of the second half
  float* partials;        // stream-K: [grid, 2, MSUB*128, BN] fp32 partial tiles
  int* counters;          // stream-K: [tiles] arrival counters, zero before launch
  // NF4 weight
  const uint8_t* packed;   // packed codes (read directly by the 2-SM pair kernel's decoders)
  const uint8_t* qabs;
  const float* absmax2;
  const float* code2;
  const float* offset;
  int64_t w_rows;          // n_out of the weight
  int64_t w_cols;          // k_in of the weight
  // A second NF4 weight of the same shape (2-SM pair kernel, WSEL != 0):
  //   WSEL 1, gate/up forward: a pair tile's rank-1 CTA decodes this weight's rows
  //           [nt*128, nt*128 + 128) while rank 0 decodes the first weight's;
  //   WSEL 2, concatenated dX: reduction blocks >= k_split decode this weight.
  const uint8_t* packed2;
  const uint8_t* qabs2;
  const float* absmax2_2;
  const float* code2_2;
  const float* offset2;
  int k_split;
  // kSwiGLUBwd: the MLP's [M, 2N] gate (columns [0, N)) / up ([N, 2N)) buffer.
  const __half* gu;
  int64_t ld_gu;
  // epilogue
  void* out;
  int64_t ldo;
  const __half* bias;
  // cross-entropy epilogues
  const int64_t* targets;
  int64_t ignore_index;
  float* stats;            // kCeStats: [n_tiles, M_alloc, 4] partial (max, sumexp, sumexp*z, target z)
  int* stats_arg;          // kCeStats: [n_tiles, M_alloc] first argmax (local column)
  int64_t stats_ld;        // rows of the stats arrays
  const float* lse;        // kCeDz
  const float* grad;       // kCeDz: per-row upstream gradient (compacted)
  const float* gain;       // kCeDz: per-row gain
  int64_t col_offset;      // vocabulary index of column 0 of this launch
};

template <int BMODE, int MSUB, int BN, int STAGES>
struct Cfg {
  static constexpr bool kNF4 = (BMODE == kNF4Fwd || BMODE == kNF4Dx);
  static constexpr bool kBMN = (BMODE == kNF4Dx || BMODE == kDenseMN);
  static constexpr int kABytes = MSUB * kTileRows * kBK * 2;
  static constexpr int kBBytes = BN * kBK * 2;
  static constexpr int kRawBytes = kNF4 ? BN * kBK / 2 : 0;
  static constexpr int kStageBytes = kABytes + kBBytes + kRawBytes;
  static constexpr int kTmemCols = 2 * MSUB * BN;
  static constexpr int kThreads = kNF4 ? 512 : 256;
  static constexpr int kBarrierBytes = 1024 + 1024;  // barriers + the 256-entry code2 table
  static constexpr int kSmemBytes = STAGES * kStageBytes + kBarrierBytes + 1024;  // + align slack
  static_assert(kTmemCols == 128 || kTmemCols == 256 || kTmemCols == 512, "TMEM columns");
  static_assert(BN % 64 == 0 && BN <= 256, "BN");
  static_assert(kSmemBytes <= 232448, "shared memory");
  static_assert(kSmemBytes > 232448 / 2, "one CTA per SM keeps TMEM allocation uncontended");
};

// ------------------------------------------------------------ NF4 decode (SMEM)
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// Expand 8 NF4 codes (one packed word) through the per-block table into 8 fp16.
// L/H hold the low/high bytes of table entries 0..15.  Entries 0-7 and 8-15 are
// looked up separately with 3-bit selectors, then merged on bit 3 of each code.
__device__ __forceinline__ uint4 nf4_expand8(uint32_t w, const uint32_t (&L)[4],
                                             const uint32_t (&H)[4]) {
  uint4 o;
  // prmt reads only the low 16 bits of its selector, so the selectors of both
  // halves come from one mask of the whole word (the high half shifted down).
  const uint32_t s_all = w & 0x77777777u;
  const uint32_t sel_all = ((w >> 1) & 0x44444444u) | 0x32103210u;
  {
    const uint32_t s = s_all, sel = sel_all;
    const uint32_t lo = prmt(prmt(L[0], L[1], s), prmt(L[2], L[3], s), sel);
    const uint32_t hi = prmt(prmt(H[0], H[1], s), prmt(H[2], H[3], s), sel);
    o.x = prmt(lo, hi, 0x4051u);  // elements 0, 1 (high nibble of byte 0 first)
    o.y = prmt(lo, hi, 0x6273u);  // elements 2, 3
  }
  {
    const uint32_t s = s_all >> 16, sel = sel_all >> 16;
    const uint32_t lo = prmt(prmt(L[0], L[1], s), prmt(L[2], L[3], s), sel);
    const uint32_t hi = prmt(prmt(H[0], H[1], s), prmt(H[2], H[3], s), sel);
    o.z = prmt(lo, hi, 0x4051u);
    o.w = prmt(lo, hi, 0x6273u);
  }
  return o;
}

__device__ __forceinline__ void nf4_table(float scale, uint32_t (&L)[4], uint32_t (&H)[4]) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    __half2 h01 = __floats2half2_rn(__fmul_rn(c_nf4_values[4 * q], scale),
                                    __fmul_rn(c_nf4_values[4 * q + 1], scale));
    __half2 h23 = __floats2half2_rn(__fmul_rn(c_nf4_values[4 * q + 2], scale),
                                    __fmul_rn(c_nf4_values[4 * q + 3], scale));
    const uint32_t a = *reinterpret_cast<uint32_t*>(&h01);
    const uint32_t b = *reinterpret_cast<uint32_t*>(&h23);
    L[q] = prmt(a, b, 0x6420u);
    H[q] = prmt(a, b, 0x7531u);
  }
}

// Decode one 64-element block given as its 32 packed bytes (p0 = bytes 0-15, p1 = 16-31)
// into a 128-byte swizzled SMEM row at `dst` (row index `r` inside its 8-row swizzle atom);
// an invalid block (outside the weight) is written as zeros.
__device__ __forceinline__ void nf4_decode_words(uint4 p0, uint4 p1, uint8_t* dst, int r, float scale,
                                                 bool valid) {
  const uint32_t swz = static_cast<uint32_t>(r & 7);
  if (!valid) {
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      *reinterpret_cast<uint4*>(dst + ((c ^ swz) << 4)) = make_uint4(0, 0, 0, 0);
    }
    return;
  }
  uint32_t L[4], H[4];
  nf4_table(scale, L, H);
  const uint32_t words[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    *reinterpret_cast<uint4*>(dst + ((c ^ swz) << 4)) = nf4_expand8(words[c], L, H);
  }
}

// Same, reading the packed bytes from shared memory (`raw_lo`: bytes 0-15, `raw_hi`: 16-31).
// nf4_decode_words with the chunk order of the row flipped by `flip` (0 or 4):
// chunk c of the row is written by store c ^ flip.  Two lanes that write the same
// row index of two panels 8 KB apart (same banks) then never hit the same
// 16-byte bank group in one store instruction when their flips differ.
__device__ __forceinline__ void nf4_decode_words_flip(uint4 p0, uint4 p1, uint8_t* dst, int r, float scale,
                                                      bool valid, uint32_t flip) {
  const uint32_t swz = static_cast<uint32_t>(r & 7) ^ flip;
  if (!valid) {
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      *reinterpret_cast<uint4*>(dst + ((c ^ swz) << 4)) = make_uint4(0, 0, 0, 0);
    }
    return;
  }
  uint32_t L[4], H[4];
  nf4_table(scale, L, H);
  const uint32_t words[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
  const bool f = flip != 0;
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    // Store c writes chunk c ^ flip, whose codes are words[c ^ flip].
    const uint32_t w = f ? words[c ^ 4] : words[c];
    *reinterpret_cast<uint4*>(dst + ((c ^ swz) << 4)) = nf4_expand8(w, L, H);
  }
}

__device__ __forceinline__ void nf4_decode_row(const uint8_t* raw_lo, const uint8_t* raw_hi,
                                               uint8_t* dst, int r, float scale, bool valid) {
  const uint4 p0 = valid ? *reinterpret_cast<const uint4*>(raw_lo) : make_uint4(0, 0, 0, 0);
  const uint4 p1 = valid ? *reinterpret_cast<const uint4*>(raw_hi) : make_uint4(0, 0, 0, 0);
  nf4_decode_words(p0, p1, dst, r, scale, valid);
}

__device__ __forceinline__ float nf4_scale(const Params& p, int64_t blk, float off) {
  const float code = __ldg(p.code2 + __ldg(p.qabs + blk));
  return __fadd_rn(__fmul_rn(code, __ldg(p.absmax2 + (blk >> 8))), off);
}

// ------------------------------------------------------------ epilogue helpers
__device__ __forceinline__ int runtime_rows(const Params& p) {
  return p.m_dev ? *p.m_dev : p.M;
}

// Per-row epilogue state carried across the 32-column chunks of one tile.
struct EpiState {
  float m, s, t, tz;   // CE stats: running max, sum exp(z-m), sum exp(z-m)*z, target logit
  int arg;             // CE stats: first argmax (column within this launch)
  int64_t tgt;         // target vocabulary index (or ignore_index)
  float lse, gscale;   // CE dz: row lse and g / gain
  float* out;          // kStoreF32 / kAccF32: output base (p.out, or p.out_split for a second half)
};

__device__ __forceinline__ float round_f16(float x) { return __half2float(__float2half_rn(x)); }

template <int EMODE>
__device__ __forceinline__ void epilogue_begin(const Params& p, EpiState& st, int row, int rows_valid) {
  st.out = static_cast<float*>(p.out);
  if constexpr (EMODE == kCeStats) {
    st.m = -INFINITY; st.s = 0.0f; st.t = 0.0f; st.tz = 0.0f; st.arg = 0x7fffffff;
    st.tgt = row < rows_valid ? p.targets[row] : p.ignore_index;
  } else if constexpr (EMODE == kCeDz) {
    st.tgt = p.ignore_index; st.lse = 0.0f; st.gscale = 0.0f;
    if (row < rows_valid) {
      st.tgt = p.targets[row];
      st.lse = p.lse[row];
      st.gscale = __fdiv_rn(p.grad[row], p.gain[row]);
    }
  }
}

template <int EMODE>
__device__ __forceinline__ void epilogue_chunk(const Params& p, EpiState& st, const uint32_t (&v)[32],
                                               int row, int col0, int rows_valid) {
  if constexpr (EMODE == kCeStats) {
    // Logits are the fp16-rounded GEMM result (reference: torch.mm with fp16 output,
    // solution/kernels/cross_entropy.py:149); statistics follow :57-89.  Columns
    // past N only occur in a launch's last chunk, which takes the guarded path.
    float z[32];
    const bool full = col0 + 32 <= p.N;
    if (full) {
#pragma unroll
      for (int j = 0; j < 32; ++j) z[j] = round_f16(__uint_as_float(v[j]));
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) z[j] = (col0 + j < p.N) ? round_f16(__uint_as_float(v[j])) : -INFINITY;
    }
    float mx[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) mx[j] = fmaxf(fmaxf(z[4 * j], z[4 * j + 1]), fmaxf(z[4 * j + 2], z[4 * j + 3]));
    const float cmax = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])), fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
    if (cmax > st.m) {
      // A new running maximum: rescale the sums and record its first column.
      int carg = 31;
#pragma unroll
      for (int j = 31; j >= 0; --j) carg = (z[j] == cmax) ? j : carg;
      const float r = st.m == -INFINITY ? 0.0f : __expf(st.m - cmax);
      st.s *= r;
      st.t *= r;
      st.m = cmax;
      st.arg = col0 + carg;
    }
    if (st.m != -INFINITY) {
      if (full) {
        // Four independent partial sums per thread (short dependency chains).
        float s4[4] = {0.0f, 0.0f, 0.0f, 0.0f}, t4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float e = __expf(z[j] - st.m);
          s4[j & 3] += e;
          t4[j & 3] = fmaf(e, z[j], t4[j & 3]);
        }
        st.s += (s4[0] + s4[1]) + (s4[2] + s4[3]);
        st.t += (t4[0] + t4[1]) + (t4[2] + t4[3]);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          if (col0 + j < p.N) {
            const float e = __expf(z[j] - st.m);
            st.s += e;
            st.t = fmaf(e, z[j], st.t);
          }
        }
      }
    }
    const int64_t g0 = p.col_offset + col0;
    if (st.tgt != p.ignore_index && st.tgt >= g0 && st.tgt < g0 + 32) {
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        if (g0 + j == st.tgt && col0 + j < p.N) st.tz = z[j];
      }
    }
  } else if constexpr (EMODE == kCeDz) {
    // dz = fp16((exp(z - lse) - onehot) * g / gain)  (solution/kernels/cross_entropy.py:108-122).
    if (row >= rows_valid) return;
    __half* out = static_cast<__half*>(p.out) + static_cast<int64_t>(row) * p.ldo;
    const int64_t g0 = p.col_offset + col0;
    float d[32];
    const bool has_tgt = st.tgt >= g0 && st.tgt < g0 + 32;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      float e = __expf(round_f16(__uint_as_float(v[j])) - st.lse);
      if (has_tgt && g0 + j == st.tgt) e -= 1.0f;
      d[j] = e * st.gscale;
    }
    if (p.vec_ok && col0 + 32 <= p.N) {
      uint32_t h[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        __half2 t = __floats2half2_rn(d[2 * j], d[2 * j + 1]);
        h[j] = *reinterpret_cast<uint32_t*>(&t);
      }
      uint4* dst = reinterpret_cast<uint4*>(out + col0);
#pragma unroll
      for (int j = 0; j < 4; ++j) dst[j] = make_uint4(h[4 * j], h[4 * j + 1], h[4 * j + 2], h[4 * j + 3]);
    } else {
      for (int j = 0; j < 32; ++j) {
        if (col0 + j < p.N) out[col0 + j] = __float2half_rn(d[j]);
      }
    }
  } else if constexpr (EMODE == kStoreF16) {
    if (row >= rows_valid) return;
    __half* out = static_cast<__half*>(p.out) + static_cast<int64_t>(row) * p.ldo;
    float f[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) f[j] = __uint_as_float(v[j]);
    if (p.bias) {
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        if (col0 + j < p.N) f[j] = __fadd_rn(f[j], __half2float(p.bias[col0 + j]));
      }
    }
    if (p.vec_ok && col0 + 32 <= p.N) {
      uint32_t h[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        __half2 t = __floats2half2_rn(f[2 * j], f[2 * j + 1]);
        h[j] = *reinterpret_cast<uint32_t*>(&t);
      }
      uint4* dst = reinterpret_cast<uint4*>(out + col0);
#pragma unroll
      for (int j = 0; j < 4; ++j) dst[j] = make_uint4(h[4 * j], h[4 * j + 1], h[4 * j + 2], h[4 * j + 3]);
    } else {
      for (int j = 0; j < 32; ++j) {
        if (col0 + j < p.N) out[col0 + j] = __float2half_rn(f[j]);
      }
    }
  } else {  // kStoreF32 / kAccF32
    if (row >= rows_valid) return;
    float* out = st.out + static_cast<int64_t>(row) * p.ldo;
    if (p.vec_ok && col0 + 32 <= p.N) {
      float4* dst = reinterpret_cast<float4*>(out + col0);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float4 a = make_float4(__uint_as_float(v[4 * j]), __uint_as_float(v[4 * j + 1]),
                               __uint_as_float(v[4 * j + 2]), __uint_as_float(v[4 * j + 3]));
        if constexpr (EMODE == kAccF32) {
          const float4 o = dst[j];
          a.x += o.x; a.y += o.y; a.z += o.z; a.w += o.w;
        }
        dst[j] = a;
      }
    } else {
      for (int j = 0; j < 32; ++j) {
        if (col0 + j < p.N) {
          const float a = __uint_as_float(v[j]);
          if constexpr (EMODE == kAccF32) out[col0 + j] += a; else out[col0 + j] = a;
        }
      }
    }
  }
}

template <int EMODE>
__device__ __forceinline__ void epilogue_end(const Params& p, const EpiState& st, int row, int nt,
                                             int rows_valid) {
  if constexpr (EMODE == kCeStats) {
    if (row < rows_valid) {
      const int64_t ld = p.stats_ld;
      float* base = p.stats + static_cast<int64_t>(nt) * 4 * ld + row;
      base[0] = st.m;
      base[ld] = st.s;
      base[2 * ld] = st.t;
      base[3 * ld] = st.tz;
      p.stats_arg[static_cast<int64_t>(nt) * ld + row] = st.arg;
    }
  }
}

// ------------------------------------------------------------ work schedule
// A work unit is one output tile over the k-blocks [k0, k1).  Tile mode: CTA c
// takes tiles c, c + grid, ... whole.  Stream-K mode: the tile-major k-iteration
// space T = tiles * k_blocks is cut into `grid` equal contiguous ranges, one per
// CTA, so every SM gets the same amount of MMA work whatever the tile count; a
// tile split between CTAs is finished by whichever contributor arrives last.
struct Unit {
  int tile, k0, k1;
  int split;  // half of a split reduction (0 without a split)
};

struct UnitIter {
  int64_t cursor, end;
  int kb, stride;
  int ks = 1, tiles = 0;
  bool streamk;
  __device__ UnitIter(const Params& p, int num_tiles) : UnitIter(p, num_tiles, blockIdx.x, gridDim.x) {}
  // Worker `id` of `count` (a CTA, or a CTA pair of a 2-SM kernel).
  __device__ UnitIter(const Params& p, int num_tiles, int id, int count) {
    streamk = p.streamk != 0;
    kb = p.k_blocks;
    if (streamk) {
      const int64_t total = static_cast<int64_t>(num_tiles) * kb;
      cursor = total * id / count;
      end = total * (id + 1) / count;
      stride = 0;
    } else {
      ks = p.ksplit > 1 ? p.ksplit : 1;
      tiles = num_tiles;
      cursor = id;
      end = static_cast<int64_t>(num_tiles) * ks;
      stride = count;
    }
  }
  __device__ bool next(Unit& u) {
    if (cursor >= end) return false;
    if (streamk) {
      u.split = 0;
      u.tile = static_cast<int>(cursor / kb);
      u.k0 = static_cast<int>(cursor % kb);
      const int64_t k1 = u.k0 + (end - cursor);
      u.k1 = static_cast<int>(k1 < kb ? k1 : kb);
      cursor += u.k1 - u.k0;
    } else {
      u.tile = static_cast<int>(cursor % tiles);
      u.split = static_cast<int>(cursor / tiles);
      u.k0 = kb * u.split / ks;
      u.k1 = kb * (u.split + 1) / ks;
      cursor += stride;
    }
    return true;
  }
};

// Stream-K: the CTA whose iteration range contains iteration x.
__device__ __forceinline__ int sk_owner(int64_t x, int64_t total, int grid) {
  int c = static_cast<int>(x * grid / total);
  while (c + 1 < grid && total * (c + 1) / grid <= x) ++c;
  while (c > 0 && total * c / grid > x) --c;
  return c;
}

// Bounded rendezvous of the 128 epilogue threads on an mbarrier (no unbounded bar.sync:
// if a wait elsewhere gave up, the others leave after the time limit instead of hanging).
__device__ __forceinline__ bool epi_sync(uint64_t* bar, uint32_t& phase, volatile int* abort) {
  mbar_arrive(bar);
  const bool ok = mbar_wait(bar, phase, kErrWaitAccFull, abort);
  phase ^= 1u;
  return ok;
}

// ------------------------------------------------------------ epilogue role
// Warps 4..7: drain each finished accumulator from TMEM (lanes 32 * (warp % 4)),
// run the epilogue and release the buffer; stream-K partial tiles are parked in
// the caller-provided partial slots and the last contributor finishes the tile.
template <int EMODE, int MSUB, int BN>
__device__ __forceinline__ void run_epilogue_role(const Params& p, uint32_t tmem_base, uint64_t* acc_full,
                                                  uint64_t* acc_empty, uint64_t* epi_mb,
                                                  volatile int* abort_flag, volatile int* last_flag,
                                                  int warp, int lane, int num_tiles, int rows_valid,
                                                  int m_tiles) {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const int etid = (warp - 4) * 32 + lane;
    const int64_t total = static_cast<int64_t>(num_tiles) * p.k_blocks;
    uint32_t tl = 0, epi_phase = 0;
    int uidx = 0;
    UnitIter iter(p, num_tiles);
    Unit u;
    while (iter.next(u)) {
      const int mt = u.tile % m_tiles, nt = u.tile / m_tiles;
      const int m0 = mt * MSUB * kTileRows, n0 = nt * BN;
      if (m0 >= rows_valid) continue;
      const int buf = tl & 1;
      const uint32_t aph = (tl >> 1) & 1;
      if (!mbar_wait(&acc_full[buf], aph, kErrWaitAccFull, abort_flag)) break;
      tc_fence_after();
      const uint32_t tacc = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + buf * MSUB * BN;
      // Whole units (every unit of the whole-tile schedule, split or not) run the
      // epilogue directly; stream-K partial units take the fix-up below.
      if (!p.streamk || (u.k0 == 0 && u.k1 == p.k_blocks)) {
#pragma unroll 1
        for (int ms = 0; ms < MSUB; ++ms) {
          const int row = m0 + ms * kTileRows + q * 32 + lane;
          EpiState st;
          epilogue_begin<EMODE>(p, st, row, rows_valid);
          if (u.split) st.out = static_cast<float*>(p.out_split);
#pragma unroll 1
          for (int c = 0; c < BN / 32; ++c) {
            uint32_t v[32];
            tmem_ld32(tacc + ms * BN + c * 32, v);
            tmem_ld_wait();
            epilogue_chunk<EMODE>(p, st, v, row, n0 + c * 32, rows_valid);
          }
          epilogue_end<EMODE>(p, st, row, nt, rows_valid);
        }
        tc_fence_before();
        mbar_arrive(&acc_empty[buf]);
      } else {
        // Stream-K partial tile: park the fp32 accumulator in this CTA's slot,
        // release TMEM, then let the last contributor to arrive sum every slot
        // in CTA order (deterministic) and run the epilogue.
        const int slot = uidx == 0 ? 0 : 1;
        // Slot layout is thread-major ([ms][chunk][j][etid] float4) so each warp
        // writes and later reads 512 contiguous bytes per instruction.
        constexpr int kSlotF4 = MSUB * (BN / 32) * 8 * 128;  // float4 per slot
        float4* mine = reinterpret_cast<float4*>(p.partials) + (static_cast<int64_t>(blockIdx.x) * 2 + slot) * kSlotF4;
#pragma unroll 1
        for (int ms = 0; ms < MSUB; ++ms) {
#pragma unroll 1
          for (int c = 0; c < BN / 32; ++c) {
            uint32_t v[32];
            tmem_ld32(tacc + ms * BN + c * 32, v);
            tmem_ld_wait();
            float4* dst = mine + ((ms * (BN / 32) + c) * 8) * 128 + etid;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              __stcg(dst + j * 128, make_float4(__uint_as_float(v[4 * j]), __uint_as_float(v[4 * j + 1]),
                                                __uint_as_float(v[4 * j + 2]), __uint_as_float(v[4 * j + 3])));
            }
          }
        }
        tc_fence_before();
        mbar_arrive(&acc_empty[buf]);
        __threadfence();
        if (!epi_sync(epi_mb, epi_phase, abort_flag)) break;
        const int64_t it0 = static_cast<int64_t>(u.tile) * p.k_blocks;
        const int c_lo = sk_owner(it0, total, gridDim.x);
        const int c_hi = sk_owner(it0 + p.k_blocks - 1, total, gridDim.x);
        if (etid == 0) {
          const int prev = atomicAdd(p.counters + u.tile, 1);
          *last_flag = (prev == c_hi - c_lo) ? 1 : 0;
        }
        if (!epi_sync(epi_mb, epi_phase, abort_flag)) break;
        const bool last = *last_flag != 0;
        // Every thread has read the flag before it can be rewritten.
        if (!epi_sync(epi_mb, epi_phase, abort_flag)) break;
        if (last) {
          __threadfence();
#pragma unroll 1
          for (int ms = 0; ms < MSUB; ++ms) {
            const int lrow = ms * kTileRows + q * 32 + lane;
            const int row = m0 + lrow;
            EpiState st;
            epilogue_begin<EMODE>(p, st, row, rows_valid);
#pragma unroll 1
            for (int c = 0; c < BN / 32; ++c) {
              float sum[32];
#pragma unroll
              for (int j = 0; j < 32; ++j) sum[j] = 0.0f;
              const int64_t off = static_cast<int64_t>((ms * (BN / 32) + c) * 8) * 128 + etid;
              // Contributors are summed in CTA order; their loads are issued
              // in batches of four so the L2 round trips overlap.
              for (int cc = c_lo; cc <= c_hi; cc += 4) {
                float4 x[4][8];
#pragma unroll
                for (int b = 0; b < 4; ++b) {
                  const int ci = cc + b;
                  if (ci <= c_hi) {
                    const int64_t first_tile = (total * ci / gridDim.x) / p.k_blocks;
                    const int cslot = first_tile == u.tile ? 0 : 1;
                    const float4* src = reinterpret_cast<const float4*>(p.partials) +
                                        (static_cast<int64_t>(ci) * 2 + cslot) * kSlotF4 + off;
#pragma unroll
                    for (int j = 0; j < 8; ++j) x[b][j] = __ldcg(src + j * 128);
                  }
                }
#pragma unroll
                for (int b = 0; b < 4; ++b) {
                  if (cc + b <= c_hi) {
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                      sum[4 * j] += x[b][j].x; sum[4 * j + 1] += x[b][j].y;
                      sum[4 * j + 2] += x[b][j].z; sum[4 * j + 3] += x[b][j].w;
                    }
                  }
                }
              }
              uint32_t v[32];
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] = __float_as_uint(sum[j]);
              epilogue_chunk<EMODE>(p, st, v, row, n0 + c * 32, rows_valid);
            }
            epilogue_end<EMODE>(p, st, row, nt, rows_valid);
          }
          if (etid == 0) p.counters[u.tile] = 0;  // ready for the next launch
        }
      }
      ++tl;
      ++uidx;
    }
}

// ------------------------------------------------------------ the kernel
template <int BMODE, int EMODE, int MSUB, int BN, int STAGES>
__global__ void __launch_bounds__(Cfg<BMODE, MSUB, BN, STAGES>::kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ CUtensorMap tmLA, const __grid_constant__ CUtensorMap tmLB,
                const Params p) {
  using C = Cfg<BMODE, MSUB, BN, STAGES>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* bar_area = smem + STAGES * C::kStageBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(bar_area);
  uint64_t* empty = full + STAGES;
  uint64_t* decoded = empty + STAGES;
  uint64_t* acc_full = decoded + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint64_t* epi_mb = drain + 1;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(epi_mb + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  volatile int* last_flag = abort_flag + 1;
  float* code2_s = reinterpret_cast<float*>(bar_area + 1024);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const bool has_lora = p.lora_r > 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      mbar_init(&decoded[s], 128);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 128);
    }
    mbar_init(drain, 1);
    mbar_init(epi_mb, 128);
    *abort_flag = 0;
    *last_flag = 0;
    fence_barrier_init();
  }
  if constexpr (C::kNF4) {
    for (int i = threadIdx.x; i < 256; i += blockDim.x) code2_s[i] = __ldg(p.code2 + i);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, C::kTmemCols);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  const int rows_valid = runtime_rows(p);
  // Tiles past the runtime row count (the CE backward's compacted labelled rows,
  // a count known only on the device) are left out of the schedule, so the
  // valid tiles are shared evenly by the CTAs.
  const int m_tiles = min(p.m_tiles, (rows_valid + MSUB * kTileRows - 1) / (MSUB * kTileRows));
  const int num_tiles = m_tiles * p.n_tiles;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      if (has_lora) {
        tma_prefetch_desc(&tmLA);
        tma_prefetch_desc(&tmLB);
      }
      uint32_t it = 0;
      bool ok = true;
      UnitIter iter(p, num_tiles);
      Unit u;
      while (ok && iter.next(u)) {
        const int mt = u.tile % m_tiles, nt = u.tile / m_tiles;
        const int m0 = mt * MSUB * kTileRows, n0 = nt * BN;
        if (m0 >= rows_valid) continue;
        const int nsteps = (u.k1 - u.k0) + ((has_lora && u.k1 == p.k_blocks) ? 1 : 0);
        for (int ls = 0; ls < nsteps; ++ls, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, kErrWaitEmpty, abort_flag)) { ok = false; break; }
          uint8_t* a_s = smem + s * C::kStageBytes;
          uint8_t* b_s = a_s + C::kABytes;
          uint8_t* raw_s = b_s + C::kBBytes;
          const int step = u.k0 + ls;
          if (step < u.k1) {
            mbar_arrive_expect_tx(&full[s], C::kABytes + (C::kNF4 ? C::kRawBytes : C::kBBytes));
#pragma unroll
            for (int ms = 0; ms < MSUB; ++ms) {
              tma_load_2d(a_s + ms * kTileRows * kBK * 2, &tmA, &full[s], step * kBK, m0 + ms * kTileRows);
            }
            if constexpr (BMODE == kNF4Fwd) {
              tma_load_2d(raw_s, &tmB, &full[s], step * (kBK / 2), n0);
            } else if constexpr (BMODE == kNF4Dx) {
              tma_load_2d(raw_s, &tmB, &full[s], n0 / 2, step * kBK);
            } else if constexpr (BMODE == kDenseK) {
              tma_load_2d(b_s, &tmB, &full[s], step * kBK, n0);
            } else {
#pragma unroll
              for (int pnl = 0; pnl < BN / 64; ++pnl) {
                tma_load_2d(b_s + pnl * 64 * 128, &tmB, &full[s], n0 + pnl * 64, step * kBK);
              }
            }
          } else {
            mbar_arrive_expect_tx(&full[s], (MSUB * kTileRows + BN) * p.lora_r * 2);
            tma_load_2d(a_s, &tmLA, &full[s], 0, m0);
            tma_load_2d(b_s, &tmLB, &full[s], 0, n0);
          }
        }
      }
      // Drain: every TMA this thread issued must land before the CTA exits.
      const uint32_t first = it > static_cast<uint32_t>(STAGES) ? it - STAGES : 0;
      for (uint32_t j = first; j < it; ++j) {
        volatile int no_abort = 0;
        mbar_wait(&full[j % STAGES], (j / STAGES) & 1, kErrWaitDrain, &no_abort);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ UMMA issuer
    if (lane == 0) {
      constexpr uint32_t kIdesc = idesc_f16_f32(kTileRows, BN, 0, C::kBMN ? 1 : 0);
      constexpr uint32_t kIdescLora = idesc_f16_f32(kTileRows, BN, 0, 0);
      const uint32_t lora_layout = p.lora_r == 16 ? kSwizzle32B : (p.lora_r == 32 ? kSwizzle64B : kSwizzle128B);
      const uint32_t lora_pitch = static_cast<uint32_t>(p.lora_r) * 2;
      uint32_t it = 0, tl = 0;
      bool ok = true;
      UnitIter iter(p, num_tiles);
      Unit u;
      while (ok && iter.next(u)) {
        if ((u.tile % m_tiles) * MSUB * kTileRows >= rows_valid) continue;
        const int buf = tl & 1;
        const uint32_t aph = (tl >> 1) & 1;
        if (!mbar_wait(&acc_empty[buf], aph ^ 1, kErrWaitAccEmpty, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint32_t acc = tmem_base + buf * MSUB * BN;
        const int nsteps = (u.k1 - u.k0) + ((has_lora && u.k1 == p.k_blocks) ? 1 : 0);
        for (int ls = 0; ls < nsteps; ++ls, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          const bool main_step = u.k0 + ls < u.k1;
          if (!mbar_wait(&full[s], ph, kErrWaitFull, abort_flag)) { ok = false; break; }
          // Every step, the LoRA step included, waits for the decoder group's arrival:
          // otherwise the stage could be refilled before a lagging group has seen
          // this phase of full[s], and its parity wait would then alias the next phase.
          if (C::kNF4) {
            if (!mbar_wait(&decoded[s], ph, kErrWaitDecoded, abort_flag)) { ok = false; break; }
          }
          tc_fence_after();
          const uint32_t a_addr = smem_addr(smem + s * C::kStageBytes);
          const uint32_t b_addr = a_addr + C::kABytes;
          if (main_step) {
#pragma unroll
            for (int k16 = 0; k16 < kBK / 16; ++k16) {
              const uint64_t bdesc = C::kBMN
                  ? smem_desc(b_addr + k16 * 16 * 128, 64 * 128, 1024, kSwizzle128B)
                  : smem_desc(b_addr + k16 * 32, 16, 1024, kSwizzle128B);
#pragma unroll
              for (int ms = 0; ms < MSUB; ++ms) {
                const uint64_t adesc = smem_desc(a_addr + ms * kTileRows * kBK * 2 + k16 * 32, 16, 1024, kSwizzle128B);
                umma_f16(acc + ms * BN, adesc, bdesc, kIdesc, (ls > 0 || k16 > 0) ? 1u : 0u);
              }
            }
          } else {
            for (int k16 = 0; k16 < p.lora_r / 16; ++k16) {
              const uint64_t bdesc = smem_desc(b_addr + k16 * 32, 16, 8 * lora_pitch, lora_layout);
#pragma unroll
              for (int ms = 0; ms < MSUB; ++ms) {
                const uint64_t adesc = smem_desc(a_addr + ms * kTileRows * lora_pitch + k16 * 32, 16,
                                                 8 * lora_pitch, lora_layout);
                umma_f16(acc + ms * BN, adesc, bdesc, kIdescLora, 1u);
              }
            }
          }
          umma_commit(&empty[s]);
        }
        if (ok) umma_commit(&acc_full[buf]);
        ++tl;
      }
      // Drain: wait for every UMMA issued above before TMEM is freed.
      umma_commit(drain);
      volatile int no_abort = 0;
      mbar_wait(drain, 0, kErrWaitDrain, &no_abort);
    }
  } else if (warp >= 4 && warp < 8) {
    run_epilogue_role<EMODE, MSUB, BN>(p, tmem_base, acc_full, acc_empty, epi_mb, abort_flag, last_flag,
                                       warp, lane, num_tiles, rows_valid, m_tiles);
  } else if (C::kNF4 && warp >= 8) {
    // ------------------------------------------------------------ NF4 decoders
    // Group g decodes the k-steps whose global index has parity g.  Each thread
    // owns BN/128 (row, 64-block) tasks per step; the qabs byte and absmax2 value
    // of its next step are loaded while the current one decodes, and code2 is
    // read from shared memory, so no dependent global load sits on the critical path.
    constexpr int kTasks = BN / 128;
    const int group = (warp - 8) >> 2;
    const int gtid = ((warp - 8) & 3) * 32 + lane;
    const float off = __ldg(p.offset);
    const int64_t bpr = p.w_cols / 64;
    uint32_t it = 0;
    bool ok = true;
    // Block index of task t at k-step `step` of the tile starting at output column n0,
    // or -1 when that (row, block) lies outside the weight (written as zeros).
    auto block_of = [&](int n0, int step, int task) -> int64_t {
      if constexpr (BMODE == kNF4Fwd) {
        const int64_t wrow = n0 + task;
        return wrow < p.w_rows ? wrow * bpr + step : -1;
      } else {
        constexpr int kPanels = BN / 64;
        const int64_t wrow = static_cast<int64_t>(step) * kBK + task / kPanels;
        const int64_t wcol = n0 + 64 * (task % kPanels);
        return (wrow < p.w_rows && wcol < p.w_cols) ? wrow * bpr + wcol / 64 : -1;
      }
    };
    UnitIter iter(p, num_tiles);
    Unit u;
    while (ok && iter.next(u)) {
      if ((u.tile % m_tiles) * MSUB * kTileRows >= rows_valid) continue;
      const int n0 = (u.tile / m_tiles) * BN;
      const int nsteps = (u.k1 - u.k0) + ((has_lora && u.k1 == p.k_blocks) ? 1 : 0);
      // First k-step of this unit owned by this group.
      const int first = u.k0 + ((static_cast<int>(it & 1) == group) ? 0 : 1);
      uint32_t q_next[kTasks];
      float a2_next[kTasks];
#pragma unroll
      for (int t = 0; t < kTasks; ++t) {
        const int64_t blk = first < u.k1 ? block_of(n0, first, gtid + 128 * t) : -1;
        q_next[t] = blk >= 0 ? __ldg(p.qabs + blk) : 0u;
        a2_next[t] = blk >= 0 ? __ldg(p.absmax2 + (blk >> 8)) : 0.0f;
      }
      for (int ls = 0; ls < nsteps; ++ls, ++it) {
        if (static_cast<int>(it & 1) != group) continue;
        const int s = it % STAGES;
        const uint32_t ph = (it / STAGES) & 1;
        const int step = u.k0 + ls;
        const bool main_step = step < u.k1;
        uint32_t q_cur[kTasks];
        float a2_cur[kTasks];
        bool valid[kTasks];
#pragma unroll
        for (int t = 0; t < kTasks; ++t) {
          q_cur[t] = q_next[t];
          a2_cur[t] = a2_next[t];
          valid[t] = main_step && block_of(n0, step, gtid + 128 * t) >= 0;
          const int64_t nb = step + 2 < u.k1 ? block_of(n0, step + 2, gtid + 128 * t) : -1;
          q_next[t] = nb >= 0 ? __ldg(p.qabs + nb) : 0u;
          a2_next[t] = nb >= 0 ? __ldg(p.absmax2 + (nb >> 8)) : 0.0f;
        }
        if (!mbar_wait(&full[s], ph, kErrWaitFull, abort_flag)) { ok = false; break; }
        if (main_step) {
          uint8_t* b_s = smem + s * C::kStageBytes + C::kABytes;
          const uint8_t* raw_s = b_s + C::kBBytes;
#pragma unroll
          for (int t = 0; t < kTasks; ++t) {
            const int task = gtid + 128 * t;
            const float scale = valid[t] ? __fadd_rn(__fmul_rn(code2_s[q_cur[t]], a2_cur[t]), off) : 0.0f;
            if constexpr (BMODE == kNF4Fwd) {
              // Raw rows are 32 B, TMA-swizzled in 32 B spans: chunk ^= (row >> 2) & 1.
              const int r = task;
              const uint32_t x = static_cast<uint32_t>((r >> 2) & 1);
              nf4_decode_row(raw_s + r * 32 + (x << 4), raw_s + r * 32 + ((x ^ 1u) << 4),
                             b_s + r * 128, r, scale, valid[t]);
            } else {
              // Raw rows are BN/2 = 64 B, TMA-swizzled in 64 B spans: chunk ^= (row >> 1) & 3.
              constexpr int kPanels = BN / 64;
              static_assert(BMODE != kNF4Dx || BN == 128, "dX raw swizzle assumes 64-byte raw rows");
              const int r = task / kPanels, j = task % kPanels;
              const uint32_t x = static_cast<uint32_t>((r >> 1) & 3);
              const uint8_t* row = raw_s + r * 64;
              nf4_decode_row(row + (((2u * j) ^ x) << 4), row + (((2u * j + 1u) ^ x) << 4),
                             b_s + j * (kBK * 128) + r * 128, r, scale, valid[t]);
            }
          }
        }
        fence_proxy_async_smem();
        mbar_arrive(&decoded[s]);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::kTmemCols);
  }
}

}  // namespace gemm
}  // namespace sb
