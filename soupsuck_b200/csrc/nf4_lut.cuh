// Small-M NF4 linear (M <= 16 activation rows): forward Y = X . deq(W)^T on mma.sync.
//
// At M <= 16 the product is bound by reading the packed weight (0.52 byte per
// weight), so the limit is how few instructions turn a packed byte into MMA
// operands.  Two modes:
//
//   * exact (default): every operand value is the reference decoder's
//     fp16(NF4[i] * scale).  One lane owns whole 64-blocks: it builds the
//     block's 16-entry table itself (sixteen fp32 products, each rounded once)
//     and expands the block's eight packed words through it with byte permutes;
//   * lookup (SB_SMALLM=lut): a 256-entry table maps a packed byte (two codes,
//     the earlier element in the high nibble) to the half2 of the two UNSCALED
//     code values, one shared-memory load per byte.  Every lane has its own copy
//     of the table (entry e of lane l at byte e * 128 + 4 l), so a warp's 32
//     lookups hit 32 different banks; the block scale s(n, b) =
//     fp32(code2[absmax[n, b]] * absmax2) + offset of the bitsandbytes format
//     multiplies, in fp32, the partial product of each 64-element block after
//     its four mma.sync.m16n8k16 steps.  The weights then enter the MMA as
//     fp16(NF4[i]) -- a different rounding of the same product, inside the GEMM
//     gate up to a reduction of kMaxReduction.
//
// The weight is the MMA's A operand (16 weight rows per warp tile) and the
// activations its B operand (8 or 16 tokens).  The k order inside each MMA is
// permuted (the activation fragment the same way), so each lane reads its packed
// bytes straight from global memory (no staging, no decoded tile): in lookup
// mode lane t of a quad holds bytes 8t .. 8t + 7 of each block of its two rows,
// in exact mode all 32 bytes of block t of each group of four.
//
// Work split: a CTA of 8 warps covers RW row tiles (16 rows each) x KW k-runs
// (RW * KW = 8); a cluster of S CTAs along grid.y splits the reduction, and the
// partial sums are combined in fixed rank order through distributed shared
// memory, then bias and the LoRA term are added and fp16 rows stored.  One launch,
// no global scratch, deterministic.
//
// Reference: bitsandbytes' MatMul4Bit / gemv_4bit small-batch path behind
// solution/nf4_patch.py:43-125; decode rule solution/kernels/nf4.py:41-59.
#pragma once

#include "common.cuh"
#include "gemm_pair.cuh"
#include "lora_mma.cuh"

namespace sb {
namespace lut {

constexpr int kThreads = 256, kWarps = 8;
constexpr int kTableBytes = 256 * 128;    // per-lane byte -> half2 table (lookup mode)
constexpr int kGroup = 4;                 // 64-blocks per load group (one absmax word per row)
constexpr int kMaxSplits = 8;             // cluster size along the reduction (portable)
constexpr int64_t kMaxReduction = 9216;   // longest reduction on this path (its error grows as sqrt)

// The table holds fp16(kAlpha * NF4[i]); the block scale is multiplied by 1/kAlpha
// in fp32.  kAlpha minimises the RMS relative rounding error of the 15 nonzero
// fp16 entries (9.2e-5 against 1.8e-4 at alpha = 1), found by scanning alpha over
// [1, 2) in steps of 2^-16.
constexpr float kAlpha = 1.3661651611328125f;
constexpr float kInvAlpha = 1.0f / 1.3661651611328125f;

// Per-lane byte -> half2 table (32 KB of shared memory).
__device__ __forceinline__ void build_table(uint32_t* table) {
  for (int i = threadIdx.x; i < 256 * 8; i += blockDim.x) {
    const int e = i >> 3, part = i & 7;
    const __half2 v = __floats2half2_rn(kAlpha * c_nf4_values[e >> 4], kAlpha * c_nf4_values[e & 15]);
    const uint32_t u = *reinterpret_cast<const uint32_t*>(&v);
    *reinterpret_cast<uint4*>(table + e * 32 + part * 4) = make_uint4(u, u, u, u);
  }
}

// Byte `I` (0..3) of `w` looked up in this lane's table copy; `tb` is the 32-bit
// shared address of the table plus 4 * lane.
template <int I>
__device__ __forceinline__ uint32_t lookup(uint32_t tb, uint32_t w) {
  uint32_t off;
  if constexpr (I == 0) off = (w << 7) & 0x7F80u;
  else if constexpr (I == 1) off = (w >> 1) & 0x7F80u;
  else if constexpr (I == 2) off = (w >> 9) & 0x7F80u;
  else off = (w >> 17) & 0x7F80u;
  uint32_t v;
  asm("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(tb + off));
  return v;
}

__device__ __forceinline__ float lds_f32(uint32_t addr) {
  float v;
  asm("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(addr));
  return v;
}

// m16n8k16 with a zero accumulator input (no register moves to clear it).
__device__ __forceinline__ void mma16816_z(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%10,%10,%10};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(0.0f));
}

struct FwdArgs {
  const __half* x;        // [M, K] row-major
  int M;
  int64_t K, N;           // reduction length (k_in), output columns (n_out)
  const uint8_t* packed;
  const uint8_t* qabs;
  const float* absmax2;
  const float* code2;
  const float* offset;
  int rw, kw;             // warp layout: rw row tiles x kw k-runs
  int kb_split;           // 64-blocks of the reduction per cluster rank
  int splits;             // cluster size along grid.y
  const __half* bias;     // [N] or null
  const __half* la;       // [M, r] (LoRA: y += la . lb^T) or null
  const __half* lb;       // [N, r]
  int r;
  __half* y;              // [M, N]
};

// Cluster epilogue shared by the forward and dX kernels.  `part` holds this CTA's
// partial sums [rows_cta][16] (row = output column, 16 token slots).  Rank q of
// the cluster finishes a contiguous share of the rows, summing the partials of
// all ranks in rank order through distributed shared memory, adds the LoRA term
// la . lb^T and the bias and stores fp16 y[tok][n_base + row] (row stride width).
__device__ __forceinline__ void cluster_finish(const float* part, int rows_cta, int64_t n_base, int64_t width,
                                               int M, int splits, uint32_t rank, const __half* bias,
                                               const __half* la, const __half* lb, int r, __half* y) {
  gemm::pair::cluster_sync_all();
  const uint32_t part_s = smem_addr(part);
  const int share = (rows_cta + splits - 1) / splits;
  const int row0 = static_cast<int>(rank) * share;
  const int nrows = row0 < rows_cta ? (rows_cta - row0 < share ? rows_cta - row0 : share) : 0;
  for (int e = threadIdx.x; e < nrows * M; e += blockDim.x) {
    const int tok = e / nrows, row = row0 + e % nrows;
    const int64_t n = n_base + row;
    if (n >= width) continue;
    float v = 0.0f;
    for (int q = 0; q < splits; ++q) {
      const uint32_t addr = gemm::pair::map_to_rank(part_s + static_cast<uint32_t>((row * 16 + tok) * 4), q);
      float pv;
      asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(pv) : "r"(addr) : "memory");
      v += pv;
    }
    if (r > 0) {
      float l = 0.0f;
      for (int j = 0; j < r; ++j) l = fmaf(__half2float(la[tok * r + j]), __half2float(lb[n * r + j]), l);
      v += l;
    }
    if (bias) v = __fadd_rn(v, __half2float(bias[n]));
    y[static_cast<int64_t>(tok) * width + n] = __float2half_rn(v);
  }
  gemm::pair::cluster_sync_all();  // no CTA leaves while another reads its partial
}

// Dynamic shared memory of the forward kernel: activation tile, code2 table,
// per-warp fragments, CTA partial.
//
// Activation tile geometry.  Lookup mode: token rows of kb * 128 bytes + 16.
// Exact mode: each 64-block of a token row takes 144 bytes (128 + 16 of skew)
// and the row pitch is 64 mod 128, so the eight lanes of a quarter-warp (two
// tokens x four consecutive blocks) read eight different 16-byte bank groups.
template <int NT>
struct FwdSmem {
  static constexpr int kTok = 8 * NT;
  static constexpr int kExactBlockBytes = 144;
  __host__ __device__ static size_t pitch(int kb, bool exact) {
    if (!exact) return static_cast<size_t>(kb) * 128 + 16;
    const size_t p = static_cast<size_t>(kb) * kExactBlockBytes;
    return p + ((64 + 128 - (p & 127)) & 127);
  }
  __host__ __device__ static size_t x_bytes(int kb, bool exact) { return kTok * pitch(kb, exact); }
  static constexpr int kRedBytes = kWarps * 16 * 16 * 4;    // per-warp C fragments (aliases the tile)
  static constexpr int kPartBytes = kWarps * 16 * 16 * 4;   // CTA partial [rows <= 128][16]
  __host__ __device__ static size_t tile_bytes(int kb, bool exact) {
    return x_bytes(kb, exact) > kRedBytes ? x_bytes(kb, exact) : kRedBytes;
  }
  __host__ __device__ static size_t bytes(int kb, bool exact) {
    return tile_bytes(kb, exact) + 1024 + kPartBytes + (exact ? 0 : kTableBytes);
  }
  // Largest reduction slice per CTA (64-blocks): keeps two CTAs per SM.
  __host__ __device__ static int kb_max(bool exact) { return NT == 1 ? 64 : (exact ? 40 : 32); }
};

// EXACT = false: the unscaled-codebook table above (fp32 block scales after the
// MMAs).  EXACT = true: each block's operand values are the reference decoder's
// fp16(NF4[i] * scale), and the k order inside the MMAs is permuted so that one
// lane owns whole blocks: in a load group of four blocks, lane t of a quad takes
// block t of its two rows (all 32 packed bytes of each), builds that block's
// 16-entry table itself (sixteen products rounded once, no exchange between
// lanes) and expands its eight packed words through it with byte permutes
// (nf4_expand8, as in the tcgen05 kernels).  MMA step j of the group multiplies,
// in lane t's k slots {2t, 2t+1, 2t+8, 2t+9}, elements 4j .. 4j+3 of block t; the
// activation fragment of the same lane reads those elements of its token row, so
// the permutation costs nothing (each lane reads its block's 128 activation bytes
// as eight 16-byte loads).  The MMAs accumulate the decoded weights directly; the
// exact mode has no reduction-length limit.
template <int NT, bool EXACT>
__global__ void __launch_bounds__(kThreads, 2) lut_fwd_kernel(const FwdArgs a) {
  extern __shared__ __align__(128) uint8_t dsm[];
  using S = FwdSmem<NT>;
  // Register ring of load groups: two slots (the next group's loads in flight
  // during this one); three measured slower for 8 token columns (7B gate at
  // M = 1: 20.75 against 20.35 us) and do not fit the registers of 16.
  constexpr int kSlots = 2;
  constexpr int kAhead = kSlots - 1;
  // Bytes of one 64-block in a token row of the activation tile.
  constexpr uint32_t kXBlock = EXACT ? S::kExactBlockBytes : 128;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const uint32_t lane4 = static_cast<uint32_t>(lane) << 2;
  const uint32_t rank = gemm::pair::cluster_rank();
  // Launched with programmatic stream serialization (pdl_ok): nothing of global
  // memory is touched before the previous grid of the stream has completed, and
  // the next grid may be scheduled from here on (its CTAs then wait the same way).
  // Without the attribute both instructions return at once.
  grid_dependency_wait();
  launch_dependents();
  const int64_t kblocks = a.K / 64;
  const int64_t kb0 = static_cast<int64_t>(rank) * a.kb_split;
  int64_t kb1 = kb0 + a.kb_split;
  if (kb1 > kblocks) kb1 = kblocks;
  const int kb_cta = kb1 > kb0 ? static_cast<int>(kb1 - kb0) : 0;
  const size_t pitch = S::pitch(a.kb_split, EXACT);
  uint8_t* xs = dsm;
  float* red = reinterpret_cast<float*>(dsm);  // reused once every warp is past the tile
  float* code2_s = reinterpret_cast<float*>(dsm + S::tile_bytes(a.kb_split, EXACT));
  float* part = code2_s + 256;
  uint32_t* table = reinterpret_cast<uint32_t*>(part + kWarps * 256);  // lookup mode only

  // Activation tile [8 NT tokens][kb_cta * 64] (zero rows past M) by cp.async.
  {
    const int chunks = kb_cta * 8;  // 16-byte pieces per token row
    for (int i = tid; i < S::kTok * chunks; i += kThreads) {
      const int tok = i / chunks, c = i % chunks;
      const bool ok = tok < a.M;
      const __half* src = ok ? a.x + tok * a.K + kb0 * 64 + c * 8 : a.x;
      const uint32_t dst = static_cast<uint32_t>(tok * pitch) + static_cast<uint32_t>(c >> 3) * kXBlock +
                           static_cast<uint32_t>(c & 7) * 16;
      lora::cp_async16(smem_addr(xs + dst), src, ok);
    }
    lora::cp_async_commit();
  }
  for (int i = tid; i < 256; i += kThreads) code2_s[i] = __ldg(a.code2 + i);
  if constexpr (!EXACT) build_table(table);
  const float off = __ldg(a.offset);

  // This warp's row tile and k-run.
  const int rw = warp % a.rw, kw = warp / a.rw;
  const int64_t n_g = (static_cast<int64_t>(blockIdx.x) * a.rw + rw) * 16 + g;
  const int64_t n_g8 = n_g + 8;
  const bool ok_g = n_g < a.N, ok_g8 = n_g8 < a.N;
  const int run = ((kb_cta + a.kw - 1) / a.kw + kGroup - 1) / kGroup * kGroup;
  const int rb0 = kw * run;                               // first block (CTA-relative)
  int rb1 = rb0 + run;
  if (rb1 > kb_cta) rb1 = kb_cta;
  const int nb = rb1 > rb0 ? rb1 - rb0 : 0;
  const int64_t row_bytes = a.K / 2;
  // Byte and block offsets of the weight fit 32 bits (checked by the host).
  // Lane t's piece of each block: bytes 8t .. 8t + 7 (lookup mode), or the whole
  // of block t of each group (exact mode).
  const uint32_t lane_off = EXACT ? 32u * t : 8u * t;
  const uint8_t* p_g = a.packed + static_cast<uint32_t>((ok_g ? n_g : 0) * row_bytes + (kb0 + rb0) * 32 + lane_off);
  const uint8_t* p_g8 = a.packed + static_cast<uint32_t>((ok_g8 ? n_g8 : 0) * row_bytes + (kb0 + rb0) * 32 + lane_off);
  const uint32_t q_g = static_cast<uint32_t>((ok_g ? n_g : 0) * kblocks + kb0 + rb0);
  const uint32_t q_g8 = static_cast<uint32_t>((ok_g8 ? n_g8 : 0) * kblocks + kb0 + rb0);
  const int ng = nb / kGroup;  // runs are whole groups of four blocks

  // Register ring of kSlots groups: per group the two rows' packed bytes (lookup
  // mode: an 8-byte piece of each of the four blocks; exact mode: all 32 bytes of
  // block t), the four absmax bytes of each row (one 32-bit word: groups start on
  // a multiple of four blocks) and the row's absmax2 (the same for the four blocks).
  uint2 pk[kSlots][kGroup][2];
  uint4 pe[kSlots][2][2];
  uint32_t qw[kSlots][2];
  float a2[kSlots][2];
  auto load = [&](int gi, int slot) {
    if (gi < ng) {
      const uint32_t boff = static_cast<uint32_t>(gi) * (kGroup * 32);
      if constexpr (EXACT) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          pe[slot][0][h] = __ldcs(reinterpret_cast<const uint4*>(p_g + boff + h * 16));
          pe[slot][1][h] = __ldcs(reinterpret_cast<const uint4*>(p_g8 + boff + h * 16));
        }
      } else {
#pragma unroll
        for (int b = 0; b < kGroup; ++b) {
          pk[slot][b][0] = __ldcs(reinterpret_cast<const uint2*>(p_g + boff + b * 32));
          pk[slot][b][1] = __ldcs(reinterpret_cast<const uint2*>(p_g8 + boff + b * 32));
        }
      }
      const uint32_t qo = static_cast<uint32_t>(gi) * kGroup;
      qw[slot][0] = __ldg(reinterpret_cast<const uint32_t*>(a.qabs + q_g + qo));
      qw[slot][1] = __ldg(reinterpret_cast<const uint32_t*>(a.qabs + q_g8 + qo));
      a2[slot][0] = __ldg(a.absmax2 + ((q_g + qo) >> 8));
      a2[slot][1] = __ldg(a.absmax2 + ((q_g8 + qo) >> 8));
    }
  };
#pragma unroll
  for (int q = 0; q < kAhead; ++q) load(q, q);

  float acc[NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.0f;

  lora::cp_async_wait<0>();
  __syncthreads();  // table, code2 and activation tile ready

  // Activation rows of this lane's B fragments (token g + 8 nt).
  // Lookup mode: lane t's 16-element piece of each block; exact mode: block t of
  // each group.
  uint32_t xrow[NT];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    xrow[nt] = smem_addr(xs) + static_cast<uint32_t>((g + 8 * nt) * pitch) + static_cast<uint32_t>(rb0) * kXBlock +
               (EXACT ? kXBlock * t : 32u * t);
  }
  const float soff = off;
  const uint32_t tb = smem_addr(table) + lane4;
  const uint32_t c2s = smem_addr(code2_s);

  for (int G = 0; G < ng; G += kSlots) {
#pragma unroll
    for (int sl = 0; sl < kSlots; ++sl) {
      const int gi = G + sl;
      if (gi < ng) {
        load(gi + kAhead, (sl + kAhead) % kSlots);
        if constexpr (EXACT) {
          // Block t of the group, rows g and g + 8: own tables, eight words each.
          const uint32_t sh = 8u * t;
          const float sc_g = ok_g ? __fadd_rn(__fmul_rn(lds_f32(c2s + ((qw[sl][0] >> sh) & 0xFFu) * 4), a2[sl][0]), soff) : 0.0f;
          const float sc_g8 = ok_g8 ? __fadd_rn(__fmul_rn(lds_f32(c2s + ((qw[sl][1] >> sh) & 0xFFu) * 4), a2[sl][1]), soff) : 0.0f;
          uint32_t Lg[4], Hg[4], L8[4], H8[4];
          gemm::nf4_table(sc_g, Lg, Hg);
          gemm::nf4_table(sc_g8, L8, H8);
          const uint32_t wg[8] = {pe[sl][0][0].x, pe[sl][0][0].y, pe[sl][0][0].z, pe[sl][0][0].w,
                                  pe[sl][0][1].x, pe[sl][0][1].y, pe[sl][0][1].z, pe[sl][0][1].w};
          const uint32_t w8[8] = {pe[sl][1][0].x, pe[sl][1][0].y, pe[sl][1][0].z, pe[sl][1][0].w,
                                  pe[sl][1][1].x, pe[sl][1][1].y, pe[sl][1][1].z, pe[sl][1][1].w};
          const uint32_t xg = static_cast<uint32_t>(gi) * (kGroup * kXBlock);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const uint4 eg = gemm::nf4_expand8(wg[i], Lg, Hg);
            const uint4 e8 = gemm::nf4_expand8(w8[i], L8, H8);
            const uint32_t a0[4] = {eg.x, e8.x, eg.y, e8.y};  // elements 8i .. 8i + 3
            const uint32_t a1[4] = {eg.z, e8.z, eg.w, e8.w};  // elements 8i + 4 .. 8i + 7
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              uint32_t xf[4];
              asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                           : "=r"(xf[0]), "=r"(xf[1]), "=r"(xf[2]), "=r"(xf[3]) : "r"(xrow[nt] + xg + 16 * i));
              lora::mma16816(acc[nt], a0, xf[0], xf[1]);
              lora::mma16816(acc[nt], a1, xf[2], xf[3]);
            }
          }
        } else {
#pragma unroll
        for (int b = 0; b < kGroup; ++b) {
          const uint32_t blk = static_cast<uint32_t>(gi * kGroup + b);
          const float sc_g = ok_g ? __fadd_rn(__fmul_rn(lds_f32(c2s + ((qw[sl][0] >> (8 * b)) & 0xFFu) * 4), a2[sl][0]), soff) : 0.0f;
          const float sc_g8 = ok_g8 ? __fadd_rn(__fmul_rn(lds_f32(c2s + ((qw[sl][1] >> (8 * b)) & 0xFFu) * 4), a2[sl][1]), soff) : 0.0f;
          // Activation B fragments (rows past M are zero in the tile).
          uint32_t xf[NT][8];
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            const uint32_t addr = xrow[nt] + blk * 128;
            asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                         : "=r"(xf[nt][0]), "=r"(xf[nt][1]), "=r"(xf[nt][2]), "=r"(xf[nt][3]) : "r"(addr));
            asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                         : "=r"(xf[nt][4]), "=r"(xf[nt][5]), "=r"(xf[nt][6]), "=r"(xf[nt][7]) : "r"(addr + 16));
          }
          const uint32_t wg[2] = {pk[sl][b][0].x, pk[sl][b][0].y}, wg8[2] = {pk[sl][b][1].x, pk[sl][b][1].y};
          const float s_g = __fmul_rn(sc_g, kInvAlpha), s_g8 = __fmul_rn(sc_g8, kInvAlpha);
          float ct[NT][4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            uint32_t af[4];
            if ((j & 1) == 0) {
              af[0] = lookup<0>(tb, wg[j >> 1]);
              af[1] = lookup<0>(tb, wg8[j >> 1]);
              af[2] = lookup<1>(tb, wg[j >> 1]);
              af[3] = lookup<1>(tb, wg8[j >> 1]);
            } else {
              af[0] = lookup<2>(tb, wg[j >> 1]);
              af[1] = lookup<2>(tb, wg8[j >> 1]);
              af[2] = lookup<3>(tb, wg[j >> 1]);
              af[3] = lookup<3>(tb, wg8[j >> 1]);
            }
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              if (j == 0) mma16816_z(ct[nt], af, xf[nt][0], xf[nt][1]);
              else lora::mma16816(ct[nt], af, xf[nt][2 * j], xf[nt][2 * j + 1]);
            }
          }
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            acc[nt][0] = fmaf(s_g, ct[nt][0], acc[nt][0]);
            acc[nt][1] = fmaf(s_g, ct[nt][1], acc[nt][1]);
            acc[nt][2] = fmaf(s_g8, ct[nt][2], acc[nt][2]);
            acc[nt][3] = fmaf(s_g8, ct[nt][3], acc[nt][3]);
          }
        }
        }
      }
    }
  }

  // Intra-CTA: warps of the same row tile (different k-runs) add in k-run order.
  __syncthreads();  // the activation tile is dead: its space takes the fragments
  {
    float* mine = red + warp * 256;  // [16 rows][16 tokens]
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int tok = 8 * nt + 2 * t;
      mine[g * 16 + tok] = acc[nt][0];
      mine[g * 16 + tok + 1] = acc[nt][1];
      mine[(g + 8) * 16 + tok] = acc[nt][2];
      mine[(g + 8) * 16 + tok + 1] = acc[nt][3];
    }
  }
  __syncthreads();
  const int rows_cta = a.rw * 16;
  for (int e = tid; e < rows_cta * 16; e += kThreads) {
    const int row = e >> 4, tok = e & 15;
    const int tile = row >> 4;
    float v = 0.0f;
    for (int q = 0; q < a.kw; ++q) v += red[(q * a.rw + tile) * 256 + (row & 15) * 16 + tok];
    part[e] = v;
  }
  cluster_finish(part, rows_cta, static_cast<int64_t>(blockIdx.x) * rows_cta, a.N, a.M, a.splits, rank, a.bias,
                 a.la, a.lb, a.r, a.y);
}

// ------------------------------------------------------------------ dX
// dX = dY . deq(W) at M <= 16: output column c = k_in index, reduction over the
// weight rows n.  The decoded weight enters the MMA as its A operand transposed
// (A[c][n] = W[n][c]), which mma.sync cannot take from registers decoded along
// k, so each warp stages its decode in shared memory and reads it back with
// ldmatrix.trans:
//
//   * a warp step covers 32 weight rows x one 64-column block; lane l decodes row
//     n0 + 32 s + l of the block -- its 32 packed bytes from global memory, its own
//     16-entry table fp16(NF4[i] * scale) (the reference decoder's values, one
//     rounding), eight nf4_expand8 -- into the warp's private 32 x 64 fp16 tile
//     (4 KB, 16-byte chunks XOR-swizzled by row: conflict-free stores and
//     ldmatrix), then __syncwarp;
//   * the warp multiplies the tile as 2 (rows) x 4 (column groups) m16n8k16 MMAs
//     per 8 tokens: A from ldmatrix.x4.trans, B = dY^T fragments (two halves of a
//     dY row at adjacent weight rows) loaded straight from global memory (L2),
//     two steps ahead with the packed bytes;
//   * a CTA is one column block x 8 warps on consecutive row runs; the warps'
//     partials add in warp order in shared memory, a cluster of S CTAs along
//     grid.y splits the rows further and cluster_finish adds the ranks in order,
//     then the LoRA term, and stores fp16.  One launch, no workspace, deterministic.
struct DxArgs {
  const __half* dy;       // [M, N] row-major
  int M;
  int64_t N, K;           // reduction length (n_out), output columns (k_in)
  const uint8_t* packed;
  const uint8_t* qabs;
  const float* absmax2;
  const float* code2;
  const float* offset;
  int rows_warp;          // weight rows per warp (multiple of 32); a CTA covers 8 runs
  int splits;             // cluster size along grid.y
  const __half* la;       // [M, r] (LoRA: y += la . lb^T) or null
  const __half* lb;       // [K, r]
  int r;
  __half* y;              // [M, K]
};

constexpr int kDxRows = 32;                     // weight rows per warp step (one per lane)
constexpr int kDxTile = kDxRows * 128;          // decoded tile per warp: 32 rows x 64 fp16
constexpr int kDxSmem = kWarps * kDxTile + 1024 + 64 * 16 * 4;  // tiles | code2 | CTA partial

template <int NT>
__global__ void __launch_bounds__(kThreads, 2) lut_dx_kernel(const DxArgs a) {
  extern __shared__ __align__(128) uint8_t dsm[];
  // Two ring slots (the next step's loads in flight during this one): deeper
  // rings measured slower on the 7B gate dX at M = 1 (26.9 us with 2 slots, 27.8
  // with 3, 29.2 with 4, 28.4 with 5).
  constexpr int kSlots = 2, kAhead = kSlots - 1;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const uint32_t rank = gemm::pair::cluster_rank();
  grid_dependency_wait();  // as in lut_fwd_kernel
  launch_dependents();
  const int64_t cb = blockIdx.x;
  const int64_t kblocks = a.K / 64, row_bytes = a.K / 2;
  const uint32_t tile = smem_addr(dsm + warp * kDxTile);
  float* red = reinterpret_cast<float*>(dsm);  // [warp][64 columns][16 tokens] once the tiles are dead
  float* code2_s = reinterpret_cast<float*>(dsm + kWarps * kDxTile);
  float* part = code2_s + 256;                 // [64 columns][16 tokens]
  for (int i = tid; i < 256; i += kThreads) code2_s[i] = __ldg(a.code2 + i);
  const float off = __ldg(a.offset);

  // This warp's rows [n0, n1); n1 is even (N % 8 == 0, runs are multiples of 32).
  const int64_t n0 = (static_cast<int64_t>(rank) * kWarps + warp) * a.rows_warp;
  int64_t n1 = n0 + a.rows_warp;
  if (n1 > a.N) n1 = a.N;
  const int steps = n1 > n0 ? static_cast<int>((n1 - n0 + kDxRows - 1) / kDxRows) : 0;

  // Register ring: the lane's 32 packed bytes, absmax byte and absmax2 of its row,
  // and the dY^T fragments of the step (rows 16 ks + 2t (+8), tokens g + 8 nt).
  uint4 pw[kSlots][2];
  uint32_t qb[kSlots];
  float a2[kSlots];
  uint32_t yf[kSlots][NT][2][2];
  auto load = [&](int s, int slot) {
    if (s < steps) {
      const int64_t n = n0 + static_cast<int64_t>(s) * kDxRows + lane;
      const bool ok = n < n1;
      // Byte and block offsets of the weight fit 32 bits (checked by the host).
      const uint32_t po = ok ? static_cast<uint32_t>(n * row_bytes + cb * 32) : 0u;
      const uint32_t qo = ok ? static_cast<uint32_t>(n * kblocks + cb) : 0u;
      pw[slot][0] = __ldcs(reinterpret_cast<const uint4*>(a.packed + po));
      pw[slot][1] = __ldcs(reinterpret_cast<const uint4*>(a.packed + po + 16));
      qb[slot] = __ldg(a.qabs + qo);
      a2[slot] = __ldg(a.absmax2 + (qo >> 8));
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const int tok = g + 8 * nt;
#pragma unroll
        for (int ks = 0; ks < 2; ++ks) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int64_t nn = n0 + static_cast<int64_t>(s) * kDxRows + 16 * ks + 2 * t + 8 * h;
            yf[slot][nt][ks][h] = (tok < a.M && nn < n1)
                                      ? __ldg(reinterpret_cast<const uint32_t*>(a.dy + tok * a.N + nn))
                                      : 0u;
          }
        }
      }
    }
  };
#pragma unroll
  for (int q = 0; q < kAhead; ++q) load(q, q);

  float acc[4][NT][4];
#pragma unroll
  for (int mt = 0; mt < 4; ++mt)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) acc[mt][nt][0] = acc[mt][nt][1] = acc[mt][nt][2] = acc[mt][nt][3] = 0.0f;
  __syncthreads();  // code2 table ready

  const uint32_t c2s = smem_addr(code2_s);
  const uint32_t my_row = tile + static_cast<uint32_t>(lane) * 128;
  const uint32_t swz = static_cast<uint32_t>(lane & 7);
  // ldmatrix.x4.trans addresses: matrix j = lane / 8 holds tile rows 8 (j / 2) + 0..7
  // and 16-byte chunk j % 2 of the 16-column group.
  const int lm_row = (lane & 7) + 8 * ((lane >> 3) >> 1), lm_chunk = (lane >> 3) & 1;

  for (int S = 0; S < steps; S += kSlots) {
#pragma unroll
    for (int sl = 0; sl < kSlots; ++sl) {
      const int s = S + sl;
      if (s < steps) {
        load(s + kAhead, (sl + kAhead) % kSlots);
        const bool ok = n0 + static_cast<int64_t>(s) * kDxRows + lane < n1;
        const float scale = ok ? __fadd_rn(__fmul_rn(lds_f32(c2s + qb[sl] * 4), a2[sl]), off) : 0.0f;
        uint32_t L[4], H[4];
        gemm::nf4_table(scale, L, H);
        const uint32_t w[8] = {pw[sl][0].x, pw[sl][0].y, pw[sl][0].z, pw[sl][0].w,
                               pw[sl][1].x, pw[sl][1].y, pw[sl][1].z, pw[sl][1].w};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const uint4 e = gemm::nf4_expand8(w[i], L, H);
          asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};"
                       :: "r"(my_row + ((static_cast<uint32_t>(i) ^ swz) << 4)), "r"(e.x), "r"(e.y), "r"(e.z), "r"(e.w)
                       : "memory");
        }
        __syncwarp();
#pragma unroll
        for (int ks = 0; ks < 2; ++ks) {
          const int row = 16 * ks + lm_row;
#pragma unroll
          for (int mt = 0; mt < 4; ++mt) {
            const int chunk = 2 * mt + lm_chunk;
            uint32_t af[4];
            lora::ldsm_x4_trans(tile + static_cast<uint32_t>(row * 128 + ((chunk ^ (row & 7)) << 4)), af);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) lora::mma16816(acc[mt][nt], af, yf[sl][nt][ks][0], yf[sl][nt][ks][1]);
          }
        }
        __syncwarp();  // every lane's ldmatrix is done before the next step overwrites the tile
      }
    }
  }

  // Warps add in warp order: D rows = columns 16 mt + g (+8), D columns = tokens 8 nt + 2t (+1).
  __syncthreads();  // the tiles are dead: their space takes the warp partials
  {
    float* mine = red + warp * 1024;
#pragma unroll
    for (int mt = 0; mt < 4; ++mt) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const int col = 16 * mt + g, tok = 8 * nt + 2 * t;
        mine[col * 16 + tok] = acc[mt][nt][0];
        mine[col * 16 + tok + 1] = acc[mt][nt][1];
        mine[(col + 8) * 16 + tok] = acc[mt][nt][2];
        mine[(col + 8) * 16 + tok + 1] = acc[mt][nt][3];
      }
    }
  }
  __syncthreads();
  for (int e = tid; e < 64 * 16; e += kThreads) {
    float v = 0.0f;
#pragma unroll
    for (int q = 0; q < kWarps; ++q) v += red[q * 1024 + e];
    part[e] = v;
  }
  cluster_finish(part, 64, cb * 64, a.K, a.M, a.splits, rank, nullptr, a.la, a.lb, a.r, a.y);
}

// ------------------------------------------------------------------ host side
// Programmatic dependent launch only for launches with clusters of at most two
// CTAs.  With larger clusters (one wave of 5-CTA clusters fills each GPC but two
// slots) the next grid's early CTAs take slots the clusters need and push part of
// a grid into a second wave: measured on the 7B projections at M = 1, q dX 8.9 ->
// 11.0 us, gate dX 27.8 -> 31.4 us with PDL, against 0.3-0.4 us gained per launch
// without a cluster.
inline bool pdl_ok(int splits) { return splits <= 2; }

struct FwdPlan {
  int nt, rw, kw, kb_split, splits;
  int64_t groups;
  size_t smem;
};

inline int fwd_slots(int nt) {
  // Two CTAs per SM (the kernel is launched with 2 blocks per SM as bound).
  (void)nt;
  return 2 * device_sm_count();
}

inline FwdPlan fwd_plan(int64_t m, int64_t n, int64_t k, bool exact) {
  FwdPlan best{};
  best.nt = m <= 8 ? 1 : 2;
  const int kb_max = best.nt == 1 ? FwdSmem<1>::kb_max(exact) : FwdSmem<2>::kb_max(exact);
  const int64_t kblocks = k / 64, row_tiles = (n + 15) / 16;
  const int slots = fwd_slots(best.nt);
  double best_cost = 1e30;
  for (int s = 1; s <= kMaxSplits; ++s) {
    const int64_t kb = ((kblocks + s - 1) / s + kGroup - 1) / kGroup * kGroup;
    if (kb > kb_max) continue;
    const int64_t splits = (kblocks + kb - 1) / kb;
    for (int rw : {8, 4, 2, 1}) {
      const int kw = kWarps / rw;
      const int64_t groups = (row_tiles + rw - 1) / rw;
      const int64_t ctas = groups * splits;
      const int64_t run = ((kb + kw - 1) / kw + kGroup - 1) / kGroup * kGroup;
      const int64_t waves = (ctas + slots - 1) / slots;
      // Per CTA: table build + activation tile + reduction, about two blocks' time.
      const double cost = static_cast<double>(waves) * static_cast<double>(run + 2);
      if (cost < best_cost - 1e-9) {
        best_cost = cost;
        best.rw = rw;
        best.kw = kw;
        best.kb_split = static_cast<int>(kb);
        best.splits = static_cast<int>(splits);
        best.groups = groups;
      }
    }
  }
  best.smem = best.nt == 1 ? FwdSmem<1>::bytes(best.kb_split, exact) : FwdSmem<2>::bytes(best.kb_split, exact);
  return best;
}

inline bool fwd_ok(int64_t m, int64_t n, int64_t k, bool exact) {
  if (m < 1 || m > 16 || k % (64 * kGroup) != 0 || n * (k / 2) >= (int64_t(1) << 32)) return false;
  if (!exact && k > kMaxReduction) return false;
  const int kb_max = m <= 8 ? FwdSmem<1>::kb_max(exact) : FwdSmem<2>::kb_max(exact);
  return k / 64 <= static_cast<int64_t>(kMaxSplits) * kb_max;
}

template <int NT, bool EXACT>
inline int launch_fwd(const FwdPlan& pl, const FwdArgs& a, cudaStream_t st) {
  static std::mutex mu;
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lock(mu);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
      cudaError_t e = cudaFuncSetAttribute(lut_fwd_kernel<NT, EXACT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(FwdSmem<NT>::bytes(FwdSmem<NT>::kb_max(EXACT), EXACT)));
      if (e != cudaSuccess) return fail(SB_ECUDA, std::string("lut fwd smem attribute: ") + cudaGetErrorString(e));
      configured[dev] = true;
    }
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(pl.groups), static_cast<unsigned>(pl.splits), 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = static_cast<unsigned>(pl.splits);
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_ok(pl.splits) ? 2 : 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, lut_fwd_kernel<NT, EXACT>, a);
  if (e != cudaSuccess) return fail(SB_ECUDA, std::string("lut_fwd_kernel launch: ") + cudaGetErrorString(e));
  count_launch();
  return check_launch("lut_fwd_kernel");
}

inline int run_fwd(const uint16_t* act, int64_t m, const sb_nf4_weight& w, const uint16_t* bias,
                   const uint16_t* lora_a, const uint16_t* lora_b, int r, uint16_t* out, bool exact,
                   cudaStream_t st) {
  const FwdPlan pl = fwd_plan(m, w.n_out, w.k_in, exact);
  FwdArgs a{};
  a.x = reinterpret_cast<const __half*>(act);
  a.M = static_cast<int>(m);
  a.K = w.k_in;
  a.N = w.n_out;
  a.packed = w.packed;
  a.qabs = w.qabs;
  a.absmax2 = w.absmax2;
  a.code2 = w.code2;
  a.offset = w.offset;
  a.rw = pl.rw;
  a.kw = pl.kw;
  a.kb_split = pl.kb_split;
  a.splits = pl.splits;
  a.bias = reinterpret_cast<const __half*>(bias);
  a.la = reinterpret_cast<const __half*>(lora_a);
  a.lb = reinterpret_cast<const __half*>(lora_b);
  a.r = r;
  a.y = reinterpret_cast<__half*>(out);
  if (exact) return pl.nt == 1 ? launch_fwd<1, true>(pl, a, st) : launch_fwd<2, true>(pl, a, st);
  return pl.nt == 1 ? launch_fwd<1, false>(pl, a, st) : launch_fwd<2, false>(pl, a, st);
}

struct DxPlan {
  int nt, rows_warp, splits;
  int64_t col_blocks;
};

// Work split of the dX kernel: one CTA per 64-column block and cluster rank; the
// cluster size S fills the two CTA slots per SM (at most 8 ranks), each of the
// 8 S warps of a column block taking an equal run of weight rows (a multiple of 32).
inline DxPlan dx_plan(int64_t m, int64_t n, int64_t k) {
  DxPlan p{};
  p.nt = m <= 8 ? 1 : 2;
  p.col_blocks = k / 64;
  int64_t s = (2 * static_cast<int64_t>(device_sm_count())) / p.col_blocks;
  if (s < 1) s = 1;
  if (s > kMaxSplits) s = kMaxSplits;
  const int64_t runs = s * kWarps;
  const int64_t rows = ((n + runs - 1) / runs + kDxRows - 1) / kDxRows * kDxRows;
  p.rows_warp = static_cast<int>(rows);
  p.splits = static_cast<int>((n + kWarps * rows - 1) / (kWarps * rows));
  return p;
}

inline bool dx_ok(int64_t m, int64_t n, int64_t k) {
  return m >= 1 && m <= 16 && k % 64 == 0 && n % 8 == 0 && n * (k / 2) < (int64_t(1) << 32) &&
         k / 64 < (int64_t(1) << 31);
}

template <int NT>
inline int launch_dx(const DxPlan& pl, const DxArgs& a, cudaStream_t st) {
  static std::mutex mu;
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lock(mu);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
      cudaError_t e = cudaFuncSetAttribute(lut_dx_kernel<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, kDxSmem);
      if (e != cudaSuccess) return fail(SB_ECUDA, std::string("lut dx smem attribute: ") + cudaGetErrorString(e));
      configured[dev] = true;
    }
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(pl.col_blocks), static_cast<unsigned>(pl.splits), 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = kDxSmem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = static_cast<unsigned>(pl.splits);
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_ok(pl.splits) ? 2 : 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, lut_dx_kernel<NT>, a);
  if (e != cudaSuccess) return fail(SB_ECUDA, std::string("lut_dx_kernel launch: ") + cudaGetErrorString(e));
  count_launch();
  return check_launch("lut_dx_kernel");
}

inline int run_dx(const uint16_t* dy, int64_t m, const sb_nf4_weight& w, const uint16_t* lora_a,
                  const uint16_t* lora_b, int r, uint16_t* out, cudaStream_t st) {
  const DxPlan pl = dx_plan(m, w.n_out, w.k_in);
  DxArgs a{};
  a.dy = reinterpret_cast<const __half*>(dy);
  a.M = static_cast<int>(m);
  a.N = w.n_out;
  a.K = w.k_in;
  a.packed = w.packed;
  a.qabs = w.qabs;
  a.absmax2 = w.absmax2;
  a.code2 = w.code2;
  a.offset = w.offset;
  a.rows_warp = pl.rows_warp;
  a.splits = pl.splits;
  a.la = reinterpret_cast<const __half*>(lora_a);
  a.lb = reinterpret_cast<const __half*>(lora_b);
  a.r = r;
  a.y = reinterpret_cast<__half*>(out);
  return pl.nt == 1 ? launch_dx<1>(pl, a, st) : launch_dx<2>(pl, a, st);
}

}  // namespace lut
}  // namespace sb
