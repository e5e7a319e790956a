// Host side of the tcgen05 GEMM: tensor maps, launch configuration, and the
// NF4-linear / cross-entropy drivers exported through the C ABI.
#pragma once

#include <cstdlib>
#include <mutex>
#include <string>

#include "common.cuh"
#include "gemm_pair.cuh"
#include "gemm_sm100.cuh"

namespace sb {
namespace gemm {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
    }
  });
  return fn;
}

// 2-D row-major tensor [outer, inner] with a row pitch in bytes; box {box_inner, box_outer}.
inline int make_map(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t inner,
                    uint64_t outer, uint64_t pitch_bytes, uint32_t box_inner, uint32_t box_outer,
                    CUtensorMapSwizzle swz) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(SB_ECUDA, "cuTensorMapEncodeTiled entry point unavailable");
  if (!aligned(base, 16) || pitch_bytes % 16 != 0) return fail(SB_EINVAL, "TMA operand not 16-byte aligned");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {pitch_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(SB_ECUDA, "cuTensorMapEncodeTiled failed (" + std::to_string(int(r)) + ")");
  return SB_OK;
}

inline CUtensorMapSwizzle lora_swizzle(int r) {
  return r == 16 ? CU_TENSOR_MAP_SWIZZLE_32B : (r == 32 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B);
}

// Schedule override from the environment: SB_STREAMK=0 (whole tiles), 1 (stream-K)
// or unset / "auto" (the heuristic below).  Read per call, so the workspace
// query and the launch of one configuration agree and tests can exercise both.
inline int streamk_override() {
  const char* e = std::getenv("SB_STREAMK");
  if (!e || !*e || std::string(e) == "auto") return -1;
  return std::string(e) == "0" ? 0 : 1;
}

// Stream-K pays off when whole tiles would leave the last wave mostly idle and a
// tile is long enough (>= 64 k-blocks) to amortise the partial-tile write and
// fix-up; measured on B200, short reductions (24 k-blocks) lose more to the
// fix-up traffic than they gain from balance.
inline bool want_streamk(int64_t tiles, int64_t k_blocks, int sms) {
  if (tiles <= 0 || k_blocks < 4) return false;
  if (streamk_override() >= 0) return streamk_override() == 1;
  if (k_blocks < 64) return false;
  const int64_t waves = (tiles + sms - 1) / sms;
  return static_cast<double>(tiles) / static_cast<double>(waves * sms) < 0.9;
}

inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// Stream-K grid: every CTA gets at least half a tile of k-iterations, so a tile is
// shared by at most about two CTAs and the fix-up stays cheap.
inline int streamk_grid(int64_t tiles, int64_t k_blocks, int sms) {
  int64_t g = 2 * tiles;
  if (g > sms) g = sms;
  const int64_t total = tiles * k_blocks;
  if (g > total) g = total;
  return static_cast<int>(g < 1 ? 1 : g);
}

// Scratch of a stream-K launch: two fp32 partial tiles per CTA, then one counter per tile.
inline size_t streamk_bytes(int grid, int tile_rows, int tile_cols, int64_t tiles) {
  return align256(static_cast<size_t>(grid) * 2 * tile_rows * tile_cols * sizeof(float)) +
         align256(static_cast<size_t>(tiles) * sizeof(int));
}

template <int BMODE, int EMODE, int MSUB, int BN, int STAGES>
int launch(const CUtensorMap& a, const CUtensorMap& b, const CUtensorMap& la,
           const CUtensorMap& lb, Params p, cudaStream_t stream, const char* name) {
  using C = Cfg<BMODE, MSUB, BN, STAGES>;
  auto kern = gemm_kernel<BMODE, EMODE, MSUB, BN, STAGES>;
  static std::mutex mu;
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lock(mu);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
      if (e != cudaSuccess) return fail(SB_ECUDA, std::string(name) + " smem attribute: " + cudaGetErrorString(e));
      configured[dev] = true;
    }
  }
  const int tiles = p.m_tiles * p.n_tiles;
  if (tiles == 0) return SB_OK;
  const int sms = device_sm_count();
  const int units = tiles * (p.ksplit > 1 ? p.ksplit : 1);
  int grid = units < sms ? units : sms;
  if (p.streamk) grid = streamk_grid(tiles, p.k_blocks, sms);
  kern<<<grid, C::kThreads, C::kSmemBytes, stream>>>(a, b, la, lb, p);
  count_launch();
  return check_launch(name);
}

// ----------------------------------------------------------------- 2-SM pair launch
constexpr int kPairStages = 6;         // dX, and the stream-K forward
constexpr int kPairFwdTileStages = 5;  // whole-tile forward (leaves room for store staging; 4 code slots)
constexpr int kPairMlpFwdStages = 4;   // gate/up + SwiGLU forward (three staging boxes per warp; 5 measured slower)
constexpr int kPairMlpBwdStages = 4;   // down dX + SwiGLU derivatives (gate/up box sets; 5 measured slower)

template <int BMODE, int EMODE, int STAGES, bool SK, int WSEL = 0>
inline int configure_pair(const char* name) {
  using C = pair::PairCfg<BMODE, STAGES, EMODE>;
  static std::mutex mu;
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(pair::pair_kernel<BMODE, EMODE, STAGES, SK, WSEL>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
    if (e != cudaSuccess) return fail(SB_ECUDA, std::string(name) + " smem attribute: " + cudaGetErrorString(e));
    configured[dev] = true;
  }
  return SB_OK;
}

template <int BMODE, int EMODE, int STAGES>
inline cudaLaunchConfig_t pair_config(int grid, cudaStream_t stream, cudaLaunchAttribute* attr) {
  using C = pair::PairCfg<BMODE, STAGES, EMODE>;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
  cfg.blockDim = dim3(C::kThreads, 1, 1);
  cfg.dynamicSmemBytes = C::kSmemBytes;
  cfg.stream = stream;
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  // Programmatic dependent launch: the kernel's set-up may overlap the previous
  // kernel of the stream (it waits for it before touching global memory).
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cfg;
}

// CTA pairs that can be resident at once on the current device (74 on a full
// B200: one pair per TPC), queried once per device.
inline int pair_slots() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return device_sm_count() / 2;
  static std::mutex mu;
  static int cached[64] = {0};
  {
    std::lock_guard<std::mutex> lock(mu);
    if (cached[dev] > 0) return cached[dev];
  }
  int n = 0;
  if (configure_pair<kNF4Fwd, kStoreF16, kPairFwdTileStages, false>("nf4_pair_fwd") == SB_OK) {
    cudaLaunchAttribute attr[2];
    cudaLaunchConfig_t cfg = pair_config<kNF4Fwd, kStoreF16, kPairFwdTileStages>(2, nullptr, attr);
    if (cudaOccupancyMaxActiveClusters(&n, pair::pair_kernel<kNF4Fwd, kStoreF16, kPairFwdTileStages, false, 0>, &cfg) !=
        cudaSuccess) {
      cudaGetLastError();
      n = 0;
    }
  }
  if (n <= 0) n = device_sm_count() / 2;
  std::lock_guard<std::mutex> lock(mu);
  cached[dev] = n;
  return n;
}

// b2 / y2: the second weight's packed-code map (gate/up forward) and the second
// output map (the SwiGLU forward's activation); any valid map otherwise.
template <int BMODE, int EMODE, int STAGES, bool SK, int WSEL = 0>
int launch_pair_sk(const CUtensorMap& a, const CUtensorMap& b, const CUtensorMap& la, const CUtensorMap& lb,
                   const CUtensorMap& y, Params p, int grid, cudaStream_t stream, const char* name,
                   const CUtensorMap* b2 = nullptr, const CUtensorMap* y2 = nullptr) {
  if (int rc = configure_pair<BMODE, EMODE, STAGES, SK, WSEL>(name)) return rc;
  if (grid <= 0) return SB_OK;
  cudaLaunchAttribute attr[2];
  cudaLaunchConfig_t cfg = pair_config<BMODE, EMODE, STAGES>(grid, stream, attr);
  cudaError_t e = cudaLaunchKernelEx(&cfg, pair::pair_kernel<BMODE, EMODE, STAGES, SK, WSEL>, a, b, la, lb, y,
                                     b2 ? *b2 : b, y2 ? *y2 : y, p);
  if (e != cudaSuccess) return fail(SB_ECUDA, std::string(name) + " launch: " + cudaGetErrorString(e));
  count_launch();
  return check_launch(name);
}

template <int BMODE, int EMODE, int STAGES, int WSEL = 0>
int launch_pair(const CUtensorMap& a, const CUtensorMap& b, const CUtensorMap& la, const CUtensorMap& lb,
                const CUtensorMap& y, Params p, int grid, cudaStream_t stream, const char* name) {
  return p.streamk ? launch_pair_sk<BMODE, EMODE, STAGES, true, WSEL>(a, b, la, lb, y, p, grid, stream, name)
                   : launch_pair_sk<BMODE, EMODE, STAGES, false, WSEL>(a, b, la, lb, y, p, grid, stream, name);
}

// ----------------------------------------------------------------- NF4 linear
constexpr int kNF4Msub = 2, kNF4BN = 128, kNF4Stages = 4;

// Kernel choice for the NF4 linear: SB_PAIR=1 forces the 2-SM pair kernel, 0 the
// one-SM kernel; unset or "auto" takes the pair kernel, which measured faster on
// every Qwen2.5 layer shape at 3300 tokens (forward and dX; B200).  Read per call
// so the workspace query and the launch of one configuration agree.
inline int pair_override() {
  const char* e = std::getenv("SB_PAIR");
  if (!e || !*e || std::string(e) == "auto") return -1;
  return std::string(e) == "0" ? 0 : 1;
}

inline bool want_pair(int64_t m, int64_t width) {
  const int o = pair_override();
  if (o >= 0) return o == 1;
  (void)m;
  (void)width;
  return true;
}

inline bool nf4_tc_shape_ok(int64_t m, int64_t n_out, int64_t k_in, bool dx) {
  if (m <= 0 || n_out <= 0 || k_in <= 0) return false;
  if (k_in % 64 != 0) return false;                  // blocks stay inside weight rows
  if (dx && (n_out % 8 != 0)) return false;          // dY rows must be 16-byte pitched
  if (m > 0x7fffffffLL || n_out > 0x7fffffffLL || k_in > 0x7fffffffLL) return false;
  return true;
}

struct NF4Plan {
  int64_t m_tiles, n_tiles, k_blocks;
  bool streamk;
  bool pair;     // 2-SM pair kernel (256 x 256 tiles over CTA pairs)
  int grid;      // CTAs (pair kernel; the one-SM launch sizes its own grid)
  size_t workspace;
};

inline NF4Plan nf4_plan(int64_t m, int64_t n_out, int64_t k_in, bool dx) {
  NF4Plan pl{};
  const int64_t red = dx ? n_out : k_in, width = dx ? k_in : n_out;
  if (want_pair(m, width)) {
    pl.pair = true;
    pl.m_tiles = (m + pair::kTileM - 1) / pair::kTileM;
    pl.n_tiles = (width + pair::kTileN - 1) / pair::kTileN;
    pl.k_blocks = (red + 63) / 64;
    const int slots = pair_slots();
    const int64_t tiles = pl.m_tiles * pl.n_tiles;
    pl.streamk = want_streamk(tiles, pl.k_blocks, slots);
    const int pairs = pl.streamk ? streamk_grid(tiles, pl.k_blocks, slots)
                                 : static_cast<int>(tiles < slots ? tiles : slots);
    pl.grid = 2 * pairs;
    pl.workspace = pl.streamk ? align256(static_cast<size_t>(pl.grid) * 2 * pair::kSlotF4 * sizeof(float4)) +
                                    align256(static_cast<size_t>(tiles) * 2 * sizeof(int))
                              : 0;
    return pl;
  }
  pl.m_tiles = (m + kNF4Msub * 128 - 1) / (kNF4Msub * 128);
  pl.n_tiles = (width + kNF4BN - 1) / kNF4BN;
  pl.k_blocks = (red + 63) / 64;
  const int sms = device_sm_count();
  pl.streamk = want_streamk(pl.m_tiles * pl.n_tiles, pl.k_blocks, sms);
  pl.workspace = pl.streamk ? streamk_bytes(streamk_grid(pl.m_tiles * pl.n_tiles, pl.k_blocks, sms),
                                            kNF4Msub * 128, kNF4BN, pl.m_tiles * pl.n_tiles) : 0;
  return pl;
}

inline int nf4_linear_tc(bool dx, const uint16_t* act, int64_t m, const sb_nf4_weight& w,
                         const uint16_t* bias, const uint16_t* lora_a, const uint16_t* lora_b,
                         int r, uint16_t* out, void* workspace, size_t workspace_bytes,
                         cudaStream_t stream) {
  const NF4Plan pl = nf4_plan(m, w.n_out, w.k_in, dx);
  if (pl.workspace > 0 && (!workspace || workspace_bytes < pl.workspace)) {
    return fail(SB_EWORKSPACE, "NF4 linear needs " + std::to_string(pl.workspace) + " workspace bytes");
  }
  const int64_t red = dx ? w.n_out : w.k_in;    // reduction length
  const int64_t width = dx ? w.k_in : w.n_out;  // output columns
  CUtensorMap ta, tb, tla, tlb;
  int rc = make_map(&ta, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, act, red, m, red * 2, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  if (!dx) {
    rc = make_map(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, w.packed, w.k_in / 2, w.n_out, w.k_in / 2, 32, kNF4BN,
                  CU_TENSOR_MAP_SWIZZLE_32B);
  } else {
    rc = make_map(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, w.packed, w.k_in / 2, w.n_out, w.k_in / 2, kNF4BN / 2, 64,
                  CU_TENSOR_MAP_SWIZZLE_64B);
  }
  if (rc) return rc;
  tla = ta;
  tlb = ta;
  if (r > 0) {
    // LoRA boxes: the A rows of one CTA tile and the B rows that CTA holds.
    const uint32_t la_rows = pl.pair ? kTileRows : kNF4Msub * 128;
    const uint32_t lb_rows = pl.pair ? pair::kHalfN : kNF4BN;
    rc = make_map(&tla, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, lora_a, r, m, r * 2, r, la_rows, lora_swizzle(r));
    if (rc) return rc;
    rc = make_map(&tlb, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, lora_b, r, width, r * 2, r, lb_rows, lora_swizzle(r));
    if (rc) return rc;
  }
  Params p{};
  p.M = static_cast<int>(m);
  p.N = static_cast<int>(width);
  p.K = static_cast<int>(red);
  p.m_tiles = static_cast<int>(pl.m_tiles);
  p.n_tiles = static_cast<int>(pl.n_tiles);
  p.k_blocks = static_cast<int>(pl.k_blocks);
  p.lora_r = r;
  if (pl.streamk && pl.pair) {
    p.streamk = 1;
    p.nfast = 1;
    p.partials = static_cast<float*>(workspace);
    p.counters = reinterpret_cast<int*>(static_cast<uint8_t*>(workspace) +
                                        align256(static_cast<size_t>(pl.grid) * 2 * pair::kSlotF4 * sizeof(float4)));
    cudaError_t e = cudaMemsetAsync(p.counters, 0, static_cast<size_t>(pl.m_tiles * pl.n_tiles) * 2 * sizeof(int), stream);
    if (e != cudaSuccess) return fail(SB_ECUDA, std::string("counter reset: ") + cudaGetErrorString(e));
  } else if (pl.streamk) {
    const int sms = device_sm_count();
    p.streamk = 1;
    p.partials = static_cast<float*>(workspace);
    const int grid = streamk_grid(pl.m_tiles * pl.n_tiles, pl.k_blocks, sms);
    p.counters = reinterpret_cast<int*>(static_cast<uint8_t*>(workspace) +
                                        align256(static_cast<size_t>(grid) * 2 * kNF4Msub * 128 * kNF4BN * sizeof(float)));
    cudaError_t e = cudaMemsetAsync(p.counters, 0, static_cast<size_t>(pl.m_tiles * pl.n_tiles) * sizeof(int), stream);
    if (e != cudaSuccess) return fail(SB_ECUDA, std::string("counter reset: ") + cudaGetErrorString(e));
  }
  p.vec_ok = aligned(out, 16) && (width % 8 == 0);
  p.packed = w.packed;
  p.qabs = w.qabs;
  p.absmax2 = w.absmax2;
  p.code2 = w.code2;
  p.offset = w.offset;
  p.w_rows = w.n_out;
  p.w_cols = w.k_in;
  p.out = out;
  p.ldo = width;
  p.bias = reinterpret_cast<const __half*>(bias);
  if (pl.pair) {
    // Output tensor map for the bulk-store epilogue: box 64 columns x 32 rows (one
    // epilogue warp's rows), 128B swizzle; needs 16-byte aligned rows.
    CUtensorMap ty = ta;
    p.store_tma = (aligned(out, 16) && width % 8 == 0) ? 1 : 0;
    if (p.store_tma) {
      rc = make_map(&ty, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, out, width, m, width * 2, 64, 32,
                    CU_TENSOR_MAP_SWIZZLE_128B);
      if (rc) return rc;
    }
    if (!dx) {
      return p.streamk
          ? launch_pair_sk<kNF4Fwd, kStoreF16, kPairStages, true>(ta, tb, tla, tlb, ty, p, pl.grid, stream, "nf4_pair_fwd")
          : launch_pair_sk<kNF4Fwd, kStoreF16, kPairFwdTileStages, false>(ta, tb, tla, tlb, ty, p, pl.grid, stream,
                                                                          "nf4_pair_fwd");
    }
    return launch_pair<kNF4Dx, kStoreF16, kPairStages>(ta, tb, tla, tlb, ty, p, pl.grid, stream, "nf4_pair_dx");
  }
  if (!dx) {
    return launch<kNF4Fwd, kStoreF16, kNF4Msub, kNF4BN, kNF4Stages>(ta, tb, tla, tlb, p, stream, "nf4_gemm_fwd");
  }
  return launch<kNF4Dx, kStoreF16, kNF4Msub, kNF4BN, kNF4Stages>(ta, tb, tla, tlb, p, stream, "nf4_gemm_dx");
}


// ----------------------------------------------------------------- Qwen2 MLP (fused SwiGLU)
// Weight descriptor fields shared by the drivers below.
inline void set_weight(Params& p, const sb_nf4_weight& w) {
  p.packed = w.packed;
  p.qabs = w.qabs;
  p.absmax2 = w.absmax2;
  p.code2 = w.code2;
  p.offset = w.offset;
  p.w_rows = w.n_out;
  p.w_cols = w.k_in;
}

inline void set_second_weight(Params& p, const sb_nf4_weight& w) {
  p.packed2 = w.packed;
  p.qabs2 = w.qabs;
  p.absmax2_2 = w.absmax2;
  p.code2_2 = w.code2;
  p.offset2 = w.offset;
}

inline bool same_shape(const sb_nf4_weight& a, const sb_nf4_weight& b) {
  return a.n_out == b.n_out && a.k_in == b.k_in;
}

// gate_up[m, 2N] = [X . deq(Wg)^T | X . deq(Wu)^T] (+ LoRA), act[m, N] = SwiGLU(gate, up):
// one pair-kernel launch whose tiles hold 128 gate and 128 up columns of the same
// outputs (rank 0 decodes Wg, rank 1 Wu).  lora_a [m, r] is [s X.Ag^T | s X.Au^T]
// and lora_b [2N, r] stacks [Bg | 0] over [0 | Bu] (r = 2 x the adapter rank).
inline int mlp_gate_up(const uint16_t* x, int64_t m, const sb_nf4_weight& wg, const sb_nf4_weight& wu,
                       const uint16_t* lora_a, const uint16_t* lora_b, int r, uint16_t* gate_up, uint16_t* act,
                       cudaStream_t stream) {
  const int64_t n = wg.n_out, k = wg.k_in;
  const int64_t m_tiles = (m + pair::kTileM - 1) / pair::kTileM, n_tiles = n / pair::kHalfN;
  CUtensorMap ta, tb, tb2, tla, tlb, ty, ty2;
  int rc = make_map(&ta, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, x, k, m, k * 2, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B);
  if (!rc) rc = make_map(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, wg.packed, k / 2, n, k / 2, 32, pair::kHalfN,
                         CU_TENSOR_MAP_SWIZZLE_32B);
  if (!rc) rc = make_map(&tb2, CU_TENSOR_MAP_DATA_TYPE_UINT8, wu.packed, k / 2, n, k / 2, 32, pair::kHalfN,
                         CU_TENSOR_MAP_SWIZZLE_32B);
  if (!rc) rc = make_map(&ty, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, gate_up, 2 * n, m, 4 * n, 64, 32,
                         CU_TENSOR_MAP_SWIZZLE_128B);
  if (!rc) rc = make_map(&ty2, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, act, n, m, 2 * n, 64, 32,
                         CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  tla = ta;
  tlb = ta;
  if (r > 0) {
    rc = make_map(&tla, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, lora_a, r, m, r * 2, r, kTileRows, lora_swizzle(r));
    if (!rc) rc = make_map(&tlb, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, lora_b, r, 2 * n, r * 2, r, pair::kHalfN,
                           lora_swizzle(r));
    if (rc) return rc;
  }
  Params p{};
  p.M = static_cast<int>(m);
  p.N = static_cast<int>(n);
  p.K = static_cast<int>(k);
  p.m_tiles = static_cast<int>(m_tiles);
  p.n_tiles = static_cast<int>(n_tiles);
  p.k_blocks = static_cast<int>(k / 64);
  p.lora_r = r;
  p.store_tma = 1;
  p.vec_ok = 1;
  set_weight(p, wg);
  set_second_weight(p, wu);
  p.out = gate_up;
  p.ldo = 2 * n;
  const int64_t tiles = m_tiles * n_tiles;
  const int slots = pair_slots();
  const int grid = 2 * static_cast<int>(tiles < slots ? tiles : slots);
  return launch_pair_sk<kNF4Fwd, kSwiGLUFwd, kPairMlpFwdStages, false, 1>(ta, tb, tla, tlb, ty, p, grid, stream,
                                                                            "nf4_mlp_gate_up", &tb2, &ty2);
}

// dgate_up[m, 2N] from the down projection's input gradient: dact = dY . deq(Wd) (+ LoRA,
// lora_a [m, r], lora_b [N, r]) rounded to fp16, then the SwiGLU derivatives against
// gate_up[m, 2N] in the epilogue (dgate to [0, N), dup to [N, 2N)).  Whole tiles.
inline int mlp_down_dx(const uint16_t* dy, int64_t m, const sb_nf4_weight& wd, const uint16_t* lora_a,
                       const uint16_t* lora_b, int r, const uint16_t* gate_up, uint16_t* dgate_up,
                       cudaStream_t stream) {
  const int64_t red = wd.n_out, n = wd.k_in;
  const int64_t m_tiles = (m + pair::kTileM - 1) / pair::kTileM, n_tiles = (n + pair::kTileN - 1) / pair::kTileN;
  CUtensorMap ta, tb, tla, tlb, ty, tgu;
  int rc = make_map(&ta, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, dy, red, m, red * 2, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B);
  if (!rc) rc = make_map(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, wd.packed, n / 2, red, n / 2, kNF4BN / 2, 64,
                         CU_TENSOR_MAP_SWIZZLE_64B);
  if (!rc) rc = make_map(&ty, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, dgate_up, 2 * n, m, 4 * n, 64, 32,
                         CU_TENSOR_MAP_SWIZZLE_128B);
  // The epilogue loads the saved gate/up in the same 32-row x 64-column boxes.
  if (!rc) rc = make_map(&tgu, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, gate_up, 2 * n, m, 4 * n, 64, 32,
                         CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  tla = ta;
  tlb = ta;
  if (r > 0) {
    rc = make_map(&tla, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, lora_a, r, m, r * 2, r, kTileRows, lora_swizzle(r));
    if (!rc) rc = make_map(&tlb, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, lora_b, r, n, r * 2, r, pair::kHalfN,
                           lora_swizzle(r));
    if (rc) return rc;
  }
  Params p{};
  p.M = static_cast<int>(m);
  p.N = static_cast<int>(n);
  p.K = static_cast<int>(red);
  p.m_tiles = static_cast<int>(m_tiles);
  p.n_tiles = static_cast<int>(n_tiles);
  p.k_blocks = static_cast<int>((red + 63) / 64);
  p.lora_r = r;
  p.store_tma = 1;
  p.vec_ok = 1;
  set_weight(p, wd);
  p.out = dgate_up;
  p.ldo = 2 * n;
  p.gu = reinterpret_cast<const __half*>(gate_up);
  p.ld_gu = 2 * n;
  const int64_t tiles = m_tiles * n_tiles;
  const int slots = pair_slots();
  const int grid = 2 * static_cast<int>(tiles < slots ? tiles : slots);
  return launch_pair_sk<kNF4Dx, kSwiGLUBwd, kPairMlpBwdStages, false, 0>(ta, tb, tla, tlb, ty, p, grid, stream,
                                                                          "nf4_mlp_down_dx", &tgu, nullptr);
}

// dX[m, K] = dY2[m, 2N] . [deq(W1); deq(W2)] (+ lora_a [m, r] . lora_b[K, r]^T): the input
// gradient of two projections of the same input as one reduction of length 2N.
inline NF4Plan dx2_plan(int64_t m, int64_t n, int64_t k) {
  NF4Plan pl{};
  pl.pair = true;
  pl.m_tiles = (m + pair::kTileM - 1) / pair::kTileM;
  pl.n_tiles = (k + pair::kTileN - 1) / pair::kTileN;
  pl.k_blocks = (2 * n + 63) / 64;
  const int slots = pair_slots();
  const int64_t tiles = pl.m_tiles * pl.n_tiles;
  pl.streamk = want_streamk(tiles, pl.k_blocks, slots);
  const int pairs = pl.streamk ? streamk_grid(tiles, pl.k_blocks, slots) : static_cast<int>(tiles < slots ? tiles : slots);
  pl.grid = 2 * pairs;
  pl.workspace = pl.streamk ? align256(static_cast<size_t>(pl.grid) * 2 * pair::kSlotF4 * sizeof(float4)) +
                                  align256(static_cast<size_t>(tiles) * 2 * sizeof(int))
                            : 0;
  return pl;
}

inline int linear_dx2(const uint16_t* dy2, int64_t m, const sb_nf4_weight& w1, const sb_nf4_weight& w2,
                      const uint16_t* lora_a, const uint16_t* lora_b, int r, uint16_t* dx, void* workspace,
                      size_t workspace_bytes, cudaStream_t stream) {
  const int64_t n = w1.n_out, k = w1.k_in;
  NF4Plan pl = dx2_plan(m, n, k);
  if (pl.workspace > 0 && (!workspace || workspace_bytes < pl.workspace)) {
    return fail(SB_EWORKSPACE, "two-weight dX needs " + std::to_string(pl.workspace) + " workspace bytes");
  }
  CUtensorMap ta, tb, tla, tlb, ty;
  int rc = make_map(&ta, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, dy2, 2 * n, m, 4 * n, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B);
  if (!rc) rc = make_map(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, w1.packed, k / 2, n, k / 2, kNF4BN / 2, 64,
                         CU_TENSOR_MAP_SWIZZLE_64B);
  if (!rc) rc = make_map(&ty, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, dx, k, m, k * 2, 64, 32, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  tla = ta;
  tlb = ta;
  if (r > 0) {
    rc = make_map(&tla, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, lora_a, r, m, r * 2, r, kTileRows, lora_swizzle(r));
    if (!rc) rc = make_map(&tlb, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, lora_b, r, k, r * 2, r, pair::kHalfN,
                           lora_swizzle(r));
    if (rc) return rc;
  }
  Params p{};
  p.M = static_cast<int>(m);
  p.N = static_cast<int>(k);
  p.K = static_cast<int>(2 * n);
  p.m_tiles = static_cast<int>(pl.m_tiles);
  p.n_tiles = static_cast<int>(pl.n_tiles);
  p.k_blocks = static_cast<int>(pl.k_blocks);
  p.k_split = static_cast<int>(n / 64);
  p.lora_r = r;
  p.store_tma = 1;
  p.vec_ok = 1;
  set_weight(p, w1);
  set_second_weight(p, w2);
  p.out = dx;
  p.ldo = k;
  if (pl.streamk) {
    p.streamk = 1;
    p.nfast = 1;
    p.partials = static_cast<float*>(workspace);
    p.counters = reinterpret_cast<int*>(static_cast<uint8_t*>(workspace) +
                                        align256(static_cast<size_t>(pl.grid) * 2 * pair::kSlotF4 * sizeof(float4)));
    cudaError_t e = cudaMemsetAsync(p.counters, 0, static_cast<size_t>(pl.m_tiles * pl.n_tiles) * 2 * sizeof(int),
                                    stream);
    if (e != cudaSuccess) return fail(SB_ECUDA, std::string("counter reset: ") + cudaGetErrorString(e));
  }
  return launch_pair<kNF4Dx, kStoreF16, kPairStages, 2>(ta, tb, tla, tlb, ty, p, pl.grid, stream, "nf4_linear_dx2");
}

}  // namespace gemm
}  // namespace sb
