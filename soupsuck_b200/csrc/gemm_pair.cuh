// Two-SM (cta_group::2) NF4 GEMM for sm_100a: one UMMA spans a CTA pair.
//
//   D[M, N] = A[M, K] . deq(W)^T (+ LA . LB^T) (+ bias)     fp16 x fp16 -> fp32 (TMEM) -> fp16
//
// A cluster of two CTAs (ranks 0 and 1, on the two SMs of one TPC) owns a
// 256 x 256 output tile.  Each CTA holds its own 128 rows of A and decodes its
// own 128 rows of B (output columns n0 + 128 * rank ...) into shared memory;
// the rank-0 CTA issues 256 x 256 x 16 UMMAs (tcgen05.mma.cta_group::2) that
// read both CTAs' operand halves and write each CTA's 128 accumulator rows x
// 256 columns into that CTA's TMEM.  Per SM this is a 128 x 256 x 16 UMMA per
// 8 KB of shared-memory operand reads -- twice the work per byte of the
// 128 x 128 x 16 UMMA of the one-SM kernel -- with half its per-flop A traffic,
// while the NF4 decode per flop stays that of a 256 x 128 one-SM tile.
//
// Per stage and CTA: A 128 x 64 fp16 (16 KB, SW128) and decoded B 128 x 64 fp16
// (16 KB, SW128; K-major for the forward, two MN-major 64-column panels for dX).
// Measured configurations (B200, Qwen2.5 layer shapes):
//   forward: a second producer thread TMA-loads each step's packed codes (4 KB)
//            into a ring of 8 slots of their own (raw_full / raw_empty), so the
//            codes wait in shared memory for their B slot; whole tiles run 4
//            operand stages and stage the output for bulk tensor stores
//            (4 x 32 KB + 32 KB codes + 32-48 KB staging), stream-K runs 6 stages
//            and stores fp16 rows directly (6 x 32 KB + 32 KB);
//   dX:      the decoders load their packed codes straight from global memory one
//            owned step ahead, and the epilogue stages 32 x 64 boxes in shared
//            memory for bulk tensor stores (6 x 32 KB + 32 KB).
// Barriers (same offsets in both CTAs):
//   full[s]      rank 0 only: A bytes of both CTAs (TMA .cta_group::2 loads signal
//                rank 0's barrier; rank 0's producer expects both halves) and 256
//                decoder-thread arrivals, 128 from each CTA -- one barrier, so the
//                UMMA issuer waits once per k-step
//   raw_full[r]  forward, each CTA: code-ring slot r loaded (plain TMA)
//   raw_empty[r] forward, each CTA: slot r read by its 128 decoder threads
//   empty[s]     each CTA: one arrival from rank 0's UMMA commit (multicast to both);
//                waited on by the producer and, for dX, the decoders (B slot)
//   acc_full[b]  each CTA: one arrival from rank 0's commit (multicast to both)
//   acc_empty[b] rank 0 only: 256 epilogue-thread arrivals, 128 from each CTA
// The protocol is the one of the CUDA PTX ISA's cta_group::2 description and of
// CUTLASS's 2-SM UMMA pipelines (a transform producer in each CTA arriving on
// the leader's barrier, the leader's commit released to both CTAs).
//
// Every mbarrier wait is bounded (common.cuh).  Before exit each role proves the
// asynchronous work aimed at its CTA has landed (producer: every stage released
// by the UMMA; rank 0's issuer: both accumulators released by both epilogues),
// then all threads of the pair meet at a cluster barrier and free TMEM.
//
// Reference: the fused NF4 + LoRA forward / input-gradient of
// solution/kernels/nf4_gemm.py (decode rule solution/kernels/nf4.py:41-59).
#pragma once

#include "gemm_sm100.cuh"
#include "swiglu.cuh"

namespace sb {
namespace gemm {
namespace pair {

// ------------------------------------------------------------ cluster PTX wrappers
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// shared::cluster address of the object at shared::cta address `saddr` in CTA `rank`.
__device__ __forceinline__ uint32_t map_to_rank(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}

// All threads of both CTAs (warp-converged).
__device__ __forceinline__ void cluster_sync_all() {
  __syncwarp();
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Arrive on an mbarrier by its shared::cluster address (this CTA's or the peer's),
// with the instruction's default semantics.  A cluster-scope release here would
// be a fence that waits for the thread's outstanding global loads (the decoders'
// scale prefetch), measured as membar stalls; the arrivals ordered by it are
// shared-memory writes made visible to the tensor core by fence.proxy.async.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t caddr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(caddr) : "memory");
}

// 16-byte read-only global load that does not allocate in L1 (L1 shares the
// SRAM and data pipe with shared memory).
__device__ __forceinline__ uint4 ld_stream16(const uint4* ptr) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(ptr));
  return v;
}

// Bulk tensor store of a shared-memory box to global memory (out-of-range rows and
// columns of the box are clipped by the tensor map), tracked by bulk groups.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int32_t x, int32_t y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_addr(src)), "r"(x), "r"(y)
               : "memory");
}
// Pull one 128-byte line toward L2 ahead of its use (no register result, no wait).
__device__ __forceinline__ void prefetch_l2(const void* ptr) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(ptr));
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until at most one committed store group still reads shared memory.
__device__ __forceinline__ void bulk_wait_read1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// Wait until no committed store group still reads shared memory.
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }

// 2-D tiled load into this CTA's shared memory whose byte count completes on the
// rank-0 CTA's mbarrier `leader_bar` (a shared::cluster address).  No multicast.
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t leader_bar,
                                                 int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(leader_bar), "r"(x), "r"(y)
      : "memory");
}

// Converged-warp forms: the whole warp executes them with warp-uniform operands
// and elect.sync picks the single lane that issues.  An issue loop run by one
// lane of a diverged warp measured ~100 cycles per tcgen05 instruction.
__device__ __forceinline__ void umma_f16_pair_warp(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                                   uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// One k-step of four 256 x 256 x 16 UMMAs and the stage's commit, issued by one
// elected lane in one sequence: the descriptors of steps 1-3 advance by a_step /
// b_step in their 16-byte address field, the first UMMA accumulates when
// `accumulate` is set and the others always.  With the issue spread over separate
// elect.sync blocks each UMMA cost ~100 cycles of the issuing warp, more than a
// quarter of a 256 x 256 x 64 k-step's tensor time.
__device__ __forceinline__ void umma_kstep_pair_warp(uint32_t d_tmem, uint32_t a_lo, uint32_t a_hi, uint32_t b_lo,
                                                     uint32_t b_hi, uint32_t a_step, uint32_t b_step, uint32_t idesc,
                                                     uint32_t accumulate, uint32_t commit_bar) {
  // Descriptors as 32-bit halves: the address field lives in the low word, so
  // the steps are 32-bit adds and the high words are loop constants.
  const uint16_t mask = 3;
  asm volatile(
      "{\n\t.reg .pred p, e, t;\n\t.reg .b32 x1, x2, x3, y1, y2, y3;\n\t"
      ".reg .b64 a0, a1, a2, a3, b0, b1, b2, b3;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "setp.ne.b32 p, %5, 0;\n\t"
      "setp.eq.b32 t, 0, 0;\n\t"
      "add.u32 x1, %1, %6;\n\tadd.u32 x2, x1, %6;\n\tadd.u32 x3, x2, %6;\n\t"
      "add.u32 y1, %3, %7;\n\tadd.u32 y2, y1, %7;\n\tadd.u32 y3, y2, %7;\n\t"
      "mov.b64 a0, {%1, %2};\n\tmov.b64 a1, {x1, %2};\n\tmov.b64 a2, {x2, %2};\n\tmov.b64 a3, {x3, %2};\n\t"
      "mov.b64 b0, {%3, %4};\n\tmov.b64 b1, {y1, %4};\n\tmov.b64 b2, {y2, %4};\n\tmov.b64 b3, {y3, %4};\n\t"
      "@e tcgen05.mma.cta_group::2.kind::f16 [%0], a0, b0, %8, p;\n\t"
      "@e tcgen05.mma.cta_group::2.kind::f16 [%0], a1, b1, %8, t;\n\t"
      "@e tcgen05.mma.cta_group::2.kind::f16 [%0], a2, b2, %8, t;\n\t"
      "@e tcgen05.mma.cta_group::2.kind::f16 [%0], a3, b3, %8, t;\n\t"
      "@e tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%9], %10;\n\t}"
      ::"r"(d_tmem), "r"(a_lo), "r"(a_hi), "r"(b_lo), "r"(b_hi), "r"(accumulate), "r"(a_step), "r"(b_step),
      "r"(idesc), "r"(commit_bar), "h"(mask)
      : "memory");
}

__device__ __forceinline__ void umma_commit_both_warp(uint64_t* bar) {
  const uint16_t mask = 3;
  asm volatile(
      "{\n\t.reg .pred e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;\n\t}" ::"r"(
          smem_addr(bar)),
      "h"(mask)
      : "memory");
}

__device__ __forceinline__ void umma_commit_local_warp(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(smem_addr(bar))
      : "memory");
}

// Bounded wait by lane 0 of a converged warp; the outcome is broadcast so the
// warp's control flow stays uniform.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int err, volatile int* abort, int lane) {
  int ok = 1;
  if (lane == 0) ok = mbar_wait(bar, parity, err, abort) ? 1 : 0;
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

// Issued by the same warp of both CTAs with the same destination offset.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(dst_smem)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// ------------------------------------------------------------ configuration
constexpr int kHalfN = 128;   // B rows (output columns) each CTA decodes per tile
constexpr int kTileN = 256;   // output columns per pair tile
constexpr int kTileM = 256;   // output rows per pair tile (128 per CTA)

template <int BMODE, int STAGES, int EMODE = kStoreF16>
struct PairCfg {
  static constexpr bool kBMN = (BMODE == kNF4Dx);
  static constexpr int kABytes = kTileRows * kBK * 2;      // 16 KB
  static constexpr int kBBytes = kHalfN * kBK * 2;         // 16 KB
  static constexpr bool kRawTma = (BMODE == kNF4Fwd);     // packed codes via TMA + smem
  // Bulk-store epilogue (output staged in shared memory, written by tensor
  // stores of whole 128-byte row segments): dX always; the forward in its
  // 4-stage whole-tile configuration, where it measured 12 % faster than direct
  // row stores (gate projection, T = 3300) -- the 6-stage stream-K forward has
  // no room for the staging and stores directly.
  static constexpr bool kStoreStage = !kRawTma || STAGES <= 5;
  // The forward's packed codes (4 KB per k-step) have their own ring, twice as
  // deep as the operand stages, filled by a second producer thread: a k-step's
  // codes are in shared memory before its B slot frees, so the decode follows the
  // UMMA that released the slot directly instead of waiting for a TMA load issued
  // after it.
  static constexpr int kRawBytes = kRawTma ? kHalfN * kBK / 2 : 0;   // 4 KB
  static constexpr int kRawStages = kRawTma ? (STAGES == 5 ? 4 : 8) : 0;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kTmemCols = 2 * kTileN;             // two accumulators of 256 columns
  // Decoder groups of four warps; k-step i is decoded by group i % kDecGroups.
  // Three groups measured faster except in the 6-stage stream-K forward, whose
  // registers at 640 threads spill (down forward 117 -> 123 us): two there.
  static constexpr int kDecGroups = (BMODE == kNF4Fwd && STAGES == 6) ? 2 : 3;
  static constexpr int kThreads = (8 + 4 * kDecGroups) * 32;
  static constexpr int kBarrierBytes = 1024 + 1024;        // barriers + the code2 table
  // Epilogue staging: per epilogue warp two 32-row x 64-column fp16 boxes (SW128);
  // three for the SwiGLU forward, whose panels go out as gate, up and activation.
  static constexpr int kStoreBoxBytes = 32 * 64 * 2;
  // ... and four (two gate/up sets loaded ahead and rewritten in place) for the
  // SwiGLU backward.
  static constexpr int kBoxes = EMODE == kSwiGLUFwd ? 3 : (EMODE == kSwiGLUBwd ? 4 : 2);
  static constexpr int kStagingBytes = kStoreStage ? 4 * kBoxes * kStoreBoxBytes : 0;
  static constexpr int kSmemBytes =
      STAGES * kStageBytes + kRawStages * kRawBytes + kStagingBytes + kBarrierBytes + 1024;
  static_assert(kSmemBytes <= 232448, "shared memory");
  static_assert(kSmemBytes > 232448 / 2, "one CTA per SM keeps TMEM allocation uncontended");
  static_assert(BMODE == kNF4Fwd || BMODE == kNF4Dx, "NF4 operand modes only");
  static_assert(EMODE != kSwiGLUFwd || (BMODE == kNF4Fwd && kStoreStage), "SwiGLU forward: staged forward");
  static_assert(EMODE != kSwiGLUBwd || BMODE == kNF4Dx, "SwiGLU backward: dX epilogue");
};

// Tile coordinates: m-fastest, or n-fastest when p.nfast is set.  Under the
// stream-K schedule consecutive pairs then hold the N-tiles of one M-tile at k
// positions a few dozen blocks apart, so a long reduction's A operand is reread
// from L2 rather than from DRAM (A of a [3300, 17920] input is 118 MB).
__device__ __forceinline__ int tile_m(const Params& p, int tile) {
  return p.nfast ? tile / p.n_tiles : tile % p.m_tiles;
}
__device__ __forceinline__ int tile_n(const Params& p, int tile) {
  return p.nfast ? tile % p.n_tiles : tile / p.m_tiles;
}

// Stream-K partial slot of one CTA: [chunk 8][float4 8][thread 128], 128 KB.
constexpr int kSlotF4 = (kTileN / 32) * 8 * 128;

// ------------------------------------------------------------ epilogue role
// Warps 4..7 of each CTA: rows m0 + 128 * rank + 32 * (warp % 4) + lane, all 256
// columns of the tile.  Releases go to rank 0's acc_empty.
// STAGE: the kernel has store staging (bulk-store epilogue available).
// tmAux: the kSwiGLUFwd activation map, or the kSwiGLUBwd gate/up map; gu_full:
// that mode's two box-set barriers per epilogue warp.
template <int EMODE, bool SK, bool STAGE>
__device__ __forceinline__ void pair_epilogue(const Params& p, const CUtensorMap* tmY, const CUtensorMap* tmAux,
                                              uint8_t* staging,
                                              uint32_t tmem_base, uint64_t* acc_full,
                                              uint32_t leader_acc_empty, uint64_t* epi_mb, uint64_t* gu_full,
                                              volatile int* abort_flag, volatile int* last_flag, int warp,
                                              int lane, int num_tiles, int rows_valid, int pair_id, int pairs,
                                              uint32_t rank) {
  const int q = warp & 3;
  const int etid = (warp - 4) * 32 + lane;
  const int64_t total = static_cast<int64_t>(num_tiles) * p.k_blocks;
  uint32_t tl = 0, epi_phase = 0, boxes = 0;
  int uidx = 0;
  // This warp's staging boxes; rows of a box are this warp's 32 TMEM lanes.
  // The SwiGLU backward keeps two sets of (gate, up) boxes that its TMA loads
  // fill one panel ahead and that it overwrites in place with (dgate, dup).
  constexpr int kBoxes = EMODE == kSwiGLUFwd ? 3 : (EMODE == kSwiGLUBwd ? 4 : 2);
  constexpr int kBoxBytes = 32 * 64 * 2;
  uint8_t* my_boxes = staging + (warp - 4) * kBoxes * kBoxBytes;
  // kSwiGLUBwd box-set bookkeeping: pc counts this warp's panels; set pc & 1,
  // its barrier phase (pc >> 1) & 1; pending[s]: a load into set s not yet waited.
  uint32_t pc = 0;
  bool pending[2] = {false, false};
  uint64_t* my_gu = gu_full + (warp - 4) * 2;
  auto gu_issue = [&](uint32_t pcx, int col, int row0) {
    const uint32_t set = pcx & 1u;
    if (lane == 0) {
      uint8_t* b = my_boxes + set * 2 * kBoxBytes;
      mbar_arrive_expect_tx(&my_gu[set], 2 * kBoxBytes);
      tma_load_2d(b, tmAux, &my_gu[set], col, row0);
      tma_load_2d(b + kBoxBytes, tmAux, &my_gu[set], p.N + col, row0);
    }
    pending[set] = true;
  };
  // Wait out every load still aimed at this warp's boxes (bounded; used on exit paths).
  auto gu_drain = [&]() {
    volatile int no_abort = 0;
    for (uint32_t d = 0; d < 2; ++d) {
      const uint32_t pcx = pc + d;
      if (pending[pcx & 1u] && lane == 0) mbar_wait(&my_gu[pcx & 1u], (pcx >> 1) & 1u, kErrWaitDrain, &no_abort);
      pending[pcx & 1u] = false;
    }
    __syncwarp();
  };
  UnitIter iter(p, num_tiles, pair_id, pairs);
  Unit u;
  while (iter.next(u)) {
    const int mt = tile_m(p, u.tile), nt = tile_n(p, u.tile);
    const int m0 = mt * kTileM, n0 = nt * kTileN;
    if (m0 >= rows_valid) continue;
    const int buf = tl & 1;
    const uint32_t aph = (tl >> 1) & 1;
    if constexpr (EMODE == kSwiGLUBwd) {
      // Panel 0's gate/up boxes do not depend on the accumulator: request them
      // before waiting for it (the other box set may still feed the previous
      // panel's stores; this set's last stores must have read it).
      const int npanels = (p.N - n0 < kTileN ? p.N - n0 : kTileN) / 64;
      if (npanels > 0) {
        if (lane == 0) bulk_wait_read1();
        __syncwarp();
        gu_issue(pc, n0, m0 + static_cast<int>(rank) * kTileRows + q * 32);
      }
      if (!mbar_wait(&acc_full[buf], aph, kErrWaitAccFull, abort_flag)) {
        gu_drain();
        break;
      }
    } else if (!mbar_wait(&acc_full[buf], aph, kErrWaitAccFull, abort_flag)) {
      break;
    }
    tc_fence_after();
    const uint32_t tacc = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + buf * kTileN;
    const int row = m0 + static_cast<int>(rank) * kTileRows + q * 32 + lane;
    if constexpr (EMODE == kSwiGLUFwd) {
      // Gate/up tile: accumulator columns [0, 128) are gate and [128, 256) up for
      // output columns nt*128 .. +128.  Per 64-column panel the warp stages fp16
      // gate, up and act = SwiGLU(gate, up) (computed from the rounded gate/up, as
      // the reference's element-wise kernel sees them) and stores the three boxes:
      // gate and up into the [M, 2N] buffer (up at column N + c), act into [M, N].
      const int row0 = m0 + static_cast<int>(rank) * kTileRows + q * 32;
      const int oc0 = nt * kHalfN;
      const uint32_t swz = static_cast<uint32_t>(lane & 7);
      uint8_t* box_g = my_boxes;
      uint8_t* box_u = my_boxes + 32 * 64 * 2;
      uint8_t* box_a = my_boxes + 2 * 32 * 64 * 2;
#pragma unroll 1
      for (int panel = 0; panel < kHalfN / 64; ++panel) {
        // The previous panel's stores must have finished reading the three boxes.
        if (lane == 0) bulk_wait_read0();
        __syncwarp();
#pragma unroll 1
        for (int half = 0; half < 2; ++half) {
          uint32_t vg[32], vu[32];
          tmem_ld32(tacc + panel * 64 + half * 32, vg);
          tmem_ld32(tacc + kHalfN + panel * 64 + half * 32, vu);
          tmem_ld_wait();
          uint32_t hg[16], hu[16], ha[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            __half2 g2 = __floats2half2_rn(__uint_as_float(vg[2 * j]), __uint_as_float(vg[2 * j + 1]));
            __half2 u2 = __floats2half2_rn(__uint_as_float(vu[2 * j]), __uint_as_float(vu[2 * j + 1]));
            const float2 gf = __half22float2(g2), uf = __half22float2(u2);
            __half2 a2 = __floats2half2_rn(swiglu::forward(gf.x, uf.x), swiglu::forward(gf.y, uf.y));
            hg[j] = *reinterpret_cast<uint32_t*>(&g2);
            hu[j] = *reinterpret_cast<uint32_t*>(&u2);
            ha[j] = *reinterpret_cast<uint32_t*>(&a2);
          }
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const uint32_t off = lane * 128 + ((static_cast<uint32_t>(half * 4 + c) ^ swz) << 4);
            *reinterpret_cast<uint4*>(box_g + off) = make_uint4(hg[4 * c], hg[4 * c + 1], hg[4 * c + 2], hg[4 * c + 3]);
            *reinterpret_cast<uint4*>(box_u + off) = make_uint4(hu[4 * c], hu[4 * c + 1], hu[4 * c + 2], hu[4 * c + 3]);
            *reinterpret_cast<uint4*>(box_a + off) = make_uint4(ha[4 * c], ha[4 * c + 1], ha[4 * c + 2], ha[4 * c + 3]);
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(tmY, box_g, oc0 + panel * 64, row0);
          tma_store_2d(tmY, box_u, p.N + oc0 + panel * 64, row0);
          tma_store_2d(tmAux, box_a, oc0 + panel * 64, row0);
          bulk_commit();
        }
      }
      tc_fence_before();
      mbar_arrive_cluster(leader_acc_empty + 8u * buf);
    } else if constexpr (EMODE == kSwiGLUBwd) {
      // Down-projection dX tile: the accumulator is dL/d(act) for columns
      // n0 .. n0+256 of this CTA's 128 rows.  Rounded to fp16 (the down
      // projection's input-gradient dtype), it meets the saved gate / up values
      // of the same positions, which TMA has brought into this warp's box set
      // one panel ahead; dgate and dup overwrite them in place and go out to
      // columns [0, N) and [N, 2N) of the [M, 2N] output.  Rows past M load
      // zeros and are clipped from the stores; N is a multiple of 64.
      const int row0 = m0 + static_cast<int>(rank) * kTileRows + q * 32;
      const uint32_t swz = static_cast<uint32_t>(lane & 7);
      const int npanels = (p.N - n0 < kTileN ? p.N - n0 : kTileN) / 64;
      bool ok_tile = true;
#pragma unroll 1
      for (int panel = 0; panel < npanels; ++panel) {
        const int c_panel = n0 + panel * 64;
        if (panel + 1 < npanels) {
          // The next panel's set last fed the previous panel's stores.
          if (lane == 0) bulk_wait_read0();
          __syncwarp();
          gu_issue(pc + 1, c_panel + 64, row0);
        }
        const uint32_t set = pc & 1u;
        if (!warp_wait(&my_gu[set], (pc >> 1) & 1u, kErrWaitFull, abort_flag, lane)) {
          ok_tile = false;
          break;
        }
        pending[set] = false;
        uint8_t* box_g = my_boxes + set * 2 * kBoxBytes;
        uint8_t* box_u = box_g + kBoxBytes;
#pragma unroll 1
        for (int half = 0; half < 2; ++half) {
          uint32_t v[32];
          tmem_ld32(tacc + panel * 64 + half * 32, v);
          tmem_ld_wait();
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const uint32_t off = lane * 128 + ((static_cast<uint32_t>(half * 4 + c) ^ swz) << 4);
            uint4 gw = *reinterpret_cast<const uint4*>(box_g + off);
            uint4 uw = *reinterpret_cast<const uint4*>(box_u + off);
            const __half2* g2 = reinterpret_cast<const __half2*>(&gw);
            const __half2* u2 = reinterpret_cast<const __half2*>(&uw);
            uint32_t hdg[4], hdu[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const int e = 8 * c + 2 * j;
              const float2 da = __half22float2(__floats2half2_rn(__uint_as_float(v[e]), __uint_as_float(v[e + 1])));
              const float2 gf = __half22float2(g2[j]), uf = __half22float2(u2[j]);
              float dg0, du0, dg1, du1;
              swiglu::backward(gf.x, uf.x, da.x, dg0, du0);
              swiglu::backward(gf.y, uf.y, da.y, dg1, du1);
              __half2 dg = __floats2half2_rn(dg0, dg1), du = __floats2half2_rn(du0, du1);
              hdg[j] = *reinterpret_cast<uint32_t*>(&dg);
              hdu[j] = *reinterpret_cast<uint32_t*>(&du);
            }
            *reinterpret_cast<uint4*>(box_g + off) = make_uint4(hdg[0], hdg[1], hdg[2], hdg[3]);
            *reinterpret_cast<uint4*>(box_u + off) = make_uint4(hdu[0], hdu[1], hdu[2], hdu[3]);
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(tmY, box_g, c_panel, row0);
          tma_store_2d(tmY, box_u, p.N + c_panel, row0);
          bulk_commit();
        }
        ++pc;
      }
      if (!ok_tile) {
        gu_drain();
        tc_fence_before();
        mbar_arrive_cluster(leader_acc_empty + 8u * buf);
        break;
      }
      tc_fence_before();
      mbar_arrive_cluster(leader_acc_empty + 8u * buf);
    } else if (STAGE && (!SK || (u.k0 == 0 && u.k1 == p.k_blocks)) && p.store_tma) {
      // fp32 (+ bias) -> fp16, staged per 64-column panel into a 128B-swizzled box
      // and written by one bulk tensor store: every global write is a full
      // 128-byte row segment instead of 32 scattered 16-byte pieces per warp store.
      const int row0 = m0 + static_cast<int>(rank) * kTileRows + q * 32;
#pragma unroll 1
      for (int panel = 0; panel < kTileN / 64; ++panel) {
        // The store issued from this box two panels ago must have finished reading it.
        if (lane == 0) bulk_wait_read1();
        __syncwarp();
        uint8_t* box = my_boxes + (boxes & 1) * (32 * 64 * 2);
        const uint32_t swz = static_cast<uint32_t>(lane & 7);
#pragma unroll 1
        for (int half = 0; half < 2; ++half) {
          uint32_t v[32];
          tmem_ld32(tacc + panel * 64 + half * 32, v);
          tmem_ld_wait();
          const int col0 = n0 + panel * 64 + half * 32;
          uint32_t h[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            float f0 = __uint_as_float(v[2 * j]), f1 = __uint_as_float(v[2 * j + 1]);
            if (p.bias) {
              if (col0 + 2 * j < p.N) f0 = __fadd_rn(f0, __half2float(p.bias[col0 + 2 * j]));
              if (col0 + 2 * j + 1 < p.N) f1 = __fadd_rn(f1, __half2float(p.bias[col0 + 2 * j + 1]));
            }
            __half2 t = __floats2half2_rn(f0, f1);
            h[j] = *reinterpret_cast<uint32_t*>(&t);
          }
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const uint32_t unit = static_cast<uint32_t>(half * 4 + c);
            *reinterpret_cast<uint4*>(box + lane * 128 + ((unit ^ swz) << 4)) =
                make_uint4(h[4 * c], h[4 * c + 1], h[4 * c + 2], h[4 * c + 3]);
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(tmY, box, n0 + panel * 64, row0);
          bulk_commit();
        }
        ++boxes;
      }
      tc_fence_before();
      mbar_arrive_cluster(leader_acc_empty + 8u * buf);
    } else if (!SK || (u.k0 == 0 && u.k1 == p.k_blocks)) {
      EpiState st;
      epilogue_begin<EMODE>(p, st, row, rows_valid);
#pragma unroll 1
      for (int c = 0; c < kTileN / 32; ++c) {
        uint32_t v[32];
        tmem_ld32(tacc + c * 32, v);
        tmem_ld_wait();
        epilogue_chunk<EMODE>(p, st, v, row, n0 + c * 32, rows_valid);
      }
      epilogue_end<EMODE>(p, st, row, nt, rows_valid);
      tc_fence_before();
      mbar_arrive_cluster(leader_acc_empty + 8u * buf);
    } else if constexpr (SK) {
      // Stream-K partial tile: park this CTA's 128 x 256 fp32 half in its slot;
      // the last contributing pair to arrive (per half, counter tile * 2 + rank)
      // sums the contributions in pair order -- its own from TMEM, the others'
      // from their slots -- and runs the epilogue.
      const int slot = uidx == 0 ? 0 : 1;
      const int cta = pair_id * 2 + static_cast<int>(rank);
      float4* mine = reinterpret_cast<float4*>(p.partials) + (static_cast<int64_t>(cta) * 2 + slot) * kSlotF4;
#pragma unroll 1
      for (int c = 0; c < kTileN / 32; ++c) {
        uint32_t v[32];
        tmem_ld32(tacc + c * 32, v);
        tmem_ld_wait();
        float4* dst = mine + (c * 8) * 128 + etid;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          __stcg(dst + j * 128, make_float4(__uint_as_float(v[4 * j]), __uint_as_float(v[4 * j + 1]),
                                            __uint_as_float(v[4 * j + 2]), __uint_as_float(v[4 * j + 3])));
        }
      }
      // The accumulator buffer stays allocated until this CTA knows whether it
      // is the last contributor: the last one reads its own part back from TMEM
      // instead of its slot.  Every exit releases it.
      auto release_acc = [&]() {
        tc_fence_before();
        mbar_arrive_cluster(leader_acc_empty + 8u * buf);
      };
      __threadfence();
      if (!epi_sync(epi_mb, epi_phase, abort_flag)) { release_acc(); break; }
      const int64_t it0 = static_cast<int64_t>(u.tile) * p.k_blocks;
      const int c_lo = sk_owner(it0, total, pairs);
      const int c_hi = sk_owner(it0 + p.k_blocks - 1, total, pairs);
      int* counter = p.counters + static_cast<int64_t>(u.tile) * 2 + rank;
      if (etid == 0) {
        const int prev = atomicAdd(counter, 1);
        *last_flag = (prev == c_hi - c_lo) ? 1 : 0;
      }
      if (!epi_sync(epi_mb, epi_phase, abort_flag)) { release_acc(); break; }
      const bool last = *last_flag != 0;
      if (!epi_sync(epi_mb, epi_phase, abort_flag)) { release_acc(); break; }
      if (!last) {
        release_acc();
      } else {
        __threadfence();
        EpiState st;
        epilogue_begin<EMODE>(p, st, row, rows_valid);
#pragma unroll 1
        for (int c = 0; c < kTileN / 32; ++c) {
          float sum[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) sum[j] = 0.0f;
          const int64_t off = static_cast<int64_t>(c * 8) * 128 + etid;
          // Contributors in pair order (the sum does not depend on who is last);
          // this pair's own part comes from TMEM, bit-identical to its slot.
          for (int ci = c_lo; ci <= c_hi; ++ci) {
            if (ci == pair_id) {
              uint32_t v[32];
              tmem_ld32(tacc + c * 32, v);
              tmem_ld_wait();
#pragma unroll
              for (int j = 0; j < 32; ++j) sum[j] += __uint_as_float(v[j]);
              continue;
            }
            const int64_t first_tile = (total * ci / pairs) / p.k_blocks;
            const int cslot = first_tile == u.tile ? 0 : 1;
            const float4* src = reinterpret_cast<const float4*>(p.partials) +
                                ((static_cast<int64_t>(ci) * 2 + rank) * 2 + cslot) * kSlotF4 + off;
            float4 x[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) x[j] = __ldcg(src + j * 128);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              sum[4 * j] += x[j].x; sum[4 * j + 1] += x[j].y;
              sum[4 * j + 2] += x[j].z; sum[4 * j + 3] += x[j].w;
            }
          }
          uint32_t v[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __float_as_uint(sum[j]);
          epilogue_chunk<EMODE>(p, st, v, row, n0 + c * 32, rows_valid);
        }
        release_acc();
        epilogue_end<EMODE>(p, st, row, nt, rows_valid);
        if (etid == 0) *counter = 0;  // ready for the next launch
      }
    }
    ++tl;
    ++uidx;
  }
  // Stores must finish reading the staging boxes before the CTA exits.
  if (STAGE && lane == 0) bulk_wait_all();
  __syncwarp();
}

// ------------------------------------------------------------ the kernel
// SK: stream-K schedule (partial tiles and their fix-up); the whole-tile
// instantiation carries no fix-up code, which keeps it free of register spills.
template <int BMODE, int EMODE, int STAGES, bool SK, int WSEL>
__global__ void __launch_bounds__(PairCfg<BMODE, STAGES, EMODE>::kThreads, 1)
    pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ CUtensorMap tmLA, const __grid_constant__ CUtensorMap tmLB,
                const __grid_constant__ CUtensorMap tmY, const __grid_constant__ CUtensorMap tmB2,
                const __grid_constant__ CUtensorMap tmY2, const Params p) {
  using C = PairCfg<BMODE, STAGES, EMODE>;
  static_assert(WSEL == 0 || (WSEL == 1 && BMODE == kNF4Fwd && !SK) || (WSEL == 2 && BMODE == kNF4Dx),
                "weight selection: 1 = gate/up forward (whole tiles), 2 = two-weight dX");
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* raw_ring = smem + STAGES * C::kStageBytes;  // forward: kRawStages x 4 KB of packed codes
  uint8_t* staging = raw_ring + C::kRawStages * C::kRawBytes;
  uint8_t* bar_area = staging + C::kStagingBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(bar_area);
  uint64_t* raw_full = full + STAGES;  // forward only: the code ring's slots
  uint64_t* raw_empty = raw_full + 8;
  uint64_t* empty = raw_empty + 8;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint64_t* epi_mb = drain + 1;
  uint64_t* gu_full = epi_mb + 1;  // kSwiGLUBwd: two box-set barriers per epilogue warp
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(gu_full + 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  volatile int* last_flag = abort_flag + 1;
  float* code2_s = reinterpret_cast<float*>(bar_area + 1024);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int pair_id = blockIdx.x >> 1;
  const int pairs = gridDim.x >> 1;
  const int num_tiles = p.m_tiles * p.n_tiles;
  const bool has_lora = p.lora_r > 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1 + 2 * 128);  // rank 0's producer + both CTAs' decoder threads
      mbar_init(&empty[s], 1);
    }
    for (int r = 0; r < C::kRawStages; ++r) {
      mbar_init(&raw_full[r], 1);
      mbar_init(&raw_empty[r], 128);  // the decoder group of the slot's k-step, this CTA
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 2 * 128);
    }
    mbar_init(drain, 1);
    mbar_init(epi_mb, 128);
    for (int i = 0; i < 8; ++i) mbar_init(&gu_full[i], 1);
    *abort_flag = 0;
    *last_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc_pair(tmem_holder, C::kTmemCols);
  tc_fence_before();
  // Barrier initialisation and the TMEM address must be visible to both CTAs
  // before any thread signals the peer.
  cluster_sync_all();
  tc_fence_after();
  // Launched with programmatic stream serialisation: the set-up above overlaps
  // the previous kernel of the stream; no global memory is read or written
  // before that kernel has completed and its writes are visible.
  grid_dependency_wait();
  launch_dependents();
  {
    // The decoders' scale table: the second weight's for the rank-1 CTA of a gate/up pair.
    const float* table = (WSEL == 1 && rank == 1) ? p.code2_2 : p.code2;
    for (int i = threadIdx.x; i < 256; i += blockDim.x) code2_s[i] = __ldg(table + i);
  }
  __syncthreads();
  const uint32_t tmem_base = *tmem_holder;
  const int rows_valid = runtime_rows(p);
  // rank 0's barriers, as shared::cluster addresses (stride 8 bytes per barrier)
  const uint32_t leader_full = map_to_rank(smem_addr(full), 0);
  const uint32_t leader_acc_empty = map_to_rank(smem_addr(acc_empty), 0);

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      if (has_lora) {
        tma_prefetch_desc(&tmLA);
        tma_prefetch_desc(&tmLB);
      }
      uint32_t it = 0;
      bool ok = true;
      UnitIter iter(p, num_tiles, pair_id, pairs);
      Unit u;
      while (ok && iter.next(u)) {
        const int mt = tile_m(p, u.tile), nt = tile_n(p, u.tile);
        const int m0 = mt * kTileM;
        if (m0 >= rows_valid) continue;
        const int arow = m0 + static_cast<int>(rank) * kTileRows;
        // A gate/up tile covers output columns nt*128.. of both weights; its LoRA B
        // rows come from the [2N, r] stack of both weights' factors.
        const int lbrow = WSEL == 1 ? static_cast<int>(rank) * p.N + nt * kHalfN
                                    : nt * kTileN + static_cast<int>(rank) * kHalfN;
        const int nsteps = (u.k1 - u.k0) + ((has_lora && u.k1 == p.k_blocks) ? 1 : 0);
        for (int ls = 0; ls < nsteps; ++ls, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, kErrWaitEmpty, abort_flag)) { ok = false; break; }
          uint8_t* a_s = smem + s * C::kStageBytes;
          uint8_t* b_s = a_s + C::kABytes;
          const int step = u.k0 + ls;
          if (step < u.k1) {
            if (leader) mbar_arrive_expect_tx(&full[s], 2 * C::kABytes);
            tma_load_2d_pair(a_s, &tmA, leader_full + 8u * s, step * kBK, arow);
          } else {
            if (leader) mbar_arrive_expect_tx(&full[s], 2 * (kTileRows + kHalfN) * p.lora_r * 2);
            tma_load_2d_pair(a_s, &tmLA, leader_full + 8u * s, 0, arow);
            tma_load_2d_pair(b_s, &tmLB, leader_full + 8u * s, 0, lbrow);
          }
        }
      }
      // Tail: every stage filled above must be released by the UMMA (which also
      // shows its bytes landed and the peer's commits arrived) before exit.  After
      // an abort rank 0 waits (bounded once in total) for the loads on its barriers.
      volatile int drain_abort = 0;
      bool clean = ok && !*abort_flag;
      for (uint32_t j = it; clean && j < it + STAGES; ++j) {
        clean = mbar_wait(&empty[j % STAGES], ((j / STAGES) & 1) ^ 1, kErrWaitDrain, abort_flag);
      }
      if (!clean) {
        const uint32_t first = it > static_cast<uint32_t>(STAGES) ? it - STAGES : 0;
        for (uint32_t j = first; j < it; ++j) {
          if (leader) mbar_wait(&full[j % STAGES], (j / STAGES) & 1, kErrWaitDrain, &drain_abort);
        }
      }
    }
  } else if (warp == 2) {
    // ------------------------------------------------------------ packed-code producer (forward, both CTAs)
    // Fills the code ring kRawStages k-steps ahead of the decoders; a slot is
    // refilled once its decoder group has read it (raw_empty).  Gate/up pairing:
    // the rank-1 CTA loads the second weight's codes.
    if constexpr (C::kRawTma) {
     if (lane == 0) {
      const CUtensorMap* bmap = (WSEL == 1 && rank == 1) ? &tmB2 : &tmB;
      tma_prefetch_desc(bmap);
      uint32_t it = 0;
      bool ok = true;
      UnitIter iter(p, num_tiles, pair_id, pairs);
      Unit u;
      while (ok && iter.next(u)) {
        const int mt = tile_m(p, u.tile), nt = tile_n(p, u.tile);
        if (mt * kTileM >= rows_valid) continue;
        const int brow = WSEL == 1 ? nt * kHalfN : nt * kTileN + static_cast<int>(rank) * kHalfN;
        const int nsteps = (u.k1 - u.k0) + ((has_lora && u.k1 == p.k_blocks) ? 1 : 0);
        for (int ls = 0; ls < nsteps; ++ls, ++it) {
          const int r = static_cast<int>(it % C::kRawStages);
          const uint32_t rph = (it / C::kRawStages) & 1;
          if (!mbar_wait(&raw_empty[r], rph ^ 1, kErrWaitEmpty, abort_flag)) { ok = false; break; }
          const int step = u.k0 + ls;
          if (step < u.k1) {
            mbar_arrive_expect_tx(&raw_full[r], C::kRawBytes);
            tma_load_2d(raw_ring + r * C::kRawBytes, bmap, &raw_full[r], step * (kBK / 2), brow);
          } else {
            mbar_arrive(&raw_full[r]);  // the LoRA step: nothing to decode
          }
        }
      }
      // Tail: every slot filled above read by its decoders before exit; after an
      // abort, wait (bounded once in total) for the loads still in flight.
      volatile int drain_abort = 0;
      bool clean = ok && !*abort_flag;
      for (uint32_t j = it; clean && j < it + C::kRawStages; ++j) {
        clean = mbar_wait(&raw_empty[j % C::kRawStages], ((j / C::kRawStages) & 1) ^ 1, kErrWaitDrain, abort_flag);
      }
      if (!clean) {
        const uint32_t first = it > static_cast<uint32_t>(C::kRawStages) ? it - C::kRawStages : 0;
        for (uint32_t j = first; j < it; ++j) {
          mbar_wait(&raw_full[j % C::kRawStages], (j / C::kRawStages) & 1, kErrWaitDrain, &drain_abort);
        }
      }
     }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ UMMA issuer (rank 0)
    // The whole warp runs the loop so the descriptors stay warp-uniform; lane 0
    // waits, one elected lane issues.
    if (leader) {
      constexpr uint32_t kIdesc = idesc_f16_f32(kTileM, kTileN, 0, C::kBMN ? 1 : 0);
      constexpr uint32_t kIdescLora = idesc_f16_f32(kTileM, kTileN, 0, 0);
      const uint32_t lora_layout = p.lora_r == 16 ? kSwizzle32B : (p.lora_r == 32 ? kSwizzle64B : kSwizzle128B);
      const uint32_t lora_pitch = static_cast<uint32_t>(p.lora_r) * 2;
      // Stage and phase of the next k-step (the step count modulo STAGES and the
      // parity of its quotient), advanced per step; stage s's descriptors are the
      // stage-0 ones plus s stages in the address field.
      uint32_t st = 0, ph = 0, tl = 0;
      static_assert(kBK == 64, "four K=16 UMMAs per k-step");
      const uint64_t ad0 = smem_desc(smem_addr(smem), 16, 1024, kSwizzle128B);
      const uint64_t bd0 = C::kBMN ? smem_desc(smem_addr(smem) + C::kABytes, 64 * 128, 1024, kSwizzle128B)
                                   : smem_desc(smem_addr(smem) + C::kABytes, 16, 1024, kSwizzle128B);
      const uint32_t a_lo0 = static_cast<uint32_t>(ad0), a_hi = static_cast<uint32_t>(ad0 >> 32);
      const uint32_t b_lo0 = static_cast<uint32_t>(bd0), b_hi = static_cast<uint32_t>(bd0 >> 32);
      const uint32_t empty_addr = smem_addr(empty);
      bool ok = true;
      UnitIter iter(p, num_tiles, pair_id, pairs);
      Unit u;
      while (ok && iter.next(u)) {
        if (tile_m(p, u.tile) * kTileM >= rows_valid) continue;
        const int buf = tl & 1;
        const uint32_t aph = (tl >> 1) & 1;
        if (!warp_wait(&acc_empty[buf], aph ^ 1, kErrWaitAccEmpty, abort_flag, lane)) { ok = false; break; }
        tc_fence_after();
        const uint32_t acc = tmem_base + buf * kTileN;
        const int nmain = u.k1 - u.k0;
        const bool lora_step = has_lora && u.k1 == p.k_blocks;
        for (int ls = 0; ls < nmain; ++ls) {
          // Both CTAs' A halves landed and both CTAs' decoders arrived.
          if (!warp_wait(full + st, ph, kErrWaitFull, abort_flag, lane)) { ok = false; break; }
          tc_fence_after();
          const uint32_t off = st * (C::kStageBytes >> 4);
          // Address-field steps (16-byte units): 32 bytes of K for a K-major operand,
          // a 16-row x 128-byte block for the MN-major dX operand.
          umma_kstep_pair_warp(acc, a_lo0 + off, a_hi, b_lo0 + off, b_hi, 32 >> 4,
                               C::kBMN ? (16 * 128) >> 4 : 32 >> 4, kIdesc, ls > 0 ? 1u : 0u, empty_addr + 8u * st);
          if (++st == static_cast<uint32_t>(STAGES)) { st = 0; ph ^= 1u; }
        }
        if (ok && lora_step) {
          if (!warp_wait(full + st, ph, kErrWaitFull, abort_flag, lane)) {
            ok = false;
          } else {
            tc_fence_after();
            const uint32_t a_addr = smem_addr(smem + st * C::kStageBytes);
            const uint32_t b_addr = a_addr + C::kABytes;
            for (int k16 = 0; k16 < p.lora_r / 16; ++k16) {
              const uint64_t bdesc = smem_desc(b_addr + k16 * 32, 16, 8 * lora_pitch, lora_layout);
              const uint64_t adesc = smem_desc(a_addr + k16 * 32, 16, 8 * lora_pitch, lora_layout);
              umma_f16_pair_warp(acc, adesc, bdesc, kIdescLora, 1u);
            }
            umma_commit_both_warp(&empty[st]);
            if (++st == static_cast<uint32_t>(STAGES)) { st = 0; ph ^= 1u; }
          }
        }
        if (ok) umma_commit_both_warp(&acc_full[buf]);
        ++tl;
      }
      // Tail: both accumulators released by both CTAs' epilogues (so their last
      // arrivals on this CTA's acc_empty have landed), then every UMMA complete.
      if (ok && !*abort_flag) {
        if (warp_wait(&acc_empty[tl & 1], ((tl >> 1) & 1) ^ 1, kErrWaitDrain, abort_flag, lane)) {
          warp_wait(&acc_empty[(tl + 1) & 1], (((tl + 1) >> 1) & 1) ^ 1, kErrWaitDrain, abort_flag, lane);
        }
      }
      umma_commit_local_warp(drain);
      volatile int no_abort = 0;
      warp_wait(drain, 0, kErrWaitDrain, &no_abort, lane);
    }
  } else if (warp >= 4 && warp < 8) {
    if (lane == 0 && C::kStoreStage && p.store_tma) tma_prefetch_desc(&tmY);
    const CUtensorMap* aux = EMODE == kSwiGLUBwd ? &tmB2 : &tmY2;
    if (lane == 0 && (EMODE == kSwiGLUFwd || EMODE == kSwiGLUBwd)) tma_prefetch_desc(aux);
    pair_epilogue<EMODE, SK, C::kStoreStage>(p, &tmY, aux, staging, tmem_base, acc_full, leader_acc_empty, epi_mb,
                                             gu_full, abort_flag, last_flag, warp, lane,
                         num_tiles, rows_valid, pair_id, pairs, rank);
  } else if (warp >= 8) {
    // ------------------------------------------------------------ NF4 decoders (both CTAs)
    // Group g decodes the k-steps whose running index has parity g; thread gtid
    // decodes one (row, 64-block) of this CTA's 128-row half per step and
    // arrives on rank 0's full barrier.  The block's 32 packed bytes, its
    // qabs byte and absmax2 value are loaded for the group's next step while the
    // current one decodes; the B slot is reused once empty[s] shows the UMMA
    // that read it has completed.
    const int group = (warp - 8) >> 2;
    const int gtid = ((warp - 8) & 3) * 32 + lane;
    // The weight a reduction step decodes: the only one (WSEL 0), this CTA's half
    // of a gate/up pair (WSEL 1), or the first / second of a concatenated
    // reduction (WSEL 2, steps >= k_split belong to the second, counted from 0).
    struct WView {
      const uint8_t* packed;
      const uint8_t* qabs;
      const float* absmax2;
      float off;
    };
    const WView first_w{p.packed, p.qabs, p.absmax2, __ldg(p.offset)};
    WView second_w = first_w;
    if constexpr (WSEL != 0) second_w = WView{p.packed2, p.qabs2, p.absmax2_2, __ldg(p.offset2)};
    const WView own_w = (WSEL == 1 && rank == 1) ? second_w : first_w;
    // A second weight's scale table is the shared-memory one when both weights
    // name the same table (bitsandbytes' dynamic map), else read through L1.
    const bool own_table = WSEL != 2 || p.code2_2 == p.code2;
    auto in_second = [&](int step) -> bool { return WSEL == 2 && step >= p.k_split; };
    auto local_step = [&](int step) -> int { return in_second(step) ? step - p.k_split : step; };
    auto view_of = [&](int step) -> const WView& { return in_second(step) ? second_w : own_w; };
    const int64_t bpr = p.w_cols / 64;
    const int64_t pitch = p.w_cols / 2;  // packed bytes per weight row
    uint32_t it = 0;
    bool ok = true;
    // Block index of this thread's (row, 64-block) at k-step `step` (within the
    // weight that step reads), or -1 outside the weight.
    auto block_of = [&](int n0, int step) -> int64_t {
      const int ls = local_step(step);
      if constexpr (BMODE == kNF4Fwd) {
        const int64_t wrow = n0 + gtid;
        return wrow < p.w_rows ? wrow * bpr + ls : -1;
      } else {
        const int64_t wrow = static_cast<int64_t>(ls) * kBK + (gtid >> 1);
        const int64_t wcol = n0 + 64 * (gtid & 1);
        return (wrow < p.w_rows && wcol < p.w_cols) ? wrow * bpr + wcol / 64 : -1;
      }
    };
    // Byte offset of that block's packed codes (row-major packing, 32 bytes per block).
    auto bytes_of = [&](int n0, int step) -> int64_t {
      const int ls = local_step(step);
      if constexpr (BMODE == kNF4Fwd) {
        return static_cast<int64_t>(n0 + gtid) * pitch + ls * (kBK / 2);
      } else {
        return (static_cast<int64_t>(ls) * kBK + (gtid >> 1)) * pitch + (n0 + 64 * (gtid & 1)) / 2;
      }
    };
    UnitIter iter(p, num_tiles, pair_id, pairs);
    Unit u;
    while (ok && iter.next(u)) {
      if (tile_m(p, u.tile) * kTileM >= rows_valid) continue;
      const int nt = tile_n(p, u.tile);
      const int n0 = WSEL == 1 ? nt * kHalfN : nt * kTileN + static_cast<int>(rank) * kHalfN;
      const int nsteps = (u.k1 - u.k0) + ((has_lora && u.k1 == p.k_blocks) ? 1 : 0);
      const int first = u.k0 + (group - static_cast<int>(it % C::kDecGroups) + C::kDecGroups) % C::kDecGroups;
      int64_t nb = first < u.k1 ? block_of(n0, first) : -1;
      uint4 w0_next = make_uint4(0, 0, 0, 0), w1_next = make_uint4(0, 0, 0, 0);
      uint32_t q_next = 0u;
      float a2_next = 0.0f;
      bool second_next = false;
      if (nb >= 0) {
        const WView& wv = view_of(first);
        if constexpr (!C::kRawTma) {
          const uint4* src = reinterpret_cast<const uint4*>(wv.packed + bytes_of(n0, first));
          w0_next = ld_stream16(src);
          w1_next = ld_stream16(src + 1);
        }
        q_next = __ldg(wv.qabs + nb);
        a2_next = __ldg(wv.absmax2 + (nb >> 8));
        second_next = in_second(first);
      }
      for (int ls = 0; ls < nsteps; ++ls, ++it) {
        if (static_cast<int>(it % C::kDecGroups) != group) continue;
        const int s = it % STAGES;
        const uint32_t ph = (it / STAGES) & 1;
        const int step = u.k0 + ls;
        const bool main_step = step < u.k1;
        const uint4 w0 = w0_next, w1 = w1_next;
        const uint32_t q_cur = q_next;
        const float a2_cur = a2_next;
        const bool second_cur = second_next;
        const bool valid = main_step && block_of(n0, step) >= 0;
        nb = step + C::kDecGroups < u.k1 ? block_of(n0, step + C::kDecGroups) : -1;
        if (nb >= 0) {
          const WView& wv = view_of(step + C::kDecGroups);
          if constexpr (!C::kRawTma) {
            const uint4* src = reinterpret_cast<const uint4*>(wv.packed + bytes_of(n0, step + C::kDecGroups));
            w0_next = ld_stream16(src);
            w1_next = ld_stream16(src + 1);
          }
          q_next = __ldg(wv.qabs + nb);
          a2_next = __ldg(wv.absmax2 + (nb >> 8));
          second_next = in_second(step + C::kDecGroups);
        }
        // Forward: the step's packed codes (raw_full), read into registers; the slot
        // is released after the decode has used them.  Every step: the B slot free
        // again (empty[s]: the UMMA that read it has completed), which also orders
        // this arrival on full[s] after the slot's previous phase.
        uint4 rp0 = make_uint4(0, 0, 0, 0), rp1 = make_uint4(0, 0, 0, 0);
        const int r = C::kRawTma ? static_cast<int>(it % (C::kRawTma ? C::kRawStages : 1)) : 0;
        if constexpr (C::kRawTma) {
          if (!mbar_wait(&raw_full[r], (it / C::kRawStages) & 1, kErrWaitFull, abort_flag)) {
            ok = false;
            break;
          }
          if (valid) {
            // Packed rows are 32 B, TMA-swizzled in 32 B spans: chunk ^= (row >> 2) & 1.
            const uint8_t* raw_s = raw_ring + r * C::kRawBytes + gtid * 32;
            const uint32_t x = static_cast<uint32_t>((gtid >> 2) & 1);
            rp0 = *reinterpret_cast<const uint4*>(raw_s + (x << 4));
            rp1 = *reinterpret_cast<const uint4*>(raw_s + ((x ^ 1u) << 4));
          }
        }
        if (!mbar_wait(&empty[s], ph ^ 1, kErrWaitEmpty, abort_flag)) {
          ok = false;
          break;
        }
        if (main_step) {
          uint8_t* b_s = smem + s * C::kStageBytes + C::kABytes;
          float scale = 0.0f;
          if (valid) {
            const float code = (!second_cur || own_table) ? code2_s[q_cur] : __ldg(p.code2_2 + q_cur);
            scale = __fadd_rn(__fmul_rn(code, a2_cur), second_cur ? second_w.off : own_w.off);
          }
          if constexpr (C::kRawTma) {
            nf4_decode_words(rp0, rp1, b_s + gtid * 128, gtid, scale, valid);
          } else if constexpr (BMODE == kNF4Fwd) {
            nf4_decode_words(w0, w1, b_s + gtid * 128, gtid, scale, valid);
          } else {
            const int r = gtid >> 1, j = gtid & 1;
            // Lanes 2r and 2r + 1 write row r of the two panels (8 KB apart, the same
            // banks): the odd lane writes its chunks in flipped order.
            nf4_decode_words_flip(w0, w1, b_s + j * (kBK * 128) + r * 128, r, scale, valid, 4u * j);
          }
        }
        // The decoded B (generic writes) before the UMMA reads it, and the code slot's
        // generic reads before the next TMA write into it (both async proxy).
        fence_proxy_async_smem();
        if constexpr (C::kRawTma) mbar_arrive(&raw_empty[r]);
        mbar_arrive_cluster(leader_full + 8u * s);
      }
    }
  }

  tc_fence_before();
  cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, C::kTmemCols);
  }
}

}  // namespace pair
}  // namespace gemm
}  // namespace sb
