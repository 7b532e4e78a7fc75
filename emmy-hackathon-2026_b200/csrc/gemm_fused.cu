// 3xTF32 GEMM kernel that splits one operand's tiles inside the tensor-core
// kernel, into tensor memory.
//
// The arithmetic is the one of gemm.cu and of the reference's tensor-core
// emitter (tf32_emitter.py:22-96 model; :647-668 split, :675-684 hh+hl+lh):
// every product is hi*hi + hi*lo + lo*hi with hi = rna_tf32(x) and
// lo = rna_tf32(x - hi), accumulated in FP32 with the chunked TMEM
// accumulation of gemm.cu.  What changes is where the split happens.  The
// reference splits every element again at every K step; the pre-pass path
// (gemm.cu) splits whole operands into a scratch copy first.  Here TMA brings
// raw FP32 tiles of the kernel's A operand into shared memory and the CTA
// splits each staged tile once.
//
// Shared-memory bandwidth decides the design.  On B200 the tensor core's
// operand reads, TMA writes and thread loads/stores of one SM share about
// 128 bytes per clock (measured: the pre-pass kernel at 128 x 256 tiles moves
// 960 128-byte wavefronts per 768 MMA cycles and runs at the predicted 80 %).
// gemm_tmem_a_kernel splits its A operand into TENSOR memory: each split
// thread owns one A row (one TMEM lane), reads the 16 raw K values of its
// staged row, splits them and writes hi and lo with tcgen05.st; the MMAs take
// A from TMEM (tcgen05.mma ... [a_tmem]), so A costs one shared-memory write
// (TMA) and one read per stage instead of a hi/lo write plus three
// tensor-core reads.  The kernel's B operand is split once per GEMM by the
// pre-pass (K-major hi/lo) because the tensor core reads B from shared
// memory; per 128 x 192 stage this is ~610 wavefronts for 576 MMA cycles.
// (Splitting both operands in shared memory instead doubles the shared-memory
// traffic the tensor core competes for and measured 1.4-2x slower.)
//
// Two orientations of C = A B (template flags A_MN, C_T):
//   direct      the kernel's A is the caller's A (rows of C, K-major), its B
//               the caller's B pre-split; C tiles are stored as computed.
//   transposed  the kernel computes C^T = B^T A^T: its A operand is the
//               caller's B (split in the kernel; a row-major [K, N] B is read
//               MN-major -- TMA boxes of 128 N x 16 K, a thread reading its
//               column of the box -- and a [N, K] B K-major), its B operand is
//               the caller's A pre-split, and the epilogue writes each
//               accumulator row as a column of C.  For a short, wide C (a
//               row shard of a multi-GPU GEMM: 512 x 4096 x 4096) this splits
//               only A in the pre-pass (8 MB instead of B's 64 MB) and tiles
//               the output 128 N-rows at a time, so 4096 / 128 x 512 / 128 =
//               128 tiles fill one wave of 148 SMs.
//
// Roles (576 threads): warp 0 TMA producer, warp 1 TMEM allocator + MMA
// issuer (the whole warp runs the loop, one elected lane issues), warps
// 2..17 split + epilogue: all sixteen fold each finished 256-wide K chunk of
// the TMEM accumulator into FP32 registers with round-to-nearest adds, then
// bias -> ReLU -> C staged in shared memory and written by TMA stores; the
// split is shared out by stage in four groups of four warps.  The kernel is
// launched with programmatic dependent launch (its set-up overlaps the B
// split's tail).  All waits are bounded.
#include <algorithm>

#include "common.cuh"
#include "sm100.cuh"
#include "tmap.cuh"

namespace {

constexpr int BM = 128;
constexpr int kChunkK = 256;            // K per accumulation chunk
constexpr int kMinK = 32;               // K of the widest stage: the kernel needs K >= this
constexpr int kWorkWarps = 16;          // split + epilogue warps
constexpr int kWorkThreads = 32 * kWorkWarps;
constexpr int kThreads = 64 + kWorkThreads;
// The split runs in stage groups: work warp w belongs to group (w - 2) / 4,
// one warp per TMEM lane quarter, and group g splits the stages kb with
// kb % kGroups == g.  Each warp then has kGroups stage times to finish one
// stage and waits on a quarter of the stage barriers.
constexpr int kGroups = 4;

// m, n are the KERNEL's extents (rows of its A operand, rows of its B
// operand).  In the transposed orientation C is the caller's [n][m] matrix
// (row stride ldc) and the bias runs over the kernel's rows.
struct FusedArgs {
  float *c;
  const float *bias;
  int64_t m, n, ldc;
  int num_kb;
  int relu;
  int tma_c;  // C is written by TMA stores (16-byte aligned, ldc % 4 == 0)
  unsigned *err;
};

// C staging for the TMA store, 16 KB boxes.  Direct orientation: [BN / 32]
// boxes of 128 rows x 32 FP32 with the 128-byte swizzle, so the
// row-per-thread 16-byte writes of a warp hit eight distinct 16-byte chunks
// per 128 bytes.  Transposed orientation: [BN / 32] boxes of 32 C rows x 128
// C columns, unswizzled; a warp's 32 threads (32 consecutive C columns)
// write one 128-byte row segment per store (no conflicts).
constexpr int kCBox = BM * 32 * 4;

// Epilogue of the kernel's work warps.  Work warp w holds the
// accumulator of TMEM lane quarter w % 4 (rows) and column slice (w - 2) / 4
// (BN / 4 columns).  BN = 128 or 192: with 576 threads a thread may hold 96
// registers, which fits 48 accumulator columns but not 64.
template <int BN>
struct Slice {
  static constexpr int CPT = BN / 4;
  static_assert(CPT % 8 == 0, "slice width");
  float acc[CPT];
  int quarter, slice, lane;

  __device__ __forceinline__ explicit Slice(int warp)
      : quarter(warp & 3), slice((warp - 2) >> 2), lane(threadIdx.x & 31) {
#pragma unroll
    for (int j = 0; j < CPT; ++j) acc[j] = 0.0f;
  }

  // Fold chunk `chunk` (TMEM accumulator buffer chunk & 1) into registers and
  // hand the buffer back to the MMA issuer.
  __device__ __forceinline__ bool fold(int chunk, uint32_t tmem_base, uint64_t *tmem_full, uint64_t *tmem_empty,
                                       unsigned *err, volatile int *abort) {
    const int buf = chunk & 1;
    if (!sm100::mbar_wait(&tmem_full[buf], (chunk >> 1) & 1, err, sm100::kSiteEpilogueAccum, abort,
                          3 * sm100::kWaitCycles))
      return false;
    sm100::tc_fence_after();
    const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(buf * BN + slice * CPT);
#pragma unroll
    for (int j = 0; j + 16 <= CPT; j += 16) {
      uint32_t r[16];
      sm100::tmem_ld_32x32b_x16(taddr + j, r);
      sm100::tmem_ld_wait();
#pragma unroll
      for (int i = 0; i < 16; ++i) acc[j + i] = __fadd_rn(acc[j + i], __uint_as_float(r[i]));
    }
    if constexpr (CPT % 16 != 0) {
      constexpr int j = CPT - 8;
      uint32_t r[8];
      sm100::tmem_ld_32x32b_x8(taddr + j, r);
      sm100::tmem_ld_wait();
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[j + i] = __fadd_rn(acc[j + i], __uint_as_float(r[i]));
    }
    sm100::tc_fence_before();
    __syncwarp();
    if (lane == 0) sm100::mbar_arrive(&tmem_empty[buf]);
    return true;
  }

  // Bias -> ReLU -> the staging boxes in shared memory (see kCBox).
  __device__ __forceinline__ void stage(uint8_t *staging, const FusedArgs &args, int64_t n0) {
    const int row = quarter * 32 + lane;
    const int c0 = slice * CPT;
#pragma unroll
    for (int j = 0; j < CPT; j += 4) {
      float v[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float x = acc[j + q];
        if (args.bias) x = __fadd_rn(x, (n0 + c0 + j + q < args.n) ? __ldg(args.bias + n0 + c0 + j + q) : 0.0f);
        if (args.relu) x = x > 0.0f ? x : 0.0f;
        v[q] = x;
      }
      const int col = c0 + j;
      const uint32_t chunk = (uint32_t)((col & 31) >> 2) ^ (uint32_t)(row & 7);
      // no compiler memory barrier: the bias loads of later groups may be
      // issued ahead of this store
      sm100::sts128_relaxed(sm100::smem_addr(staging + (col >> 5) * kCBox + row * 128 + chunk * 16),
                            make_float4(v[0], v[1], v[2], v[3]));
    }
  }

  __device__ __forceinline__ void store(const FusedArgs &args, int64_t m0, int64_t n0) {
    const int64_t row = m0 + quarter * 32 + lane;
    const int64_t col0 = n0 + slice * CPT;
    if (row >= args.m || col0 >= args.n) return;
    float *crow = args.c + row * args.ldc + col0;
    const bool vec =
        ((args.ldc & 3) == 0) && ((reinterpret_cast<uintptr_t>(args.c) & 15) == 0) && col0 + CPT <= args.n;
#pragma unroll
    for (int j = 0; j < CPT; ++j) {
      float x = acc[j];
      if (args.bias) x = __fadd_rn(x, (col0 + j < args.n) ? __ldg(args.bias + col0 + j) : 0.0f);
      if (args.relu) x = x > 0.0f ? x : 0.0f;
      acc[j] = x;
    }
    if (vec) {
#pragma unroll
      for (int j = 0; j < CPT; j += 4)
        *reinterpret_cast<float4 *>(crow + j) = make_float4(acc[j], acc[j + 1], acc[j + 2], acc[j + 3]);
    } else {
#pragma unroll
      for (int j = 0; j < CPT; ++j)
        if (col0 + j < args.n) crow[j] = acc[j];
    }
  }

  // Transposed orientation: this thread's accumulator row is C column
  // m0 + row, its columns are C rows n0 + c0 + j.  Bias (one value: the
  // column's) -> ReLU -> the unswizzled [32 C rows][128 C columns] boxes.
  __device__ __forceinline__ void stage_t(uint8_t *staging, const FusedArgs &args, int64_t m0) {
    const int row = quarter * 32 + lane;
    const int c0 = slice * CPT;
    const float b = (args.bias && m0 + row < args.m) ? __ldg(args.bias + m0 + row) : 0.0f;
    const uint32_t base = sm100::smem_addr(staging) + (uint32_t)row * 4u;
#pragma unroll
    for (int j = 0; j < CPT; ++j) {
      float x = acc[j];
      if (args.bias) x = __fadd_rn(x, b);
      if (args.relu) x = x > 0.0f ? x : 0.0f;
      const int col = c0 + j;
      asm volatile("st.shared.f32 [%0], %1;" ::"r"(base + (uint32_t)((col >> 5) * kCBox + (col & 31) * 512)), "f"(x));
    }
  }

  // Transposed orientation without TMA stores: column m0 + row of C rows
  // n0 + c0 + j; a warp stores 32 consecutive columns of one row per step.
  __device__ __forceinline__ void store_t(const FusedArgs &args, int64_t m0, int64_t n0) {
    const int64_t col = m0 + quarter * 32 + lane;
    if (col >= args.m) return;
    const float b = args.bias ? __ldg(args.bias + col) : 0.0f;
#pragma unroll
    for (int j = 0; j < CPT; ++j) {
      const int64_t crow = n0 + slice * CPT + j;
      float x = acc[j];
      if (args.bias) x = __fadd_rn(x, b);
      if (args.relu) x = x > 0.0f ? x : 0.0f;
      if (crow < args.n) args.c[crow * args.ldc + col] = x;
    }
  }
};

// ============================================================================
// A split into tensor memory, B pre-split.
// ============================================================================
// Stage K: 16 (64-byte rows, 64-byte swizzle) for 192-wide tiles, 32
// (128-byte rows, 128-byte swizzle) for 128-wide tiles.  A stage carries one
// wait, six (BK 16) or twelve (BK 32) MMAs and one commit for the MMA issuer;
// at N = 128 a 16-wide stage is only 565 tensor cycles and the issuer's
// per-stage cost showed (25 % below the 192-wide tiles' rate per flop,
// measured on B200), so the narrow tile takes twice the K per stage.
template <int BN>
struct TmemAShape {
  static constexpr int BK = BN == 128 ? 32 : 16;
  static constexpr int SW = BK * 4;           // bytes per K-major row = swizzle span
  static constexpr int kChunkBlocks = kChunkK / BK;
  static constexpr int kTileA = BM * BK * 4;  // raw A: 128 rows x BK
  static constexpr int kTileB = BN * BK * 4;  // each of B_hi, B_lo
  static constexpr int kStage = kTileA + 2 * kTileB;
  static constexpr int kStages = (200 * 1024) / kStage < 8 ? (200 * 1024) / kStage : 8;
  static constexpr int kSmem = kStages * kStage + 1024;
  // TMEM columns: two accumulator buffers of BN, then the A ring: per stage
  // BK hi columns + BK lo columns (one column per K element, one lane per row).
  // The A ring is shorter than the shared-memory ring (TMEM is the scarcer of
  // the two; TMA latency wants the longer ring).  TMEM A stage kb % kAStages
  // is free once the MMAs of block kb - kAStages are done, which is the
  // completion of empty_bar for that block: one commit per stage serves both.
  static constexpr int kAccCols = 2 * BN;
  static constexpr int kAStages = (512 - kAccCols) / (2 * BK) < kStages ? (512 - kAccCols) / (2 * BK) : kStages;
  // A split warp at block kb has seen the MMA finish block kb - kAStages, so
  // chunk c is complete once kb >= (c + 1) * kChunkBlocks + kAStages - 1.
  static constexpr int kFoldLag = kAStages;
  static_assert(BN == 128 || BN == 192, "BN");
  static_assert(kAStages >= 2 && kChunkBlocks > kFoldLag, "TMEM ring");
  static_assert(kSmem <= 227 * 1024, "stage ring exceeds shared memory");
};

// A_MN: the raw A operand is MN-major in global memory ([K][M], the caller's
// row-major B of the transposed orientation); its TMA box is 128 M x 16 K
// (unswizzled, 512-byte rows) instead of 128 rows x 16 K (64-byte swizzle).
// C_T: the epilogue writes the accumulator transposed (stage_t / store_t).
template <int BN, bool A_MN, bool C_T>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tmem_a_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_bhi,
                       const __grid_constant__ CUtensorMap map_blo, const __grid_constant__ CUtensorMap map_c,
                       const FusedArgs args) {
  constexpr int G = kGroups;
  using Shape = TmemAShape<BN>;
  constexpr int BK = Shape::BK, kChunkBlocks = Shape::kChunkBlocks;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[Shape::kStages];   // raw A + B hi/lo landed
  __shared__ __align__(8) uint64_t empty_bar[Shape::kStages];  // MMAs done with the block in the stage
  __shared__ __align__(8) uint64_t a_full[Shape::kAStages];    // A hi/lo stored in TMEM
  __shared__ __align__(8) uint64_t tmem_full[2];
  __shared__ __align__(8) uint64_t tmem_empty[2];
  __shared__ __align__(8) uint64_t drain_bar;
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_word;

  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5;
  // M-fastest raster: the CTAs resident at one time share a few B column
  // tiles (B_hi/B_lo are twice A's size) and sweep A, so both stay in L2.
  const int64_t m0 = (int64_t)blockIdx.x * BM;
  const int64_t n0 = (int64_t)blockIdx.y * BN;
  const int num_kb = args.num_kb;
  const int num_chunks = (num_kb + kChunkBlocks - 1) / kChunkBlocks;
  volatile int *abort = &abort_word;

  auto a_raw = [&](int s) { return smem + s * Shape::kStage; };
  auto b_hi = [&](int s) { return smem + s * Shape::kStage + Shape::kTileA; };
  auto b_lo = [&](int s) { return smem + s * Shape::kStage + Shape::kTileA + Shape::kTileB; };

  if (threadIdx.x == 0) {
    abort_word = 0;
    for (int s = 0; s < Shape::kStages; ++s) {
      sm100::mbar_init(&full_bar[s], 1);
      sm100::mbar_init(&empty_bar[s], 1);
    }
    for (int t = 0; t < Shape::kAStages; ++t) sm100::mbar_init(&a_full[t], kWorkWarps / G);
    for (int b = 0; b < 2; ++b) {
      sm100::mbar_init(&tmem_full[b], 1);
      sm100::mbar_init(&tmem_empty[b], kWorkWarps);
    }
    sm100::mbar_init(&drain_bar, 1);
    sm100::fence_barrier_init();
    sm100::prefetch_tensormap(&map_a);
    sm100::prefetch_tensormap(&map_bhi);
    sm100::prefetch_tensormap(&map_blo);
  }
  if (warp == 1) sm100::tmem_alloc(&tmem_slot, 512);
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem_base = tmem_slot;
  const uint32_t tmem_a = tmem_base + Shape::kAccCols;  // A ring, lane 0
  // Nothing above touched global memory: under programmatic dependent
  // launch the set-up overlaps the B split kernel's tail.
  grid_dependency_wait();
  grid_dependents_launch();

  if (warp == 0) {
    if (sm100::elect_lane0()) {
      int issued = 0;
      for (int kb = 0; kb < num_kb; ++kb) {
        const int s = kb % Shape::kStages;
        if (kb >= Shape::kStages && !sm100::mbar_wait(&empty_bar[s], ((kb / Shape::kStages) & 1) ^ 1, args.err,
                                                      sm100::kSiteProducerEmpty, abort))
          break;
        sm100::mbar_arrive_expect_tx(&full_bar[s], Shape::kTileA + 2 * Shape::kTileB);
        const int kx = kb * BK;
        if constexpr (A_MN)
          sm100::tma_load_2d(a_raw(s), &map_a, &full_bar[s], (int)m0, kx);
        else
          sm100::tma_load_2d(a_raw(s), &map_a, &full_bar[s], kx, (int)m0);
        sm100::tma_load_2d(b_hi(s), &map_bhi, &full_bar[s], kx, (int)n0);
        sm100::tma_load_2d(b_lo(s), &map_blo, &full_bar[s], kx, (int)n0);
        issued = kb + 1;
      }
      int never = 0;
      for (int kb = issued > Shape::kStages ? issued - Shape::kStages : 0; kb < issued; ++kb)
        sm100::mbar_wait(&full_bar[kb % Shape::kStages], (kb / Shape::kStages) & 1, args.err, sm100::kSiteDrain,
                         &never);
    }
  } else if (warp == 1) {
    {
      constexpr uint32_t idesc = sm100::idesc_tf32(BM, BN);
      for (int kb = 0; kb < num_kb; ++kb) {
        const int chunk = kb / kChunkBlocks;
        const int buf = chunk & 1;
        const bool first = (kb % kChunkBlocks) == 0;
        const bool last = ((kb + 1) % kChunkBlocks) == 0 || kb + 1 == num_kb;
        if (first && chunk >= 2 &&
            !sm100::mbar_wait_warp(&tmem_empty[buf], ((chunk >> 1) & 1) ^ 1, args.err, sm100::kSiteMmaFull, abort))
          break;
        // a_full[s] is raised by split warps that saw full_bar[s] complete,
        // so it also orders the stage's TMA writes (B) before these MMAs.
        const int s = kb % Shape::kStages;
        const int t = kb % Shape::kAStages;
        if (!sm100::mbar_wait_warp(&a_full[t], (kb / Shape::kAStages) & 1, args.err, sm100::kSiteMmaFull, abort))
          break;
        sm100::tc_fence_after();
        const uint32_t d = tmem_base + (uint32_t)(buf * BN);
        const uint32_t ahi = tmem_a + (uint32_t)(t * 2 * BK), alo = ahi + BK;
        const uint32_t bhi = sm100::smem_addr(b_hi(s)), blo = sm100::smem_addr(b_lo(s));
#pragma unroll
        for (int k = 0; k < BK / 8; ++k) {
          const uint64_t dbh = sm100::desc_kmajor<Shape::SW>(bhi + k * 32);
          const uint64_t dbl = sm100::desc_kmajor<Shape::SW>(blo + k * 32);
          sm100::mma_tf32_ts(d, alo + 8 * k, dbh, idesc, (first && k == 0) ? 0u : 1u);
          sm100::mma_tf32_ts(d, ahi + 8 * k, dbl, idesc, 1u);
          sm100::mma_tf32_ts(d, ahi + 8 * k, dbh, idesc, 1u);
        }
        sm100::mma_commit(&empty_bar[s]);
        if (last) sm100::mma_commit(&tmem_full[buf]);
      }
      sm100::mma_commit(&drain_bar);
      int never = 0;
      sm100::mbar_wait(&drain_bar, 0, args.err, sm100::kSiteDrain, &never);
    }
  } else {
    // Split: thread (quarter q, lane l) owns A row 32q + l = TMEM lane 32q + l
    // and splits all 16 K values of its row in the stages of its group (one
    // warp per TMEM lane quarter in each of the four groups).
    Slice<BN> out(warp);
    const int group = out.slice;
    const int row = out.quarter * 32 + out.lane;
    // K-major raw A rows are SW bytes with the SW-byte TMA swizzle: 16-byte
    // chunk c of row r sits at chunk c ^ ((r >> 1) & 3) for 64-byte rows and
    // c ^ (r & 7) for 128-byte rows (conflict-free across 8 rows either way).
    // MN-major: element (k, r) at k * 512 + 4 r, so a warp's loads of one k
    // are 128 consecutive bytes.
    const uint32_t swz = Shape::SW == 64 ? (uint32_t)((row >> 1) & 3) : (uint32_t)(row & 7);
    const uint32_t row_off = A_MN ? (uint32_t)(row * 4) : (uint32_t)(row * Shape::SW);
    const uint32_t lane_base = (uint32_t)(out.quarter * 32) << 16;
    bool ok = true;
    int folded = 0;
    for (int kb = group; kb < num_kb && ok; kb += G) {
      // TMEM A stage t is free once the MMAs of block kb - kAStages are done.
      // That block's empty_bar phase cannot complete again before this
      // group's block kb has been consumed, so the parity is unambiguous.
      // It is waited first: with those MMAs done, the load of block
      // kb - kStages into stage s (kStages >= kAStages) has landed and been
      // consumed, so the full_bar wait below cannot meet the stage a phase
      // behind.  (Stage s alternates between groups when kStages is not a
      // multiple of the group count; waited the other way round, a group
      // could see another group's load still in flight as its own.)
      const int s = kb % Shape::kStages;
      const int t = kb % Shape::kAStages;
      if (kb >= Shape::kAStages) {
        const int prev = kb - Shape::kAStages;
        if (!sm100::mbar_wait(&empty_bar[prev % Shape::kStages], (prev / Shape::kStages) & 1, args.err,
                              sm100::kSiteConvert, abort)) {
          ok = false;
          break;
        }
      }
      if (!sm100::mbar_wait(&full_bar[s], (kb / Shape::kStages) & 1, args.err, sm100::kSiteConvert, abort)) {
        ok = false;
        break;
      }
      sm100::tc_fence_after();
      const uint32_t src = sm100::smem_addr(a_raw(s)) + row_off;
      const uint32_t dst = tmem_a + lane_base + (uint32_t)(t * 2 * BK);
#pragma unroll
      for (int p = 0; p < BK / 16; ++p) {
        // 16 elements of the row at a time, loaded at once, split and stored
        // in two halves of 8 columns each for hi and lo: with the 48
        // accumulators this stays inside the 96 registers a 576-thread CTA
        // may use (16-column halves spilled).
        float4 v[4];
        if constexpr (A_MN) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            float e[4];
#pragma unroll
            for (int u = 0; u < 4; ++u)
              asm volatile("ld.shared.f32 %0, [%1];"
                           : "=f"(e[u])
                           : "r"(src + (uint32_t)(16 * p + 4 * q + u) * 512u)
                           : "memory");
            v[q] = make_float4(e[0], e[1], e[2], e[3]);
          }
        } else {
#pragma unroll
          for (int q = 0; q < 4; ++q) v[q] = sm100::lds128(src + 16u * ((uint32_t)(4 * p + q) ^ swz));
        }
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          uint32_t h[8], l[8];
#pragma unroll
          for (int q = 0; q < 2; ++q) {
            float4 hv, lv;
            split_tf32x4(v[2 * half + q], hv, lv);
            h[4 * q + 0] = __float_as_uint(hv.x), h[4 * q + 1] = __float_as_uint(hv.y);
            h[4 * q + 2] = __float_as_uint(hv.z), h[4 * q + 3] = __float_as_uint(hv.w);
            l[4 * q + 0] = __float_as_uint(lv.x), l[4 * q + 1] = __float_as_uint(lv.y);
            l[4 * q + 2] = __float_as_uint(lv.z), l[4 * q + 3] = __float_as_uint(lv.w);
          }
          sm100::tmem_st_32x32b_x8(dst + 16 * p + 8 * half, h);
          sm100::tmem_st_32x32b_x8(dst + BK + 16 * p + 8 * half, l);
        }
      }
      sm100::tmem_st_wait();
      sm100::tc_fence_before();
      __syncwarp();
      if (out.lane == 0) sm100::mbar_arrive(&a_full[t]);
      while (folded < num_chunks && kb >= (folded + 1) * kChunkBlocks + Shape::kFoldLag) {
        if (!out.fold(folded, tmem_base, tmem_full, tmem_empty, args.err, abort)) {
          ok = false;
          break;
        }
        ++folded;
      }
    }
    while (ok && folded < num_chunks) {
      ok = out.fold(folded, tmem_base, tmem_full, tmem_empty, args.err, abort);
      ++folded;
    }
    if (args.tma_c) {
      // The ring is idle once the last chunk is folded (every MMA, hence
      // every load it consumed, is done): stage C there, one TMA store per box.
      if (ok) {
        if constexpr (C_T)
          out.stage_t(smem, args, m0);
        else
          out.stage(smem, args, n0);
      }
      sm100::fence_proxy_async_smem();
      sm100::named_barrier(1, kWorkThreads);
      if (threadIdx.x == 64 && ok) {
#pragma unroll 1
        for (int b = 0; b < BN / 32; ++b) {
          // transposed: box b holds C rows n0 + 32 b .. +31, columns m0 .. +127
          if constexpr (C_T)
            sm100::tma_store_2d(&map_c, smem + b * kCBox, (int)m0, (int)n0 + 32 * b);
          else
            sm100::tma_store_2d(&map_c, smem + b * kCBox, (int)n0 + 32 * b, (int)m0);
        }
        sm100::tma_store_flush();
      }
    } else if (ok) {
      if constexpr (C_T)
        out.store_t(args, m0, n0);
      else
        out.store(args, m0, n0);
    }
  }
  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem_base, 512);
  }
}

// --- host side -------------------------------------------------------------
// `a` is the kernel's raw A operand: [m][k] with row stride lda (K-major) or,
// with A_MN, [k][m] with row stride lda.  ops.b_hi / b_lo hold the kernel's B
// operand split K-major ([n][kp]).  C is [m][n] (row stride ldc), or [n][m]
// with C_T.
template <int BN, bool A_MN, bool C_T>
int launch_tmem_a(b2k_ctx *ctx, const float *a, int64_t k, int64_t lda, const b2k::SplitOperands &ops, float *c,
                  int64_t m, int64_t n, int64_t ldc, const float *bias, int relu, cudaStream_t s) {
  using Shape = TmemAShape<BN>;
  constexpr int BK = Shape::BK;
  constexpr CUtensorMapSwizzle kSwizzle = Shape::SW == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B;
  CUtensorMap map_a, map_bhi, map_blo;
  // A's map keeps the true K: the K blocks past it (up to B's zero-padded
  // kp) read as zero through TMA's out-of-range fill, never beyond the row.
  int status = A_MN ? b2k::make_map_2d(ctx, &map_a, a, m, k, lda, BM, BK, CU_TENSOR_MAP_SWIZZLE_NONE)
                    : b2k::make_map_2d(ctx, &map_a, a, k, m, lda, BK, BM, kSwizzle);
  if (status == B2K_OK) status = b2k::make_map_2d(ctx, &map_bhi, ops.b_hi, ops.kp, n, ops.kp, BK, BN, kSwizzle);
  if (status == B2K_OK) status = b2k::make_map_2d(ctx, &map_blo, ops.b_lo, ops.kp, n, ops.kp, BK, BN, kSwizzle);
  if (status != B2K_OK) return status;
  // C through TMA stores when it is TMA-writable, else row stores by the threads.
  CUtensorMap map_c{};
  const int tma_c = b2k::aligned16(c) && ldc % 4 == 0;
  if (tma_c) {
    status = C_T ? b2k::make_map_2d(ctx, &map_c, c, m, n, ldc, BM, 32, CU_TENSOR_MAP_SWIZZLE_NONE)
                 : b2k::make_map_2d(ctx, &map_c, c, n, m, ldc, 32, BM, CU_TENSOR_MAP_SWIZZLE_128B);
    if (status != B2K_OK) return status;
  }
  static_assert((BN / 32) * kCBox <= Shape::kStages * Shape::kStage, "C staging exceeds the ring");
  FusedArgs args{c, bias, m, n, ldc, (int)(ops.kp / BK), relu, tma_c, ctx->error_flag};
  auto kernel = gemm_tmem_a_kernel<BN, A_MN, C_T>;
  cudaError_t err = b2k::set_max_smem(ctx, (const void *)kernel, Shape::kSmem);
  if (err != cudaSuccess) return b2k::cuda_fail(ctx, err, "gemm (TMEM A): set smem");
  if ((n + BN - 1) / BN > 65535) return b2k::fail(ctx, B2K_EINVAL, "gemm: N exceeds %d", 65535 * BN);
  dim3 grid((unsigned)((m + BM - 1) / BM), (unsigned)((n + BN - 1) / BN), 1);
  err = b2k::launch_kernel(b2k::pdl_enabled(), kernel, grid, dim3(kThreads), Shape::kSmem, s, map_a, map_bhi, map_blo,
                           map_c, args);
  if (err != cudaSuccess) return b2k::cuda_fail(ctx, err, "gemm (TMEM A) launch");
  return b2k::check_launch(ctx, "gemm (TMEM A) launch");
}

}  // namespace

// b2k_gemm_set_fused_split: 0 = pre-pass split of both operands, 1 = choose
// by the cost estimate below (default), 2 = the transposed orientation
// wherever TMA can read B, 3 = the direct orientation wherever TMA can read A.
static int g_split_mode = 1;

extern "C" int b2k_gemm_set_fused_split(int mode) {
  if (mode < 0 || mode > 3) return B2K_EINVAL;
  g_split_mode = mode;
  return B2K_OK;
}

namespace b2k {

// TMA reads a caller's operand directly when its base is 16-byte aligned and
// its row stride is a multiple of 4 elements.
static bool tma_readable(const float *p, int64_t ld) { return aligned16(p) && (ld % 4 == 0); }

// Estimated microseconds of one call on each path, to choose between them.
// Every kernel computes one 128-row tile per CTA, so its time is (waves of
// tiles over the SMs) x (tile width x K x the kernel's time per column and K
// element), plus the pre-pass split of the operands it does not split itself
// (12 bytes moved per element at ~5 TB/s).  Calibrated on B200 at K = 4096
// (one wave at full clock): the pre-pass kernel's 128 x 256 tiles take
// 131 us, the in-kernel split's 128 x 192 tiles 108 us and its 128 x 128
// tiles 84 us; the calibration reproduces the measured 4096^3 (direct, 578 us)
// and the row shards M = 2048 (pre-pass, 323 us), 1024 (transposed, 193 us)
// and 512 (transposed, 87-98 us) within a few per cent.
constexpr double kColUsPrepass = 1.25e-4, kColUs192 = 1.37e-4, kColUs128 = 1.60e-4;

static double col_us(int bn) { return bn == 128 ? kColUs128 : kColUs192; }

static double path_cost_us(int64_t tiles, int bn, int64_t kp, double per_col_k, int64_t split_rows, int sms) {
  const int64_t waves = (tiles + sms - 1) / sms;
  return (double)waves * (double)bn * (double)kp * per_col_k + (double)split_rows * (double)kp * 2.4e-6;
}

static int tmem_tile_width(int64_t n) { return (n <= 128 || gemm_variant() == 2) ? 128 : 192; }

int gemm_direct_tile_width(int64_t n) { return tmem_tile_width(n); }

// Tile width of the transposed orientation's kernel B operand (the caller's
// M): 128 or 192, whichever covers the output in less estimated time.
int gemm_transposed_tile_width(int64_t m, int64_t n, int sms) {
  if (m <= 128 || gemm_variant() == 2 || sms <= 0) return 128;
  const int64_t rows = (n + BM - 1) / BM;
  const double c128 = (double)((rows * ((m + 127) / 128) + sms - 1) / sms) * 128 * kColUs128;
  const double c192 = (double)((rows * ((m + 191) / 192) + sms - 1) / sms) * 192 * kColUs192;
  return c192 < c128 ? 192 : 128;
}

int gemm_split_mode(const float *a, const float *b, int64_t m, int64_t n, int64_t k, int64_t lda, int64_t ldb,
                    int layout, int sms, bool chunks_ok) {
  if (g_split_mode == 0 || k < kMinK || m > INT32_MAX - 256 || n > INT32_MAX - 256 || k > INT32_MAX - 64) return 0;
  const bool a_t = (layout & B2K_A_KM) != 0, b_nk = (layout & B2K_B_NK) != 0;
  // direct: A [m][k] read by TMA; transposed: B read by TMA, [n][k] K-major
  // or [k][n] MN-major (whole 128-column boxes: n >= 128)
  const bool direct_ok = !a_t && tma_readable(a, lda);
  const bool transposed_ok = tma_readable(b, ldb) && (b_nk || n >= BM);
  if (g_split_mode == 3) return direct_ok ? kSplitDirect : 0;
  if (g_split_mode == 2) return transposed_ok ? kSplitTransposed : 0;
  if (sms <= 0) return direct_ok ? kSplitDirect : 0;
  const int64_t kp = gemm_kpad(k);
  const int bn0 = main_tile_width(m, n, 1, kp, sms), bn1 = tmem_tile_width(n);
  const int bn2 = gemm_transposed_tile_width(m, n, sms);
  const int64_t mt = (m + BM - 1) / BM, nt = (n + BM - 1) / BM;
  // the pre-pass kernel's cost per column grows as its tile narrows (A's
  // operand reads are shared by fewer columns): (128 + bn) / bn, relative to
  // the 256-wide tile the constant is calibrated on
  double c0 = path_cost_us(mt * ((n + bn0 - 1) / bn0), bn0, kp, kColUsPrepass * ((128.0 + bn0) / bn0) / 1.5, m + n,
                           sms);
  // the pre-pass kernel split over K chunks (gemm_main takes it when faster)
  if (chunks_ok) c0 = std::min(c0, chunked_cost_us(m, n, kp, sms) + (double)(m + n) * (double)kp * 2.4e-6);
  const double c1 = direct_ok ? path_cost_us(mt * ((n + bn1 - 1) / bn1), bn1, kp, col_us(bn1), n, sms) : 1e300;
  const double c2 = transposed_ok ? path_cost_us(nt * ((m + bn2 - 1) / bn2), bn2, kp, col_us(bn2), m, sms) : 1e300;
  if (c1 <= c0 && c1 <= c2) return kSplitDirect;
  if (c2 < c0) return kSplitTransposed;
  return 0;
}

int gemm_tmem_a(b2k_ctx *ctx, const float *a, int64_t k, int64_t lda, const SplitOperands &ops, float *c, int64_t m,
                int64_t n, int64_t ldc, const float *bias, int relu, cudaStream_t s) {
  PhaseTimer timer(ctx, B2K_PHASE_MMA, s);
  if (tmem_tile_width(n) == 128)
    return launch_tmem_a<128, false, false>(ctx, a, k, lda, ops, c, m, n, ldc, bias, relu, s);
  return launch_tmem_a<192, false, false>(ctx, a, k, lda, ops, c, m, n, ldc, bias, relu, s);
}

int gemm_tmem_b(b2k_ctx *ctx, const float *b, int64_t k, int64_t ldb, bool b_nk, const SplitOperands &ops, float *c,
                int64_t m, int64_t n, int64_t ldc, const float *bias, int relu, cudaStream_t s, int bn) {
  PhaseTimer timer(ctx, B2K_PHASE_MMA, s);
  // The kernel computes C^T [n][m] = B^T A^T: its rows are the caller's n.
  const bool wide = (bn ? bn : gemm_transposed_tile_width(m, n, ctx->sm_count)) == 192;
  if (b_nk)
    return wide ? launch_tmem_a<192, false, true>(ctx, b, k, ldb, ops, c, n, m, ldc, bias, relu, s)
                : launch_tmem_a<128, false, true>(ctx, b, k, ldb, ops, c, n, m, ldc, bias, relu, s);
  return wide ? launch_tmem_a<192, true, true>(ctx, b, k, ldb, ops, c, n, m, ldc, bias, relu, s)
              : launch_tmem_a<128, true, true>(ctx, b, k, ldb, ops, c, n, m, ldc, bias, relu, s);
}

}  // namespace b2k
