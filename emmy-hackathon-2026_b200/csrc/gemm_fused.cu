// 3xTF32 GEMM kernels that split operand tiles inside the tensor-core kernel.
//
// The arithmetic is the one of gemm.cu and of the reference's tensor-core
// emitter (tf32_emitter.py:22-96 model; :647-668 split, :675-684 hh+hl+lh):
// every product is hi*hi + hi*lo + lo*hi with hi = rna_tf32(x) and
// lo = rna_tf32(x - hi), accumulated in FP32 with the chunked TMEM
// accumulation of gemm.cu.  What changes is where the split happens.  The
// reference splits every element again at every K step; the pre-pass path
// (gemm.cu) splits whole operands into a scratch copy first.  Here TMA brings
// raw FP32 tiles into shared memory and the CTA splits each staged tile once.
//
// Shared-memory bandwidth decides the design.  On B200 the tensor core's
// operand reads, TMA writes and thread loads/stores of one SM share about
// 128 bytes per clock (measured: the pre-pass kernel at 128 x 256 tiles moves
// 960 128-byte wavefronts per 768 MMA cycles and runs at the predicted 80 %).
// Two kernels:
//
//   gemm_tmem_a_kernel (default unless the pre-pass kernel's wider tiles
//       cover the output in enough fewer waves)  A is split into TENSOR memory: each split
//       thread owns one A row (one TMEM lane), reads one raw 16-byte chunk of
//       the staged row, splits it and writes hi and lo with tcgen05.st; the
//       MMAs take A from TMEM (tcgen05.mma ... [a_tmem]), so A costs one
//       shared-memory write (TMA) and one read per stage instead of a hi/lo
//       write plus three tensor-core reads.  B is split once per GEMM by the
//       pre-pass (K-major hi/lo) because B must be read from shared memory by
//       the tensor core; per 128 x 192 stage this is ~610 wavefronts for 576
//       MMA cycles.
//   gemm_smem_split_kernel         both operands staged raw and split in
//       shared memory (hi in place, lo beside it; B either K-major or
//       MN-major with the 128-byte/32-byte-atom swizzle so a row-major B needs
//       no transpose).  No pre-pass and no scratch, but the split's thread
//       traffic doubles the shared-memory load (~1120 wavefronts per 576 MMA
//       cycles): measured about 2x slower than the pre-pass kernel, so it is
//       kept for comparison only (b2k_gemm_set_fused_split(2)).
//
// Roles (576 threads): warp 0 TMA producer, warp 1 TMEM allocator + MMA
// issuer (the whole warp runs the loop, one elected lane issues), warps
// 2..17 split + epilogue: all sixteen fold each finished 256-wide K chunk of
// the TMEM accumulator into FP32 registers with round-to-nearest adds, then
// bias -> ReLU -> C staged in shared memory and written by TMA stores; the
// split is shared out by stage in four groups of four warps.  The kernel is
// launched with programmatic dependent launch (its set-up overlaps the B
// split's tail).  All waits are bounded.
#include "common.cuh"
#include "sm100.cuh"
#include "tmap.cuh"

namespace {

constexpr int BM = 128;
constexpr int BK = 16;                  // FP32 elements of K per stage (64-byte K-major rows)
constexpr int kChunkBlocks = 256 / BK;  // K blocks per accumulation chunk
constexpr int kWorkWarps = 16;          // split + epilogue warps
constexpr int kWorkThreads = 32 * kWorkWarps;
constexpr int kThreads = 64 + kWorkThreads;
// The split runs in stage groups: work warp w belongs to group (w - 2) / 4,
// one warp per TMEM lane quarter, and group g splits the stages kb with
// kb % kGroups == g.  Each warp then has kGroups stage times to finish one
// stage and waits on a quarter of the stage barriers.
constexpr int kGroups = 4;
constexpr int kGroupWarps = kWorkWarps / kGroups;
constexpr int kGroupThreads = 32 * kGroupWarps;

struct FusedArgs {
  float *c;
  const float *bias;
  int64_t m, n, ldc;
  int num_kb;
  int relu;
  int tma_c;  // C is written by TMA stores (16-byte aligned, ldc % 4 == 0)
  unsigned *err;
};

// C staging for the TMA store: the tile as [BN / 32] boxes of 128 rows x 32
// FP32 (16 KB each) with the 128-byte swizzle, so the row-per-thread writes
// of a warp hit eight distinct 16-byte chunks per 128 bytes (no conflicts).
constexpr int kCBox = BM * 32 * 4;

// Epilogue helpers shared by both kernels.  Work warp w holds the
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
};

// ============================================================================
// A split into tensor memory, B pre-split.
// ============================================================================
template <int BN>
struct TmemAShape {
  static constexpr int kTileA = BM * BK * 4;  // raw A: 128 rows x 64 bytes
  static constexpr int kTileB = BN * BK * 4;  // each of B_hi, B_lo
  static constexpr int kStage = kTileA + 2 * kTileB;
  static constexpr int kStages = (200 * 1024) / kStage < 8 ? (200 * 1024) / kStage : 8;
  static constexpr int kSmem = kStages * kStage + 1024;
  // TMEM columns: two accumulator buffers of BN, then the A ring: per stage
  // 16 hi columns + 16 lo columns (one column per K element, one lane per row).
  // The A ring is shorter than the shared-memory ring (TMEM is the scarcer of
  // the two; TMA latency wants the longer ring).  TMEM A stage kb % kAStages
  // is free once the MMAs of block kb - kAStages are done, which is the
  // completion of empty_bar for that block: one commit per stage serves both.
  static constexpr int kAccCols = 2 * BN;
  static constexpr int kAStages = (512 - kAccCols) / 32 < kStages ? (512 - kAccCols) / 32 : kStages;
  // A split warp at block kb has seen the MMA finish block kb - kAStages, so
  // chunk c is complete once kb >= (c + 1) * kChunkBlocks + kAStages - 1.
  static constexpr int kFoldLag = kAStages;
  static_assert(BN == 128 || BN == 192, "BN");
  static_assert(kAStages >= 2 && kChunkBlocks > kFoldLag, "TMEM ring");
  static_assert(kSmem <= 227 * 1024, "stage ring exceeds shared memory");
};

template <int BN, int G>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tmem_a_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_bhi,
                       const __grid_constant__ CUtensorMap map_blo, const __grid_constant__ CUtensorMap map_c,
                       const FusedArgs args) {
  using Shape = TmemAShape<BN>;
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
        const uint32_t ahi = tmem_a + (uint32_t)(t * 32), alo = ahi + 16;
        const uint32_t bhi = sm100::smem_addr(b_hi(s)), blo = sm100::smem_addr(b_lo(s));
#pragma unroll
        for (int k = 0; k < BK / 8; ++k) {
          const uint64_t dbh = sm100::desc_kmajor<64>(bhi + k * 32), dbl = sm100::desc_kmajor<64>(blo + k * 32);
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
    // Split: thread (quarter q, lane l) owns A row 32q + l = TMEM lane 32q + l.
    // The 16 K values of a staged row are four 16-byte chunks; with G stage
    // groups each of the 4 / G warps of a quarter in a group splits G chunks.
    Slice<BN> out(warp);
    constexpr int kPerQuarter = 4 / G;  // warps of one quarter in one group
    const int group = out.slice / kPerQuarter;
    const int chunk0 = (out.slice % kPerQuarter) * G;
    const int row = out.quarter * 32 + out.lane;
    // Raw A rows are 64 bytes with the 64-byte TMA swizzle: 16-byte chunk c of
    // row r sits at chunk c ^ ((r >> 1) & 3) (conflict-free across 8 rows).
    const uint32_t swz = (uint32_t)((row >> 1) & 3);
    const uint32_t row_off = (uint32_t)(row * 64);
    const uint32_t lane_base = (uint32_t)(out.quarter * 32) << 16;
    bool ok = true;
    int folded = 0;
    for (int kb = group; kb < num_kb && ok; kb += G) {
      const int s = kb % Shape::kStages;
      if (!sm100::mbar_wait(&full_bar[s], (kb / Shape::kStages) & 1, args.err, sm100::kSiteConvert, abort)) {
        ok = false;
        break;
      }
      // TMEM A stage t is free once the MMAs of block kb - kAStages are done.
      // That block's empty_bar phase cannot complete again before this
      // group's block kb has been consumed, so the parity is unambiguous.
      const int t = kb % Shape::kAStages;
      if (kb >= Shape::kAStages) {
        const int prev = kb - Shape::kAStages;
        if (!sm100::mbar_wait(&empty_bar[prev % Shape::kStages], (prev / Shape::kStages) & 1, args.err,
                              sm100::kSiteConvert, abort)) {
          ok = false;
          break;
        }
      }
      sm100::tc_fence_after();
      const uint32_t src = sm100::smem_addr(a_raw(s)) + row_off;
      const uint32_t dst = tmem_a + lane_base + (uint32_t)(t * 32);
      if constexpr (G == 4) {
        // The whole 16-element row chunk, loaded at once, split and stored
        // in two halves of 8 columns each for hi and lo: with the 48
        // accumulators this stays inside the 96 registers a 576-thread CTA
        // may use (16-column halves spilled).
        float4 v[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) v[q] = sm100::lds128(src + 16u * ((uint32_t)q ^ swz));
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
          sm100::tmem_st_32x32b_x8(dst + 8 * half, h);
          sm100::tmem_st_32x32b_x8(dst + 16 + 8 * half, l);
        }
      } else {
#pragma unroll
        for (int q = 0; q < G; ++q) {
          const uint32_t c = (uint32_t)(chunk0 + q);
          float4 hv, lv;
          split_tf32x4(sm100::lds128(src + 16u * (c ^ swz)), hv, lv);
          sm100::tmem_st_32x32b_x4(dst + 4 * c, __float_as_uint(hv.x), __float_as_uint(hv.y), __float_as_uint(hv.z),
                                   __float_as_uint(hv.w));
          sm100::tmem_st_32x32b_x4(dst + 16 + 4 * c, __float_as_uint(lv.x), __float_as_uint(lv.y),
                                   __float_as_uint(lv.z), __float_as_uint(lv.w));
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
      if (ok) out.stage(smem, args, n0);
      sm100::fence_proxy_async_smem();
      sm100::named_barrier(1, kWorkThreads);
      if (threadIdx.x == 64 && ok) {
#pragma unroll 1
        for (int b = 0; b < BN / 32; ++b) sm100::tma_store_2d(&map_c, smem + b * kCBox, (int)n0 + 32 * b, (int)m0);
        sm100::tma_store_flush();
      }
    } else if (ok) {
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

// ============================================================================
// Both operands split in shared memory (comparison kernel).
// ============================================================================
template <int BN, bool B_MN>
struct SmemSplitShape {
  static constexpr int kTileA = BM * BK * 4;  // bytes of one A slot
  static constexpr int kTileB = BN * BK * 4;
  static constexpr int kStage = 2 * kTileA + 2 * kTileB;  // hi + lo of A and B
  static constexpr int kStages = (200 * 1024) / kStage < 6 ? (200 * 1024) / kStage : 6;
  // A split warp at block kb has seen TMA refill a stage the MMA released
  // kStages blocks earlier, so chunk c is complete once
  // kb >= (c + 1) * kChunkBlocks + kStages - 1.
  static constexpr int kFoldLag = kStages;
  static constexpr int kSmem = kStages * kStage + 1024;
  static constexpr uint32_t kTmemCols = 2 * BN <= 256 ? 256u : 512u;
  static constexpr int kVecA = kTileA / 16;  // float4 per slot
  static constexpr int kVecB = kTileB / 16;
  // MN-major B: boxes of 32 N x BK K (2 KB); each box is four 512-byte
  // swizzle atoms stacked along K.
  static constexpr int kBoxB = 32 * BK * 4;
  static_assert(kBoxB % 512 == 0, "MN-major B boxes hold whole swizzle atoms");
  static_assert(BN == 128 || BN == 192, "BN");
  static_assert(kVecA % kGroupThreads == 0 && kVecB % kGroupThreads == 0, "split work split");
  static_assert(kChunkBlocks > kFoldLag, "fold lag");
  static_assert(kSmem <= 227 * 1024, "stage ring exceeds shared memory");
};

template <int BN, bool B_MN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_smem_split_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                           const FusedArgs args) {
  using Shape = SmemSplitShape<BN, B_MN>;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[Shape::kStages];   // raw tiles landed
  __shared__ __align__(8) uint64_t split_bar[Shape::kStages];  // hi/lo written
  __shared__ __align__(8) uint64_t empty_bar[Shape::kStages];  // MMAs done with the stage
  __shared__ __align__(8) uint64_t tmem_full[2];
  __shared__ __align__(8) uint64_t tmem_empty[2];
  __shared__ __align__(8) uint64_t drain_bar;
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_word;

  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t n0 = (int64_t)blockIdx.x * BN;
  const int64_t m0 = (int64_t)blockIdx.y * BM;
  const int num_kb = args.num_kb;
  const int num_chunks = (num_kb + kChunkBlocks - 1) / kChunkBlocks;
  volatile int *abort = &abort_word;

  auto a_hi = [&](int s) { return smem + s * Shape::kStage; };
  auto a_lo = [&](int s) { return smem + s * Shape::kStage + Shape::kTileA; };
  auto b_hi = [&](int s) { return smem + s * Shape::kStage + 2 * Shape::kTileA; };
  auto b_lo = [&](int s) { return smem + s * Shape::kStage + 2 * Shape::kTileA + Shape::kTileB; };

  if (threadIdx.x == 0) {
    abort_word = 0;
    for (int s = 0; s < Shape::kStages; ++s) {
      sm100::mbar_init(&full_bar[s], 1);
      sm100::mbar_init(&split_bar[s], kGroupWarps);
      sm100::mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      sm100::mbar_init(&tmem_full[b], 1);
      sm100::mbar_init(&tmem_empty[b], kWorkWarps);
    }
    sm100::mbar_init(&drain_bar, 1);
    sm100::fence_barrier_init();
    sm100::prefetch_tensormap(&map_a);
    sm100::prefetch_tensormap(&map_b);
  }
  if (warp == 1) sm100::tmem_alloc(&tmem_slot, Shape::kTmemCols);
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem_base = tmem_slot;

  if (warp == 0) {
    if (sm100::elect_lane0()) {
      int issued = 0;
      for (int kb = 0; kb < num_kb; ++kb) {
        const int s = kb % Shape::kStages;
        if (kb >= Shape::kStages && !sm100::mbar_wait(&empty_bar[s], ((kb / Shape::kStages) & 1) ^ 1, args.err,
                                                      sm100::kSiteProducerEmpty, abort))
          break;
        sm100::mbar_arrive_expect_tx(&full_bar[s], Shape::kTileA + Shape::kTileB);
        const int kx = kb * BK;
        sm100::tma_load_2d(a_hi(s), &map_a, &full_bar[s], kx, (int)m0);
        if constexpr (B_MN) {
#pragma unroll
          for (int j = 0; j < BN / 32; ++j)
            sm100::tma_load_2d(b_hi(s) + j * Shape::kBoxB, &map_b, &full_bar[s], (int)n0 + 32 * j, kx);
        } else {
          sm100::tma_load_2d(b_hi(s), &map_b, &full_bar[s], kx, (int)n0);
        }
        issued = kb + 1;
      }
      // Every issued load must land before the CTA may exit (budget only).
      int never = 0;
      for (int kb = issued > Shape::kStages ? issued - Shape::kStages : 0; kb < issued; ++kb)
        sm100::mbar_wait(&full_bar[kb % Shape::kStages], (kb / Shape::kStages) & 1, args.err, sm100::kSiteDrain,
                         &never);
    }
  } else if (warp == 1) {
    {
      constexpr uint32_t idesc = sm100::idesc_tf32(BM, BN, B_MN);
      for (int kb = 0; kb < num_kb; ++kb) {
        const int chunk = kb / kChunkBlocks;
        const int buf = chunk & 1;
        const bool first = (kb % kChunkBlocks) == 0;
        const bool last = ((kb + 1) % kChunkBlocks) == 0 || kb + 1 == num_kb;
        if (first && chunk >= 2 &&
            !sm100::mbar_wait_warp(&tmem_empty[buf], ((chunk >> 1) & 1) ^ 1, args.err, sm100::kSiteMmaFull, abort))
          break;
        const int s = kb % Shape::kStages;
        if (!sm100::mbar_wait_warp(&split_bar[s], (kb / Shape::kStages) & 1, args.err, sm100::kSiteMmaFull, abort))
          break;
        sm100::tc_fence_after();
        const uint32_t d = tmem_base + (uint32_t)(buf * BN);
        const uint32_t ahi = sm100::smem_addr(a_hi(s)), alo = sm100::smem_addr(a_lo(s));
        const uint32_t bhi = sm100::smem_addr(b_hi(s)), blo = sm100::smem_addr(b_lo(s));
#pragma unroll
        for (int k = 0; k < BK / 8; ++k) {
          // A: 8 TF32 = 32 bytes along the swizzled K-major row.
          const uint64_t dah = sm100::desc_kmajor<64>(ahi + k * 32), dal = sm100::desc_kmajor<64>(alo + k * 32);
          uint64_t dbh, dbl;
          if constexpr (B_MN) {
            // 8 K rows = two 512-byte atoms; atoms of consecutive N are one box (2 KB) apart.
            dbh = sm100::desc_mn_sw128_32b(bhi + k * 1024, Shape::kBoxB, 512);
            dbl = sm100::desc_mn_sw128_32b(blo + k * 1024, Shape::kBoxB, 512);
          } else {
            dbh = sm100::desc_kmajor<64>(bhi + k * 32);
            dbl = sm100::desc_kmajor<64>(blo + k * 32);
          }
          sm100::mma_tf32(d, dal, dbh, idesc, (first && k == 0) ? 0u : 1u);
          sm100::mma_tf32(d, dah, dbl, idesc, 1u);
          sm100::mma_tf32(d, dah, dbh, idesc, 1u);
        }
        sm100::mma_commit(&empty_bar[s]);
        if (last) sm100::mma_commit(&tmem_full[buf]);
      }
      sm100::mma_commit(&drain_bar);
      int never = 0;
      sm100::mbar_wait(&drain_bar, 0, args.err, sm100::kSiteDrain, &never);
    }
  } else {
    Slice<BN> out(warp);
    const int group = out.slice;
    const int gt = out.quarter * 32 + lane;  // thread index within the group
    bool ok = true;
    int folded = 0;
    for (int kb = group; kb < num_kb && ok; kb += kGroups) {
      const int s = kb % Shape::kStages;
      if (!sm100::mbar_wait(&full_bar[s], (kb / Shape::kStages) & 1, args.err, sm100::kSiteConvert, abort)) {
        ok = false;
        break;
      }
      // Slot order within a stage is A_hi, A_lo, B_hi, B_lo; float4 index i
      // < kVecA lies in A (lo slot kTileA further), else in B (lo slot
      // kTileB further).  The split is elementwise, so the swizzle carries over.
      const uint32_t stage = sm100::smem_addr(a_hi(s));
#pragma unroll 2
      for (int i = gt; i < Shape::kVecA + Shape::kVecB; i += kGroupThreads) {
        const uint32_t hi = i < Shape::kVecA ? stage + 16u * i : stage + Shape::kTileA + 16u * i;
        const uint32_t lo = hi + (i < Shape::kVecA ? Shape::kTileA : Shape::kTileB);
        float4 h, l;
        split_tf32x4(sm100::lds128(hi), h, l);
        sm100::sts128(hi, h);
        sm100::sts128(lo, l);
      }
      sm100::fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(&split_bar[s]);
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
    if (ok) out.store(args, m0, n0);
  }
  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem_base, Shape::kTmemCols);
  }
}

// --- host side -------------------------------------------------------------
template <int BN, int G>
int launch_tmem_a(b2k_ctx *ctx, const float *a, int64_t k, int64_t lda, const b2k::SplitOperands &ops, float *c,
                  int64_t m, int64_t n, int64_t ldc, const float *bias, int relu, cudaStream_t s) {
  using Shape = TmemAShape<BN>;
  CUtensorMap map_a, map_bhi, map_blo;
  // A's map keeps the true K: the K blocks past it (up to B's zero-padded
  // kp) read as zero through TMA's out-of-range fill, never beyond the row.
  int status = b2k::make_map_2d(ctx, &map_a, a, k, m, lda, BK, BM, CU_TENSOR_MAP_SWIZZLE_64B);
  if (status == B2K_OK)
    status = b2k::make_map_2d(ctx, &map_bhi, ops.b_hi, ops.kp, n, ops.kp, BK, BN, CU_TENSOR_MAP_SWIZZLE_64B);
  if (status == B2K_OK)
    status = b2k::make_map_2d(ctx, &map_blo, ops.b_lo, ops.kp, n, ops.kp, BK, BN, CU_TENSOR_MAP_SWIZZLE_64B);
  if (status != B2K_OK) return status;
  // C through TMA stores when it is TMA-writable, else row stores by the threads.
  CUtensorMap map_c{};
  const int tma_c = b2k::aligned16(c) && ldc % 4 == 0;
  if (tma_c && (status = b2k::make_map_2d(ctx, &map_c, c, n, m, ldc, 32, BM, CU_TENSOR_MAP_SWIZZLE_128B)) != B2K_OK)
    return status;
  static_assert((BN / 32) * kCBox <= Shape::kStages * Shape::kStage, "C staging exceeds the ring");
  FusedArgs args{c, bias, m, n, ldc, (int)(ops.kp / BK), relu, tma_c, ctx->error_flag};
  auto kernel = gemm_tmem_a_kernel<BN, G>;
  cudaError_t err = b2k::set_max_smem(ctx, (const void *)kernel, Shape::kSmem);
  if (err != cudaSuccess) return b2k::cuda_fail(ctx, err, "gemm (TMEM A): set smem");
  if ((n + BN - 1) / BN > 65535) return b2k::fail(ctx, B2K_EINVAL, "gemm: N exceeds %d", 65535 * BN);
  dim3 grid((unsigned)((m + BM - 1) / BM), (unsigned)((n + BN - 1) / BN), 1);
  err = b2k::launch_kernel(b2k::pdl_enabled(), kernel, grid, dim3(kThreads), Shape::kSmem, s, map_a, map_bhi, map_blo,
                           map_c, args);
  if (err != cudaSuccess) return b2k::cuda_fail(ctx, err, "gemm (TMEM A) launch");
  return b2k::check_launch(ctx, "gemm (TMEM A) launch");
}

template <int BN, bool B_MN>
int launch_smem_split(b2k_ctx *ctx, const float *a, const float *b, float *c, int64_t m, int64_t n, int64_t k,
                      int64_t lda, int64_t ldb, int64_t ldc, const float *bias, int relu, cudaStream_t s) {
  using Shape = SmemSplitShape<BN, B_MN>;
  CUtensorMap map_a, map_b;
  int status = b2k::make_map_2d(ctx, &map_a, a, k, m, lda, BK, BM, CU_TENSOR_MAP_SWIZZLE_64B);
  if (status != B2K_OK) return status;
  status = B_MN ? b2k::make_map_2d(ctx, &map_b, b, n, k, ldb, 32, BK, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B)
                : b2k::make_map_2d(ctx, &map_b, b, k, n, ldb, BK, BN, CU_TENSOR_MAP_SWIZZLE_64B);
  if (status != B2K_OK) return status;
  FusedArgs args{c, bias, m, n, ldc, (int)((k + BK - 1) / BK), relu, 0, ctx->error_flag};
  auto kernel = gemm_smem_split_kernel<BN, B_MN>;
  cudaError_t err = b2k::set_max_smem(ctx, (const void *)kernel, Shape::kSmem);
  if (err != cudaSuccess) return b2k::cuda_fail(ctx, err, "gemm (shared-memory split): set smem");
  dim3 grid((unsigned)((n + BN - 1) / BN), (unsigned)((m + BM - 1) / BM), 1);
  kernel<<<grid, kThreads, Shape::kSmem, s>>>(map_a, map_b, args);
  return b2k::check_launch(ctx, "gemm (shared-memory split) launch");
}

}  // namespace

// 0 = pre-pass split of both operands, 1 = A split into TMEM inside the
// kernel + B pre-pass where that tiles no worse (default), 2 = both split in
// shared memory, 3 = A split into TMEM wherever TMA can read A.
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

// Each CTA of either kernel computes one 128-row tile, so a call takes about
// (waves of tiles over the SMs) x (tile width) x K.  The in-kernel split
// (tiles 192 wide) is kept unless the pre-pass kernel (256 wide) needs 10 %
// less by that estimate: it also saves the pre-pass over A.  Measured on
// B200: 4096^3 takes 5 waves x 192 against 4 x 256, and the in-kernel split
// is 7 % faster; 4097 x 1000 x 776 takes 2 waves x 192 (198 tiles on 148
// SMs) against 1 x 256, and the pre-pass kernel is 35 % faster.
static bool prepass_tiles_better(int64_t m, int64_t n, int sms) {
  if (sms <= 0) return false;
  const int64_t bn1 = (n <= 128 || gemm_variant() == 2) ? 128 : 192, bn0 = main_tile_width(n);
  const int64_t rows = (m + BM - 1) / BM;
  const int64_t cost1 = (rows * ((n + bn1 - 1) / bn1) + sms - 1) / sms * bn1;
  const int64_t cost0 = (rows * ((n + bn0 - 1) / bn0) + sms - 1) / sms * bn0;
  return 10 * cost1 > 11 * cost0;
}

int gemm_split_mode(const float *a, const float *b, int64_t m, int64_t n, int64_t k, int64_t lda, int64_t ldb,
                    int sms) {
  if (g_split_mode == 0 || k < BK || m > INT32_MAX - BM || n > INT32_MAX - 256 || k > INT32_MAX - 64) return 0;
  if (!tma_readable(a, lda)) return 0;
  if (g_split_mode == 2) return tma_readable(b, ldb) ? 2 : 1;
  if (g_split_mode == 1 && prepass_tiles_better(m, n, sms)) return 0;
  return 1;
}

int gemm_tmem_a(b2k_ctx *ctx, const float *a, int64_t k, int64_t lda, const SplitOperands &ops, float *c, int64_t m,
                int64_t n, int64_t ldc, const float *bias, int relu, cudaStream_t s) {
  PhaseTimer timer(ctx, B2K_PHASE_MMA, s);
  // Four stage groups measured fastest (vs. 2 and 1) on B200.
  if (n <= 128 || gemm_variant() == 2) return launch_tmem_a<128, 4>(ctx, a, k, lda, ops, c, m, n, ldc, bias, relu, s);
  return launch_tmem_a<192, 4>(ctx, a, k, lda, ops, c, m, n, ldc, bias, relu, s);
}

int gemm_smem_split(b2k_ctx *ctx, const float *a, const float *b, float *c, int64_t m, int64_t n, int64_t k,
                    int64_t lda, int64_t ldb, int64_t ldc, int b_kmajor, const float *bias, int relu,
                    cudaStream_t s) {
  PhaseTimer timer(ctx, B2K_PHASE_MMA, s);
  if (n <= 128 || gemm_variant() == 2)
    return b_kmajor ? launch_smem_split<128, false>(ctx, a, b, c, m, n, k, lda, ldb, ldc, bias, relu, s)
                    : launch_smem_split<128, true>(ctx, a, b, c, m, n, k, lda, ldb, ldc, bias, relu, s);
  return b_kmajor ? launch_smem_split<192, false>(ctx, a, b, c, m, n, k, lda, ldb, ldc, bias, relu, s)
                  : launch_smem_split<192, true>(ctx, a, b, c, m, n, k, lda, ldb, ldc, bias, relu, s);
}

}  // namespace b2k
