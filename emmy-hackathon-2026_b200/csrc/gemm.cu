// 3xTF32 FP32 GEMM on the 5th-generation tensor cores (tcgen05, sm_100a).
//
// C[M,N] = epilogue(A[M,K] * B[K,N]), every product computed as the three-term
// TF32 expansion hi*hi + hi*lo + lo*hi with FP32 accumulation -- the
// arithmetic contract of the reference's tensor-core emitter
// (tf32_emitter.py:22-96 model, :291-710 production_ptx, three mma.sync per
// K step and a hh+hl+lh epilogue at :675-684).
//
// Pipeline (per CTA, one 128 x BN output tile):
//   split pre-pass   A -> A_hi, A_lo ; B -> B_hi, B_lo (K-major, K padded to 32),
//                    once per GEMM instead of once per element per K step
//                    (A and a K-major B in one launch)
//   warp 0           TMA producer: four swizzled tiles (A/B hi/lo) per stage
//   warp 1           TMEM allocator + MMA issuer (the whole warp runs the
//                    loop, one elected lane issues): per 8-wide K step,
//                    lo*hi, hi*lo and hi*hi into one FP32 TMEM accumulator
//                    (128 lanes x BN columns) per 256-wide K chunk,
//                    double-buffered
//   warps 2..9       epilogue: fold each chunk into FP32 registers, then
//                    bias -> ReLU -> C staged in shared memory -> TMA stores
//                    (row stores when C is not TMA-writable)
// The tensor-core kernel is launched with programmatic dependent launch: its
// set-up overlaps the split kernel's tail.  All mbarrier waits are bounded
// (see sm100.cuh).
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "sm100.cuh"
#include "tmap.cuh"

namespace {

constexpr int BM = 128;

// --- split pre-pass --------------------------------------------------------
// (the split rule split_tf32 lives in common.cuh)

// Row-major operand rows -> hi/lo rows [R][Kp] (R = batch * rows), zero
// padded along K.  A block is 16 rows x 32 float4 columns: blockIdx.x picks
// the 128-column slice, blockIdx.y (strided) the 16-row tile, over the tiles
// of job 0 and then of job 1, so two operands split in one launch.  Each
// thread loads its two rows (threadIdx.y + 8 u) before it splits and stores
// either.  Two rows per thread (37 registers, six blocks per SM) measured
// 1.6 % faster on the ragged 4097 x 1000 x 777 GEMM than four rows (56
// registers, four blocks per SM); bounding the registers further spilled or
// ran slower.
struct RowSplitJob {
  const float *src;
  float *hi, *lo;
  int64_t rows;        // rows per batch entry (all rows when the batch is contiguous)
  int64_t k, ld, bs;   // valid columns, row stride, batch stride (elements)
  int64_t total_rows;  // batch * rows
  int64_t tiles;       // row tiles
  int vec;             // rows 16-byte aligned: float4 loads
};
constexpr int kSplitRows = 16;  // rows per tile
constexpr int kSplitRowsPerThread = kSplitRows / 8;

__global__ void __launch_bounds__(256) split_rows_kernel(const RowSplitJob j0, const RowSplitJob j1, int64_t Kp) {
  grid_dependency_wait();
  grid_dependents_launch();
  const int64_t k = ((int64_t)blockIdx.x * 32 + threadIdx.x) * 4;
  if (k >= Kp) return;
  const int64_t tiles = j0.tiles + j1.tiles;
  for (int64_t t = blockIdx.y; t < tiles; t += gridDim.y) {
    const bool second = t >= j0.tiles;
    const int64_t R0 = (second ? t - j0.tiles : t) * kSplitRows + threadIdx.y;
    const int64_t total_rows = second ? j1.total_rows : j0.total_rows;
    const int64_t rows = second ? j1.rows : j0.rows, K = second ? j1.k : j0.k;
    const int64_t ld = second ? j1.ld : j0.ld, bs = second ? j1.bs : j0.bs;
    const float *src = second ? j1.src : j0.src;
    const bool vec = (second ? j1.vec : j0.vec) && k + 3 < K;
    float4 v[kSplitRowsPerThread];
#pragma unroll
    for (int u = 0; u < kSplitRowsPerThread; ++u) {
      const int64_t R = R0 + 8 * u;
      v[u] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      if (R < total_rows) {
        const float *row = rows == total_rows ? src + R * ld : src + (R / rows) * bs + (R % rows) * ld;
        if (vec) {
          v[u] = __ldg(reinterpret_cast<const float4 *>(row + k));
        } else {
          v[u].x = k < K ? __ldg(row + k) : 0.0f;
          v[u].y = k + 1 < K ? __ldg(row + k + 1) : 0.0f;
          v[u].z = k + 2 < K ? __ldg(row + k + 2) : 0.0f;
          v[u].w = k + 3 < K ? __ldg(row + k + 3) : 0.0f;
        }
      }
    }
    float *hi = second ? j1.hi : j0.hi, *lo = second ? j1.lo : j0.lo;
#pragma unroll
    for (int u = 0; u < kSplitRowsPerThread; ++u) {
      const int64_t R = R0 + 8 * u;
      if (R < total_rows) {
        float4 h, l;
        split_tf32x4(v[u], h, l);
        *reinterpret_cast<float4 *>(hi + R * Kp + k) = h;
        *reinterpret_cast<float4 *>(lo + R * Kp + k) = l;
      }
    }
  }
}

// Row-major B [batch][K, N] (row stride ld, batch stride bs) -> transposed
// hi/lo [batch][N][Kp] (K-major), zero padded.  A block moves a 32 (k) x 128
// (n) tile: rows of 128 n read as float4 (VEC: 16-byte aligned rows), then
// per output row n its 32 k written as eight float4 of hi and of lo.  In
// shared memory element (k, n) sits at k * 128 + (n ^ 4 * (k / 4)): the
// float4 writes of a row and the column reads (lanes over k / 4 and four n)
// are both free of bank conflicts.  blockIdx.z is the batch.
constexpr int kTrK = 32, kTrN = 128;

__device__ __forceinline__ int tr_col(int k, int n) { return n ^ ((k >> 2) << 2); }

template <bool VEC>
__global__ void __launch_bounds__(256) split_transpose_kernel(const float *__restrict__ src, int64_t K, int64_t N,
                                                              int64_t ld, int64_t bs, int64_t Kp,
                                                              float *__restrict__ hi, float *__restrict__ lo) {
  __shared__ __align__(16) float tile[kTrK * kTrN];
  grid_dependency_wait();
  grid_dependents_launch();
  const int64_t k0 = (int64_t)blockIdx.y * kTrK, n0 = (int64_t)blockIdx.x * kTrN;
  const float *base = src + (int64_t)blockIdx.z * bs;
  float *hb = hi + (int64_t)blockIdx.z * N * Kp, *lb = lo + (int64_t)blockIdx.z * N * Kp;
  const int t = threadIdx.x;
  {
    // load: thread t covers n = 4 (t % 32) .. +3 of rows k = t / 32 + 8 i
    const int nl = 4 * (t & 31);
    const int64_t n = n0 + nl;
#pragma unroll
    for (int i = 0; i < kTrK; i += 8) {
      const int kl = (t >> 5) + i;
      const int64_t k = k0 + kl;
      float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      if (k < K) {
        const float *row = base + k * ld;
        if (VEC && n + 3 < N) {
          v = __ldg(reinterpret_cast<const float4 *>(row + n));
        } else {
          v.x = n < N ? __ldg(row + n) : 0.0f;
          v.y = n + 1 < N ? __ldg(row + n + 1) : 0.0f;
          v.z = n + 2 < N ? __ldg(row + n + 2) : 0.0f;
          v.w = n + 3 < N ? __ldg(row + n + 3) : 0.0f;
        }
      }
      *reinterpret_cast<float4 *>(&tile[kl * kTrN + tr_col(kl, nl)]) = v;
    }
  }
  __syncthreads();
  {
    // store: thread t writes k = 4 (t % 8) .. +3 of output rows n = t / 8 + 32 i
    const int kl = 4 * (t & 7);
    const int64_t k = k0 + kl;
    if (k < Kp) {  // Kp is a multiple of 32: the float4 never straddles it
#pragma unroll
      for (int i = 0; i < kTrN; i += 32) {
        const int nl = (t >> 3) + i;
        const int64_t n = n0 + nl;
        if (n < N) {
          const int c = tr_col(kl, nl);  // the same column for k .. k + 3
          const float4 v = make_float4(tile[kl * kTrN + c], tile[(kl + 1) * kTrN + c], tile[(kl + 2) * kTrN + c],
                                       tile[(kl + 3) * kTrN + c]);
          float4 h, l;
          split_tf32x4(v, h, l);
          *reinterpret_cast<float4 *>(hb + n * Kp + k) = h;
          *reinterpret_cast<float4 *>(lb + n * Kp + k) = l;
        }
      }
    }
  }
}

// --- main kernel -----------------------------------------------------------
// The tensor core's in-instruction accumulation is not round-to-nearest: its
// error grows linearly with the number of MMAs folded into one accumulator
// (measured ~1.1e-8 relative per MMA on B200, 2.8e-6 at K = 256).  So K is
// cut into chunks of kChunkK: each chunk accumulates into a fresh TMEM
// buffer (two buffers, double-buffered), and the epilogue warps fold every
// finished chunk into FP32 registers with round-to-nearest adds while the
// tensor core fills the other buffer.
constexpr int kChunkK = 256;
constexpr int kEpilogueWarps = 8;
constexpr int kThreads = 64 + 32 * kEpilogueWarps;  // producer, MMA, epilogue

struct GemmArgs {
  float *c;
  const float *bias;
  const float *div_ptr;  // epilogue divisor read from device memory (or null)
  float div_value;       // epilogue divisor when div_ptr is null (1 = none)
  int64_t m, n, ldc, batch_stride_c;
  int num_kb;
  int relu;
  unsigned *err;
  int tma_c;  // C written by TMA stores from shared memory (main kernel only)
};

// C staging for the TMA store: BN / 32 boxes of 128 rows x 32 FP32 (16 KB)
// with the 128-byte swizzle; a warp's row-per-thread 16-byte writes then hit
// eight distinct chunks per 128 bytes, and TMA clips the ragged edges.
constexpr int kCBox = BM * 32 * 4;

template <int BN, int SW, int STAGES>
struct GemmShape {
  static constexpr int BK = SW / 4;                       // FP32 elements per K block
  static constexpr int kTileA = BM * SW;                  // bytes of one A tile
  static constexpr int kTileB = BN * SW;
  static constexpr int kStage = 2 * kTileA + 2 * kTileB;  // hi + lo of A and B
  static constexpr int kSmem = STAGES * kStage + 1024;
  static constexpr int kChunkBlocks = kChunkK / BK;
  static constexpr int kColsPerThread = BN / 2;           // two epilogue warps per TMEM lane quarter
  // tcgen05.alloc takes a power of two >= 32 columns; two accumulators of BN.
  static constexpr uint32_t kTmemCols = 2 * BN <= 256 ? 256u : 512u;
  static_assert(BN == 128 || BN == 192 || BN == 256, "BN");
  static_assert(kSmem <= 227 * 1024, "stage ring exceeds shared memory");
};

// TMA_C selects the C write path at compile time: one kernel holding both
// paths needs more registers than the 168 a 320-thread CTA may use, and its
// spills cost more than the whole epilogue.
//
// PARTIAL (chunk split, batch 1 only): blockIdx.z is a 256-wide K chunk
// instead of a batch entry.  The CTA accumulates that one chunk and stores
// the raw accumulator (no fold, divisor, bias or ReLU) through map_c, a map
// over the partial arena [chunks][m][round_up(n, 4)]; chunk_fold_kernel then
// folds the chunks in order exactly as the epilogue below does.
template <int BN, int SW, int STAGES, bool TMA_C, bool PARTIAL = false>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tf32x3_kernel(const __grid_constant__ CUtensorMap map_ahi, const __grid_constant__ CUtensorMap map_alo,
                       const __grid_constant__ CUtensorMap map_bhi, const __grid_constant__ CUtensorMap map_blo,
                       const __grid_constant__ CUtensorMap map_c, const GemmArgs args) {
  static_assert(!PARTIAL || TMA_C, "partial accumulators leave through TMA stores");
  using Shape = GemmShape<BN, SW, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[STAGES];
  __shared__ __align__(8) uint64_t empty_bar[STAGES];
  __shared__ __align__(8) uint64_t tmem_full[2];
  __shared__ __align__(8) uint64_t tmem_empty[2];
  __shared__ __align__(8) uint64_t drain_bar;
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_word;
  __shared__ float bias_tile[BN];  // this tile's bias columns (TMA_C epilogue)

  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t n0 = (int64_t)blockIdx.x * BN;
  const int64_t m0 = (int64_t)blockIdx.y * BM;
  // PARTIAL: this CTA's K blocks are chunk blockIdx.z's; the operand maps'
  // batch coordinate is 0.
  const int kb_base = PARTIAL ? (int)blockIdx.z * Shape::kChunkBlocks : 0;
  const int num_kb = PARTIAL ? min(Shape::kChunkBlocks, args.num_kb - kb_base) : args.num_kb;
  const int zb = PARTIAL ? 0 : (int)blockIdx.z;
  const int num_chunks = (num_kb + Shape::kChunkBlocks - 1) / Shape::kChunkBlocks;
  volatile int *abort = &abort_word;

  auto a_hi = [&](int s) { return smem + s * Shape::kStage; };
  auto a_lo = [&](int s) { return smem + s * Shape::kStage + Shape::kTileA; };
  auto b_hi = [&](int s) { return smem + s * Shape::kStage + 2 * Shape::kTileA; };
  auto b_lo = [&](int s) { return smem + s * Shape::kStage + 2 * Shape::kTileA + Shape::kTileB; };

  if (threadIdx.x == 0) {
    abort_word = 0;
    for (int s = 0; s < STAGES; ++s) {
      sm100::mbar_init(&full_bar[s], 1);
      sm100::mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      sm100::mbar_init(&tmem_full[b], 1);
      sm100::mbar_init(&tmem_empty[b], kEpilogueWarps);
    }
    sm100::mbar_init(&drain_bar, 1);
    sm100::fence_barrier_init();
    sm100::prefetch_tensormap(&map_ahi);
    sm100::prefetch_tensormap(&map_alo);
    sm100::prefetch_tensormap(&map_bhi);
    sm100::prefetch_tensormap(&map_blo);
  }
  if (warp == 1) sm100::tmem_alloc(&tmem_slot, Shape::kTmemCols);
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem_base = tmem_slot;
  // Nothing above touched global memory: under programmatic dependent
  // launch the set-up overlaps the split kernel's tail.
  grid_dependency_wait();
  grid_dependents_launch();

  if (warp == 0) {
    if (sm100::elect_lane0()) {
      // TMA producer.
      int issued = 0;
      for (int kb = 0; kb < num_kb; ++kb) {
        const int s = kb % STAGES;
        const uint32_t round = kb / STAGES;
        if (kb >= STAGES &&
            !sm100::mbar_wait(&empty_bar[s], (round & 1) ^ 1, args.err, sm100::kSiteProducerEmpty, abort))
          break;
        sm100::mbar_arrive_expect_tx(&full_bar[s], Shape::kStage);
        const int kx = (kb_base + kb) * Shape::BK;
        const int z = zb;
        sm100::tma_load_3d(a_hi(s), &map_ahi, &full_bar[s], kx, (int)m0, z);
        sm100::tma_load_3d(a_lo(s), &map_alo, &full_bar[s], kx, (int)m0, z);
        sm100::tma_load_3d(b_hi(s), &map_bhi, &full_bar[s], kx, (int)n0, z);
        sm100::tma_load_3d(b_lo(s), &map_blo, &full_bar[s], kx, (int)n0, z);
        issued = kb + 1;
      }
      // Drain: every issued load must land before the CTA may exit.  These
      // waits ignore the abort word (budget only): the data is in flight.
      int never = 0;
      for (int kb = issued > STAGES ? issued - STAGES : 0; kb < issued; ++kb)
        sm100::mbar_wait(&full_bar[kb % STAGES], (kb / STAGES) & 1, args.err, sm100::kSiteDrain, &never);
    }
  } else if (warp == 1) {
    {
      // MMA issuer: chunk c accumulates into TMEM buffer c & 1.
      constexpr uint32_t idesc = sm100::idesc_tf32(BM, BN);
      for (int kb = 0; kb < num_kb; ++kb) {
        const int chunk = kb / Shape::kChunkBlocks;
        const int buf = chunk & 1;
        const bool first = (kb % Shape::kChunkBlocks) == 0;
        const bool last = ((kb + 1) % Shape::kChunkBlocks) == 0 || kb + 1 == num_kb;
        if (first && chunk >= 2 &&
            !sm100::mbar_wait_warp(&tmem_empty[buf], ((chunk >> 1) & 1) ^ 1, args.err, sm100::kSiteMmaFull, abort))
          break;
        const int s = kb % STAGES;
        if (!sm100::mbar_wait_warp(&full_bar[s], (kb / STAGES) & 1, args.err, sm100::kSiteMmaFull, abort)) break;
        sm100::tc_fence_after();
        const uint32_t d = tmem_base + (uint32_t)(buf * BN);
        const uint32_t ahi = sm100::smem_addr(a_hi(s)), alo = sm100::smem_addr(a_lo(s));
        const uint32_t bhi = sm100::smem_addr(b_hi(s)), blo = sm100::smem_addr(b_lo(s));
#pragma unroll
        for (int k = 0; k < Shape::BK / 8; ++k) {
          const uint32_t off = k * 32;  // 8 TF32 elements = 32 bytes along the swizzled row
          const uint64_t dah = sm100::desc_kmajor<SW>(ahi + off), dal = sm100::desc_kmajor<SW>(alo + off);
          const uint64_t dbh = sm100::desc_kmajor<SW>(bhi + off), dbl = sm100::desc_kmajor<SW>(blo + off);
          sm100::mma_tf32(d, dal, dbh, idesc, (first && k == 0) ? 0u : 1u);
          sm100::mma_tf32(d, dah, dbl, idesc, 1u);
          sm100::mma_tf32(d, dah, dbh, idesc, 1u);
        }
        sm100::mma_commit(&empty_bar[s]);
        if (last) sm100::mma_commit(&tmem_full[buf]);
      }
      // Every MMA issued so far must finish before TMEM is released.
      sm100::mma_commit(&drain_bar);
      int never = 0;
      sm100::mbar_wait(&drain_bar, 0, args.err, sm100::kSiteDrain, &never);
    }
  } else {
    // Epilogue warps 2..9: warp w reads TMEM lanes 32*(w%4)..+31 (its lane
    // quarter) and half (w-2)/4 of the BN columns.
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    constexpr int CPT = Shape::kColsPerThread;
    float acc[CPT];
#pragma unroll
    for (int j = 0; j < CPT; ++j) acc[j] = 0.0f;
    if (TMA_C && !PARTIAL && args.bias) {
      // The tile's bias columns, read once while the first chunk accumulates;
      // the staging loop then reads them as shared-memory broadcasts.
      for (int i = threadIdx.x - 64; i < BN; i += 32 * kEpilogueWarps)
        bias_tile[i] = n0 + i < args.n ? __ldg(args.bias + n0 + i) : 0.0f;
      sm100::named_barrier(2, 32 * kEpilogueWarps);
    }
    bool ok = true;
    for (int chunk = 0; chunk < num_chunks; ++chunk) {
      const int buf = chunk & 1;
      ok = sm100::mbar_wait(&tmem_full[buf], (chunk >> 1) & 1, args.err, sm100::kSiteEpilogueAccum, abort,
                            3 * sm100::kWaitCycles);
      if (!ok) break;
      sm100::tc_fence_after();
      const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(buf * BN + half * CPT);
      // 16 columns per load: CPT accumulators + 16 loaded values stay within
      // the register budget of a 320-thread CTA (168), with no spills.
#pragma unroll
      for (int j = 0; j < CPT; j += 16) {
        uint32_t r[16];
        sm100::tmem_ld_32x32b_x16(taddr + j, r);
        sm100::tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 16; ++i)
          acc[j + i] = PARTIAL ? __uint_as_float(r[i]) : __fadd_rn(acc[j + i], __uint_as_float(r[i]));
      }
      sm100::tc_fence_before();
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(&tmem_empty[buf]);
    }
    const int64_t row = m0 + quarter * 32 + lane;
    const int64_t col0 = n0 + half * CPT;
    if constexpr (TMA_C) {
      // The ring is idle once the last chunk is folded: stage C there, one
      // 128 x 32 box at a time per column half, and let the half's first
      // thread store each box as soon as its four warps have written it, so
      // the stores overlap the staging of the next box.
      const float divisor = args.div_ptr ? __ldg(args.div_ptr) : args.div_value;
      const bool divide = args.div_ptr != nullptr || args.div_value != 1.0f;
      const int r = quarter * 32 + lane;
      const bool has_bias = args.bias != nullptr;
      const bool leader = threadIdx.x == (unsigned)(64 + 128 * half);
#pragma unroll
      for (int b = 0; b < CPT / 32; ++b) {
        if (ok) {
#pragma unroll
          for (int j = 32 * b; j < 32 * b + 32; j += 4) {
            float v[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              float x = acc[j + q];
              if (!PARTIAL) {
                if (divide) x = __fdiv_rn(x, divisor);
                if (has_bias) x = __fadd_rn(x, bias_tile[half * CPT + j + q]);
                if (args.relu) x = x > 0.0f ? x : 0.0f;
              }
              v[q] = x;
            }
            const int col = half * CPT + j;
            const int chunk = ((col & 31) >> 2) ^ (r & 7);
            *reinterpret_cast<float4 *>(smem + (col >> 5) * kCBox + r * 128 + chunk * 16) =
                make_float4(v[0], v[1], v[2], v[3]);
          }
        }
        sm100::fence_proxy_async_smem();
        sm100::named_barrier(3 + half * 4 + b, 128);  // this half's four warps
        if (leader && ok) {
          const int box = half * (CPT / 32) + b;
          sm100::tma_store_3d(&map_c, smem + box * kCBox, (int)n0 + 32 * box, (int)m0, (int)blockIdx.z);  // z: chunk when PARTIAL
        }
      }
      if (leader && ok) sm100::tma_store_flush();
    } else if (ok && row < args.m && col0 < args.n) {
      float *crow = args.c + (int64_t)blockIdx.z * args.batch_stride_c + row * args.ldc + col0;
      const float divisor = args.div_ptr ? __ldg(args.div_ptr) : args.div_value;
      const bool divide = args.div_ptr != nullptr || args.div_value != 1.0f;
      const bool vec = ((args.ldc & 3) == 0) && ((args.batch_stride_c & 3) == 0) &&
                       ((reinterpret_cast<uintptr_t>(args.c) & 15) == 0) && col0 + CPT <= args.n;
      const int64_t ncols = args.n - col0;
      // Four columns at a time, each group stored as soon as it is final.
#pragma unroll
      for (int j = 0; j < CPT; j += 4) {
        float v[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float x = acc[j + q];
          if (divide) x = __fdiv_rn(x, divisor);
          if (args.bias) x = __fadd_rn(x, (j + q < ncols) ? __ldg(args.bias + col0 + j + q) : 0.0f);
          if (args.relu) x = x > 0.0f ? x : 0.0f;
          v[q] = x;
        }
        if (vec) {
          *reinterpret_cast<float4 *>(crow + j) = make_float4(v[0], v[1], v[2], v[3]);
        } else {
#pragma unroll
          for (int q = 0; q < 4; ++q)
            if (j + q < ncols) crow[j + q] = v[q];
        }
      }
    }
  }
  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem_base, Shape::kTmemCols);
  }
}

// Chunk split, second kernel: folds the raw chunk accumulators that the
// PARTIAL kernel left in `part` ([chunks][m][ldp]) in chunk order -- acc = 0,
// then acc = acc + chunk with round-to-nearest for each chunk in turn, the
// fold of gemm_tf32x3_kernel's epilogue -- then applies the divisor, the
// bias and ReLU in that epilogue's order and writes C.  So C is bit for bit
// what the unsplit kernel writes.  Four columns of one row per thread.
__global__ void __launch_bounds__(256)
    chunk_fold_kernel(const float *__restrict__ part, int chunks, int64_t m, int64_t n, int64_t ldp,
                      float *__restrict__ c, int64_t ldc, const float *__restrict__ bias, int relu,
                      const float *__restrict__ div_ptr, float div_value, int vec_c) {
  grid_dependency_wait();
  const float divisor = div_ptr ? __ldg(div_ptr) : div_value;
  const bool divide = div_ptr != nullptr || div_value != 1.0f;
  const int64_t quads = ldp / 4, total = m * quads, plane = m * ldp;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i / quads, col = (i - row * quads) * 4;
    const float *p = part + row * ldp + col;
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    // Four chunks' loads in flight at a time, added strictly in chunk order.
    for (int g0 = 0; g0 < chunks; g0 += 4) {
      float4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (g0 + u < chunks) v[u] = __ldcs(reinterpret_cast<const float4 *>(p + (int64_t)(g0 + u) * plane));
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (g0 + u < chunks) {
          acc[0] = __fadd_rn(acc[0], v[u].x);
          acc[1] = __fadd_rn(acc[1], v[u].y);
          acc[2] = __fadd_rn(acc[2], v[u].z);
          acc[3] = __fadd_rn(acc[3], v[u].w);
        }
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float x = acc[q];
      if (divide) x = __fdiv_rn(x, divisor);
      if (bias) x = __fadd_rn(x, col + q < n ? __ldg(bias + col + q) : 0.0f);
      if (relu) x = x > 0.0f ? x : 0.0f;
      acc[q] = x;
    }
    float *crow = c + row * ldc + col;
    if (vec_c && col + 4 <= n) {
      *reinterpret_cast<float4 *>(crow) = make_float4(acc[0], acc[1], acc[2], acc[3]);
    } else {
#pragma unroll
      for (int q = 0; q < 4; ++q)
        if (col + q < n) crow[q] = acc[q];
    }
  }
}

// --- host side -------------------------------------------------------------
// K-major FP32 operand [batch][rows][Kp]: box [1, box_rows, SW/4] with the
// SW-byte swizzle.
int make_operand_map(b2k_ctx *ctx, CUtensorMap *map, const float *base, int64_t rows, int64_t Kp, int64_t batch,
                     int box_rows, int sw) {
  auto encode = b2k::tensor_map_encoder();
  if (!encode) return b2k::fail(ctx, B2K_ECUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[3] = {(cuuint64_t)Kp, (cuuint64_t)rows, (cuuint64_t)batch};
  cuuint64_t strides[2] = {(cuuint64_t)Kp * 4, (cuuint64_t)(rows * Kp * 4)};
  cuuint32_t box[3] = {(cuuint32_t)(sw / 4), (cuuint32_t)box_rows, 1};
  cuuint32_t elem[3] = {1, 1, 1};
  const CUtensorMapSwizzle swizzle = sw == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  CUresult res = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float *>(base), dims, strides, box, elem,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (res != CUDA_SUCCESS) return b2k::fail(ctx, B2K_ECUDA, "cuTensorMapEncodeTiled failed (%d)", (int)res);
  return B2K_OK;
}

template <int BN, int SW, int STAGES>
int launch_main(b2k_ctx *ctx, const b2k::SplitOperands &ops, int64_t batch, GemmArgs args, cudaStream_t s) {
  using Shape = GemmShape<BN, SW, STAGES>;
  CUtensorMap maps[4];
  int status;
  if ((status = make_operand_map(ctx, &maps[0], ops.a_hi, args.m, ops.kp, batch, BM, SW)) != B2K_OK) return status;
  if ((status = make_operand_map(ctx, &maps[1], ops.a_lo, args.m, ops.kp, batch, BM, SW)) != B2K_OK) return status;
  if ((status = make_operand_map(ctx, &maps[2], ops.b_hi, args.n, ops.kp, batch, BN, SW)) != B2K_OK) return status;
  if ((status = make_operand_map(ctx, &maps[3], ops.b_lo, args.n, ops.kp, batch, BN, SW)) != B2K_OK) return status;
  args.num_kb = (int)(ops.kp / Shape::BK);
  // C through TMA stores when it is TMA-writable, else row stores by the threads.
  CUtensorMap map_c{};
  args.tma_c = b2k::aligned16(args.c) && args.ldc % 4 == 0 && (batch == 1 || args.batch_stride_c % 4 == 0);
  if (args.tma_c) {
    auto encode = b2k::tensor_map_encoder();
    if (!encode) return b2k::fail(ctx, B2K_ECUDA, "cuTensorMapEncodeTiled is unavailable");
    cuuint64_t dims[3] = {(cuuint64_t)args.n, (cuuint64_t)args.m, (cuuint64_t)batch};
    cuuint64_t strides[2] = {(cuuint64_t)args.ldc * 4,
                             (cuuint64_t)(batch == 1 ? args.m * args.ldc : args.batch_stride_c) * 4};
    cuuint32_t box[3] = {32, (cuuint32_t)BM, 1};
    cuuint32_t elem[3] = {1, 1, 1};
    CUresult res = encode(&map_c, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, args.c, dims, strides, box, elem,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (res != CUDA_SUCCESS) return b2k::fail(ctx, B2K_ECUDA, "cuTensorMapEncodeTiled (C) failed (%d)", (int)res);
  }
  static_assert((BN / 32) * kCBox <= STAGES * Shape::kStage, "C staging exceeds the ring");
  auto kernel = args.tma_c ? gemm_tf32x3_kernel<BN, SW, STAGES, true> : gemm_tf32x3_kernel<BN, SW, STAGES, false>;
  cudaError_t err = b2k::set_max_smem(ctx, (const void *)kernel, Shape::kSmem);
  if (err != cudaSuccess) return b2k::cuda_fail(ctx, err, "gemm: set smem");
  dim3 grid((unsigned)((args.n + BN - 1) / BN), (unsigned)((args.m + BM - 1) / BM), (unsigned)batch);
  err = b2k::launch_kernel(b2k::pdl_enabled(), kernel, grid, dim3(kThreads), Shape::kSmem, s, maps[0], maps[1],
                           maps[2], maps[3], map_c, args);
  if (err != cudaSuccess) return b2k::cuda_fail(ctx, err, "gemm launch");
  return b2k::check_launch(ctx, "gemm launch");
}

// Chunk split: every (128 x 128 tile, 256-wide K chunk) pair is one CTA of
// the PARTIAL kernel, then chunk_fold_kernel folds the chunks in order and
// applies the epilogue.  Batch 1 only.
int launch_chunked(b2k_ctx *ctx, const b2k::SplitOperands &ops, GemmArgs args, cudaStream_t s) {
  using Shape = GemmShape<128, 128, 3>;
  const int num_kb = (int)(ops.kp / Shape::BK);
  const int64_t chunks = (num_kb + Shape::kChunkBlocks - 1) / Shape::kChunkBlocks;
  const int64_t ldp = (args.n + 3) / 4 * 4;
  int status = b2k::reserve_partials(ctx, (size_t)(chunks * args.m * ldp) * sizeof(float), s);
  if (status != B2K_OK) return status;
  float *part = static_cast<float *>(ctx->partials);
  CUtensorMap maps[4];
  if ((status = make_operand_map(ctx, &maps[0], ops.a_hi, args.m, ops.kp, 1, BM, 128)) != B2K_OK) return status;
  if ((status = make_operand_map(ctx, &maps[1], ops.a_lo, args.m, ops.kp, 1, BM, 128)) != B2K_OK) return status;
  if ((status = make_operand_map(ctx, &maps[2], ops.b_hi, args.n, ops.kp, 1, 128, 128)) != B2K_OK) return status;
  if ((status = make_operand_map(ctx, &maps[3], ops.b_lo, args.n, ops.kp, 1, 128, 128)) != B2K_OK) return status;
  // the partial arena as [chunks][m][ldp], written in the C map's 128 x 32 boxes
  auto encode = b2k::tensor_map_encoder();
  if (!encode) return b2k::fail(ctx, B2K_ECUDA, "cuTensorMapEncodeTiled is unavailable");
  CUtensorMap map_p{};
  cuuint64_t dims[3] = {(cuuint64_t)args.n, (cuuint64_t)args.m, (cuuint64_t)chunks};
  cuuint64_t strides[2] = {(cuuint64_t)ldp * 4, (cuuint64_t)(args.m * ldp) * 4};
  cuuint32_t box[3] = {32, (cuuint32_t)BM, 1};
  cuuint32_t elem[3] = {1, 1, 1};
  CUresult res = encode(&map_p, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, part, dims, strides, box, elem,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (res != CUDA_SUCCESS) return b2k::fail(ctx, B2K_ECUDA, "cuTensorMapEncodeTiled (partials) failed (%d)", (int)res);
  GemmArgs pargs = args;
  pargs.num_kb = num_kb;
  pargs.tma_c = 1;
  auto kernel = gemm_tf32x3_kernel<128, 128, 3, true, true>;
  cudaError_t err = b2k::set_max_smem(ctx, (const void *)kernel, Shape::kSmem);
  if (err != cudaSuccess) return b2k::cuda_fail(ctx, err, "gemm (chunks): set smem");
  const dim3 grid((unsigned)((args.n + 127) / 128), (unsigned)((args.m + BM - 1) / BM), (unsigned)chunks);
  err = b2k::launch_kernel(b2k::pdl_enabled(), kernel, grid, dim3(kThreads), Shape::kSmem, s, maps[0], maps[1],
                           maps[2], maps[3], map_p, pargs);
  if (err != cudaSuccess) return b2k::cuda_fail(ctx, err, "gemm (chunks) launch");
  if ((status = b2k::check_launch(ctx, "gemm (chunks) launch")) != B2K_OK) return status;
  const int64_t quads = args.m * (ldp / 4);
  const int64_t blocks = std::max<int64_t>(1, std::min<int64_t>((quads + 255) / 256, (int64_t)ctx->sm_count * 8));
  const int vec_c = b2k::aligned16(args.c) && args.ldc % 4 == 0;
  err = b2k::launch_kernel(b2k::pdl_enabled(), chunk_fold_kernel, dim3((unsigned)blocks), dim3(256), 0, s,
                           (const float *)part, (int)chunks, args.m, args.n, ldp, args.c, args.ldc, args.bias,
                           args.relu, args.div_ptr, args.div_value, vec_c);
  if (err != cudaSuccess) return b2k::cuda_fail(ctx, err, "chunk fold launch");
  return b2k::check_launch(ctx, "chunk fold launch");
}

}  // namespace

// Kernel variant selector (tile width, swizzle, stage count); settable for
// tuning through b2k_gemm_set_variant.  Outputs at most 128 wide always use
// the 128-wide tile.
static int g_gemm_variant = 1;
// Chunk split of the pre-pass kernel (b2k_gemm_set_chunk_split): 0 never,
// 1 where the estimate says it is faster (default), 2 wherever it applies.
static int g_chunk_split = 1;
namespace b2k {

static void fill_job(RowSplitJob &o, const RowSplit &r) {
  // A batch stored back to back is one tall matrix: no per-row division.
  const bool flat = r.batch == 1 || r.bs == r.rows * r.ld;
  o.src = r.src;
  o.hi = r.hi;
  o.lo = r.lo;
  o.total_rows = r.rows * r.batch;
  o.rows = flat ? o.total_rows : r.rows;
  o.k = r.k;
  o.ld = r.ld;
  o.bs = r.bs;
  o.tiles = (o.total_rows + kSplitRows - 1) / kSplitRows;
  o.vec = r.ld % 4 == 0 && (flat || r.bs % 4 == 0) && aligned16(r.src);
}

int split_rows2(b2k_ctx *ctx, const RowSplit &a, const RowSplit *b, int64_t kp, cudaStream_t s) {
  RowSplitJob j[2] = {};
  fill_job(j[0], a);
  if (b) fill_job(j[1], *b);
  const int64_t tiles = j[0].tiles + j[1].tiles;
  if (tiles == 0 || kp == 0) return B2K_OK;
  const dim3 grid((unsigned)((kp / 4 + 31) / 32), (unsigned)std::min<int64_t>(tiles, 65535));
  cudaError_t err = launch_kernel(pdl_enabled(), split_rows_kernel, grid, dim3(32, kSplitRows / kSplitRowsPerThread), 0, s, j[0], j[1], kp);
  if (err != cudaSuccess) return cuda_fail(ctx, err, "split_rows launch");
  return check_launch(ctx, "split_rows launch");
}

int split_rows(b2k_ctx *ctx, const float *src, int64_t rows, int64_t k, int64_t ld, int64_t bs, int64_t batch,
               int64_t kp, float *hi, float *lo, cudaStream_t s) {
  return split_rows2(ctx, RowSplit{src, rows, k, ld, bs, batch, hi, lo}, nullptr, kp, s);
}

int split_transpose(b2k_ctx *ctx, const float *src, int64_t k, int64_t n, int64_t ld, int64_t bs, int64_t batch,
                    int64_t kp, float *hi, float *lo, cudaStream_t s) {
  if (batch > 65535) return fail(ctx, B2K_EINVAL, "split_transpose: batch exceeds 65535");
  dim3 grid((unsigned)((n + kTrN - 1) / kTrN), (unsigned)((kp + kTrK - 1) / kTrK), (unsigned)batch);
  const bool vec = ld % 4 == 0 && (batch == 1 || bs % 4 == 0) && aligned16(src);
  cudaError_t err = vec ? launch_kernel(pdl_enabled(), split_transpose_kernel<true>, grid, dim3(256), 0, s, src, k, n,
                                        ld, bs, kp, hi, lo)
                        : launch_kernel(pdl_enabled(), split_transpose_kernel<false>, grid, dim3(256), 0, s, src, k,
                                        n, ld, bs, kp, hi, lo);
  if (err != cudaSuccess) return cuda_fail(ctx, err, "split_transpose launch");
  return check_launch(ctx, "split_transpose launch");
}

// Estimated microseconds of one pre-pass kernel launch with 128 x bn tiles:
// (waves of tiles over the SMs) x (one tile's time).  A tile is bound by the
// tensor core's operand reads from shared memory, (128 + bn) words per K
// element (A's 128 rows and B's bn), plus a fixed set-up and epilogue.
// Calibrated on B200 on the 4097 x 1000 x 777 GEMM and its row shards (2049,
// 1025 and 513 rows; one wave each, burst clock): 128 x 256 tiles
// 30.8-32.9 us, 128 x 192 26.7-28.6 us, 128 x 128 22.6-22.8 us.  The
// widths give identical bits (same products and chunk folds per element).
double prepass_cost_us(int64_t tiles, int bn, int64_t kp, int sms) {
  const int64_t waves = sms > 0 ? (tiles + sms - 1) / sms : tiles;
  return (double)waves * ((double)(128 + bn) * (double)kp * 9.86e-5 + 2.5);
}

int main_tile_width(int64_t m, int64_t n, int64_t batch, int64_t kp, int sms) {
  if (n <= 128) return 128;
  switch (g_gemm_variant) {
    case 0: return 256;
    case 2: return 128;
    case 3: return 192;
    default: {
      // the width whose tiles cover the output in the least estimated time
      // (ties to the wider tile)
      const int64_t mt = (m + BM - 1) / BM * std::max<int64_t>(batch, 1);
      int best = 256;
      double best_us = prepass_cost_us(mt * ((n + 255) / 256), 256, kp, sms);
      for (int bn : {192, 128}) {
        const double us = prepass_cost_us(mt * ((n + bn - 1) / bn), bn, kp, sms);
        if (us < best_us * 0.97) best = bn, best_us = us;
      }
      return best;
    }
  }
}

// The chunk split's estimate: its CTAs run chunk-major, so the short last
// chunk's CTAs (K of kp - 256 (chunks - 1)) fill the last waves; each CTA is
// a 128 x 128 tile of the pre-pass kernel over one chunk (the per-wave cost
// of prepass_cost_us).  The fold streams the chunks' partials once more and
// writes C: (2 chunks + 1) m n floats at ~5 TB/s, plus its launch.
double chunked_cost_us(int64_t m, int64_t n, int64_t kp, int sms) {
  if (g_chunk_split == 0 || sms <= 0) return 1e300;
  const int64_t chunks = (kp + kChunkK - 1) / kChunkK;
  if (chunks < 2 || chunks > 65535) return 1e300;
  const int64_t ldp = (n + 3) / 4 * 4;
  if ((double)chunks * (double)m * (double)ldp * 4.0 > double(size_t(1) << 31)) return 1e300;
  const int64_t tiles = ((m + BM - 1) / BM) * ((n + 127) / 128);
  const int64_t full = tiles * (chunks - 1), units = tiles * chunks;
  const int64_t waves_full = (full + sms - 1) / sms, waves = (units + sms - 1) / sms;
  const int64_t tail_k = kp - (chunks - 1) * kChunkK;
  const double t_full = 256.0 * (double)kChunkK * 9.86e-5 + 2.5, t_tail = 256.0 * (double)tail_k * 9.86e-5 + 2.5;
  return (double)waves_full * t_full + (double)(waves - waves_full) * t_tail + 2.0 +
         (double)(2 * chunks + 1) * (double)m * (double)n * 4.0 / 5.0e6;
}

bool gemm_takes_chunks(int64_t m, int64_t n, int64_t kp, int sms) {
  if (g_chunk_split == 0 || (g_gemm_variant != 1 && g_chunk_split != 2)) return false;
  const double split_us = chunked_cost_us(m, n, kp, sms);
  if (split_us >= 1e299) return false;
  if (g_chunk_split == 2) return true;
  const int bn = main_tile_width(m, n, 1, kp, sms);
  return split_us < 0.85 * prepass_cost_us(((m + BM - 1) / BM) * ((n + bn - 1) / bn), bn, kp, sms);
}

int gemm_main(b2k_ctx *ctx, const SplitOperands &ops, int64_t m, int64_t n, int64_t batch, float *c, int64_t ldc,
              int64_t batch_stride_c, const float *bias, int relu, const float *div_ptr, float div_value,
              cudaStream_t s, bool allow_chunks) {
  if (batch > 65535) return fail(ctx, B2K_EINVAL, "gemm: batch exceeds 65535");
  GemmArgs args{c, bias, div_ptr, div_value, m, n, ldc, batch_stride_c, 0, relu, ctx->error_flag, 0};
  PhaseTimer timer(ctx, B2K_PHASE_MMA, s);
  if (allow_chunks && batch == 1 && !ctx->fixed_scratch && gemm_takes_chunks(m, n, ops.kp, ctx->sm_count))
    return launch_chunked(ctx, ops, args, s);
  if (n <= 128) return launch_main<128, 128, 3>(ctx, ops, batch, args, s);
  if (g_gemm_variant == 0) return launch_main<256, 128, 2>(ctx, ops, batch, args, s);
  switch (main_tile_width(m, n, batch, ops.kp, ctx->sm_count)) {
    case 128: return launch_main<128, 128, 3>(ctx, ops, batch, args, s);
    case 192: return launch_main<192, 64, 5>(ctx, ops, batch, args, s);
    default: return launch_main<256, 64, 4>(ctx, ops, batch, args, s);
  }
}

}  // namespace b2k

// Shared by the public entry points.  By default the path with the lowest
// estimated time is taken (gemm_split_mode): a TMA-readable A split inside
// the kernel with only B pre-split into `ws` (direct orientation), a
// TMA-readable B split inside the kernel with only A pre-split into `ws`
// (transposed orientation, for short wide outputs), or both operands split
// into `ws` (A_hi, A_lo: m x Kp; B_hi, B_lo: n x Kp) for the kernel above.
// `layout`: B2K_B_NK -- B is stored [n, K] (else [K, n]); B2K_A_KM -- A is
// stored [K, m] (else [m, K]).  `ws` holds at least 2 (m + n) Kp floats.
int b2k_gemm_tf32x3_impl(b2k_ctx *ctx, const float *a, const float *b, float *c, int64_t m, int64_t n, int64_t k,
                         int64_t lda, int64_t ldb, int64_t ldc, int layout, const float *bias, int relu,
                         float *ws, cudaStream_t s, const float *div_ptr, float div_value) {
  const int b_kmajor = (layout & B2K_B_NK) != 0;
  const bool a_t = (layout & B2K_A_KM) != 0;
  // A divided product runs on the pre-pass kernel, whose epilogue divides.
  const bool divide = div_ptr != nullptr || div_value != 1.0f;
  const int mode = divide ? 0 : b2k::gemm_split_mode(a, b, m, n, k, lda, ldb, layout, ctx->sm_count, !ctx->fixed_scratch);
  const int64_t kp = b2k::gemm_kpad(k);
  int status;
  if (mode == b2k::kSplitDirect) {
    // A is split inside the kernel (into TMEM); only B is pre-split.
    b2k::SplitOperands ops{nullptr, nullptr, ws, ws + n * kp, kp};
    {
      b2k::PhaseTimer timer(ctx, B2K_PHASE_SPLIT, s);
      status = b_kmajor ? b2k::split_rows(ctx, b, n, k, ldb, n * ldb, 1, kp, ops.b_hi, ops.b_lo, s)
                        : b2k::split_transpose(ctx, b, k, n, ldb, k * ldb, 1, kp, ops.b_hi, ops.b_lo, s);
    }
    if (status != B2K_OK) return status;
    return b2k::gemm_tmem_a(ctx, a, k, lda, ops, c, m, n, ldc, bias, relu, s);
  }
  if (mode == b2k::kSplitTransposed) {
    // B is split inside the kernel (into TMEM); only A is pre-split, K-major.
    b2k::SplitOperands ops{nullptr, nullptr, ws, ws + m * kp, kp};
    {
      b2k::PhaseTimer timer(ctx, B2K_PHASE_SPLIT, s);
      status = a_t ? b2k::split_transpose(ctx, a, k, m, lda, k * lda, 1, kp, ops.b_hi, ops.b_lo, s)
                   : b2k::split_rows(ctx, a, m, k, lda, m * lda, 1, kp, ops.b_hi, ops.b_lo, s);
    }
    if (status != B2K_OK) return status;
    return b2k::gemm_tmem_b(ctx, b, k, ldb, b_kmajor != 0, ops, c, m, n, ldc, bias, relu, s);
  }
  b2k::SplitOperands ops{ws, ws + m * kp, ws + 2 * m * kp, ws + 2 * m * kp + n * kp, kp};
  {
    b2k::PhaseTimer timer(ctx, B2K_PHASE_SPLIT, s);
    const b2k::RowSplit sa{a, m, k, lda, m * lda, 1, ops.a_hi, ops.a_lo};
    if (a_t) {
      // A [K, m] -> hi/lo [m][Kp], the same transform as a [K, n] B
      status = b2k::split_transpose(ctx, a, k, m, lda, k * lda, 1, kp, ops.a_hi, ops.a_lo, s);
      if (status == B2K_OK)
        status = b_kmajor ? b2k::split_rows(ctx, b, n, k, ldb, n * ldb, 1, kp, ops.b_hi, ops.b_lo, s)
                          : b2k::split_transpose(ctx, b, k, n, ldb, k * ldb, 1, kp, ops.b_hi, ops.b_lo, s);
    } else if (b_kmajor) {
      // A and a K-major B in one launch
      const b2k::RowSplit sb{b, n, k, ldb, n * ldb, 1, ops.b_hi, ops.b_lo};
      status = b2k::split_rows2(ctx, sa, &sb, kp, s);
    } else {
      status = b2k::split_rows2(ctx, sa, nullptr, kp, s);
      if (status == B2K_OK) status = b2k::split_transpose(ctx, b, k, n, ldb, k * ldb, 1, kp, ops.b_hi, ops.b_lo, s);
    }
  }
  if (status != B2K_OK) return status;
  return b2k::gemm_main(ctx, ops, m, n, 1, c, ldc, m * ldc, bias, relu, div_ptr, div_value, s, !ctx->fixed_scratch);
}

int b2k::gemm_variant() { return g_gemm_variant; }

extern "C" int b2k_gemm_set_chunk_split(int mode) {
  if (mode < 0 || mode > 2) return B2K_EINVAL;
  g_chunk_split = mode;
  return B2K_OK;
}

// The path b2k_gemm_tf32x3 takes for a call, decided by the same functions
// in the same order as the dispatch (b2k_gemm_tf32x3_impl, then gemm_main),
// without touching the GPU.
extern "C" int b2k_gemm_plan(int32_t sms, const float *a, const float *b, int64_t m, int64_t n, int64_t k, int64_t lda,
                             int64_t ldb, int32_t b_layout, b2k_gemm_plan_info *out) {
  if (!out || sms <= 0 || m <= 0 || n <= 0 || k <= 0) return B2K_EINVAL;
  if ((b_layout & ~(B2K_B_NK | B2K_A_KM)) != 0) return B2K_EINVAL;
  if (m > INT32_MAX - 256 || n > INT32_MAX - 256 || k > INT32_MAX - 64) return B2K_EINVAL;
  const bool a_t = (b_layout & B2K_A_KM) != 0, b_nk = (b_layout & B2K_B_NK) != 0;
  if (lda < (a_t ? m : k) || ldb < (b_nk ? k : n)) return B2K_EINVAL;
  const int64_t kp = b2k::gemm_kpad(k);
  const int mode = b2k::gemm_split_mode(a, b, m, n, k, lda, ldb, b_layout, sms, true);
  out->split_mode = mode;
  out->chunks = (int32_t)((kp + kChunkK - 1) / kChunkK);
  out->chunk_split = 0;
  if (mode == b2k::kSplitDirect) {
    out->tile_width = b2k::gemm_direct_tile_width(n);
  } else if (mode == b2k::kSplitTransposed) {
    out->tile_width = b2k::gemm_transposed_tile_width(m, n, sms);
  } else if (b2k::gemm_takes_chunks(m, n, kp, sms)) {
    out->chunk_split = 1;
    out->tile_width = 128;
  } else {
    out->tile_width = n <= 128 ? 128 : g_gemm_variant == 0 ? 256 : b2k::main_tile_width(m, n, 1, kp, sms);
  }
  return B2K_OK;
}

extern "C" int b2k_gemm_set_variant(int variant) {
  if (variant < 0 || variant > 3) return B2K_EINVAL;
  g_gemm_variant = variant;
  return B2K_OK;
}

size_t b2k_gemm_workspace_bytes(int64_t m, int64_t n, int64_t k) {
  return (size_t)(2 * (m + n) * b2k::gemm_kpad(k)) * sizeof(float);
}

// Validation, scratch and dispatch shared by b2k_gemm_tf32x3 and its scaled form.
static int gemm_entry(b2k_ctx *ctx, const float *a, const float *b, float *c, int64_t m, int64_t n, int64_t k,
                      int64_t lda, int64_t ldb, int64_t ldc, int32_t b_layout, const float *bias, int32_t relu,
                      const float *div_ptr, float div_value, void *stream) {
  B2K_CHECK_CTX(ctx);
  if (m < 0 || n < 0 || k < 0) return b2k::fail(ctx, B2K_EINVAL, "gemm: negative extent");
  if ((b_layout & ~(B2K_B_NK | B2K_A_KM)) != 0) return b2k::fail(ctx, B2K_EINVAL, "gemm: bad b_layout");
  const bool a_t = (b_layout & B2K_A_KM) != 0, b_nk = (b_layout & B2K_B_NK) != 0;
  if (m == 0 || n == 0) return B2K_OK;
  if (!a || !b || !c) return b2k::fail(ctx, B2K_EINVAL, "gemm: null buffer");
  if (lda < (a_t ? m : k) || ldc < n || ldb < (b_nk ? k : n))
    return b2k::fail(ctx, B2K_EINVAL, "gemm: leading dimension too small");
  if (m > INT32_MAX - 256 || n > INT32_MAX - 256 || k > INT32_MAX - 64)
    return b2k::fail(ctx, B2K_EINVAL, "gemm: extent exceeds 32-bit TMA coordinates");
  cudaStream_t s = (cudaStream_t)stream;
  const bool divide = div_ptr != nullptr || div_value != 1.0f;
  if (k == 0) {
    // Empty contraction: C = epilogue(0).
    if (bias) return b2k::fail(ctx, B2K_EUNSUPPORTED, "gemm: bias with K = 0");
    if (divide) return b2k::fail(ctx, B2K_EUNSUPPORTED, "gemm: divisor with K = 0");
    cudaError_t err = cudaMemset2DAsync(c, (size_t)ldc * 4, 0, (size_t)n * 4, (size_t)m, s);
    if (err != cudaSuccess) return b2k::cuda_fail(ctx, err, "gemm: zero fill");
    return B2K_OK;
  }
  // scratch: the split operands
  int status = b2k::reserve_workspace(ctx, b2k_gemm_workspace_bytes(m, n, k), s);
  if (status != B2K_OK) return status;
  return b2k_gemm_tf32x3_impl(ctx, a, b, c, m, n, k, lda, ldb, ldc, b_layout, bias, relu,
                              static_cast<float *>(ctx->workspace), s, div_ptr, div_value);
}

extern "C" int b2k_gemm_tf32x3(b2k_ctx *ctx, const float *a, const float *b, float *c, int64_t m, int64_t n,
                               int64_t k, int64_t lda, int64_t ldb, int64_t ldc, int32_t b_layout,
                               const float *bias, int32_t relu, void *stream) {
  return gemm_entry(ctx, a, b, c, m, n, k, lda, ldb, ldc, b_layout, bias, relu, nullptr, 1.0f, stream);
}

extern "C" int b2k_gemm_tf32x3_batched(b2k_ctx *ctx, const float *a, const float *b, float *c, int64_t batch,
                                       int64_t m, int64_t n, int64_t k, int64_t lda, int64_t ldb, int64_t ldc,
                                       int64_t stride_a, int64_t stride_b, int64_t stride_c, int32_t b_layout,
                                       const float *bias, int32_t relu, void *stream) {
  B2K_CHECK_CTX(ctx);
  if (batch < 0 || m < 0 || n < 0 || k < 0) return b2k::fail(ctx, B2K_EINVAL, "gemm_batched: negative extent");
  if (b_layout != B2K_B_KN && b_layout != B2K_B_NK) return b2k::fail(ctx, B2K_EINVAL, "gemm_batched: bad b_layout");
  if (batch == 0 || m == 0 || n == 0) return B2K_OK;
  if (batch == 1)
    return gemm_entry(ctx, a, b, c, m, n, k, lda, ldb, ldc, b_layout, bias, relu, nullptr, 1.0f, stream);
  if (!a || !b || !c) return b2k::fail(ctx, B2K_EINVAL, "gemm_batched: null buffer");
  const bool b_nk = b_layout == B2K_B_NK;
  if (lda < k || ldc < n || ldb < (b_nk ? k : n))
    return b2k::fail(ctx, B2K_EINVAL, "gemm_batched: leading dimension too small");
  if (stride_a < m * lda || stride_b < (b_nk ? n : k) * ldb || stride_c < m * ldc)
    return b2k::fail(ctx, B2K_EINVAL, "gemm_batched: batch stride smaller than a matrix");
  if (batch > 65535) return b2k::fail(ctx, B2K_EINVAL, "gemm_batched: batch exceeds 65535");
  if (m > INT32_MAX - 256 || n > INT32_MAX - 256 || k > INT32_MAX - 64)
    return b2k::fail(ctx, B2K_EINVAL, "gemm_batched: extent exceeds 32-bit TMA coordinates");
  if (k == 0) return b2k::fail(ctx, B2K_EUNSUPPORTED, "gemm_batched: K = 0");
  cudaStream_t s = (cudaStream_t)stream;
  const int64_t kp = b2k::gemm_kpad(k);
  int status = b2k::reserve_workspace(ctx, (size_t)(2 * (m + n) * kp * batch) * sizeof(float), s);
  if (status != B2K_OK) return status;
  float *ws = static_cast<float *>(ctx->workspace);
  // [batch][rows][kp] hi/lo halves, the layout the kernel's 3-D tensor maps walk
  b2k::SplitOperands ops{ws, ws + batch * m * kp, ws + 2 * batch * m * kp, ws + 2 * batch * m * kp + batch * n * kp,
                         kp};
  {
    b2k::PhaseTimer timer(ctx, B2K_PHASE_SPLIT, s);
    const b2k::RowSplit sa{a, m, k, lda, stride_a, batch, ops.a_hi, ops.a_lo};
    if (b_nk) {
      const b2k::RowSplit sb{b, n, k, ldb, stride_b, batch, ops.b_hi, ops.b_lo};
      status = b2k::split_rows2(ctx, sa, &sb, kp, s);
    } else {
      status = b2k::split_rows2(ctx, sa, nullptr, kp, s);
      if (status == B2K_OK) status = b2k::split_transpose(ctx, b, k, n, ldb, stride_b, batch, kp, ops.b_hi, ops.b_lo, s);
    }
  }
  if (status != B2K_OK) return status;
  return b2k::gemm_main(ctx, ops, m, n, batch, c, ldc, stride_c, bias, relu, nullptr, 1.0f, s);
}

extern "C" int b2k_gemm_tf32x3_scaled(b2k_ctx *ctx, const float *a, const float *b, float *c, int64_t m, int64_t n,
                                      int64_t k, int64_t lda, int64_t ldb, int64_t ldc, int32_t b_layout,
                                      const float *bias, int32_t relu, const float *div_ptr, float div_value,
                                      void *stream) {
  return gemm_entry(ctx, a, b, c, m, n, k, lda, ldb, ldc, b_layout, bias, relu, div_ptr, div_value, stream);
}
