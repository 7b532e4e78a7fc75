// 3xTF32 GEMM on 128 x 256 output tiles with the A operand split inside the
// kernel into tensor memory, for any row stride of A.
//
// The arithmetic is the one of gemm.cu and gemm_fused.cu (the reference's
// tensor-core emitter, tf32_emitter.py:22-96 model, :647-668 split, :675-684
// hh + hl + lh): every product is hi*hi + hi*lo + lo*hi with hi = rna_tf32(x),
// lo = rna_tf32(x - hi), accumulated in FP32 chunk by chunk.
//
// Why a third tensor-core kernel.  Some outputs are covered by 128 x 256
// tiles in one wave of the 148 SMs and by 128 x 192 tiles only in two: the
// ragged 4097 x 1000 x 777 configuration is 33 x 4 = 132 tiles of 128 x 256
// against 198 of 128 x 192.  The pre-pass kernel (gemm.cu) has 128 x 256
// tiles but needs both operands split into a scratch copy first (for this
// configuration 26 MB of A hi/lo written and read back, a fifth of the step),
// and its tensor core reads A's hi and lo from shared memory three times per
// K step.  The TMEM-A kernel (gemm_fused.cu) splits A inside the kernel but
// keeps two accumulator buffers, which at N = 256 fill all 512 TMEM columns.
// This kernel keeps ONE accumulator buffer (256 columns) and a five-stage
// ring of A's hi/lo halves in the other columns.  The price is that the
// tensor core waits while the work warps fold a finished K chunk into their
// FP32 registers (a few hundred cycles per chunk, three times at K = 777).
//
// A's rows need not be 16-byte aligned.  TMA needs a row stride that is a
// multiple of 16 bytes; a row stride of `lda` floats with lda % 4 != 0 is not.
// But G consecutive rows (G = 4 for odd lda, 2 for lda = 2 mod 4) are: the
// map describes A as [m / G groups][G * lda floats].  Row G g + j, columns
// kx .. kx + 15, lie at group g, x = j lda + kx; that x is off a 16-byte
// boundary by o_j = (j lda) mod 4 floats, so the producer loads, for each
// j, a box of 20 floats starting at x - o_j (aligned) for the tile's 128 / G
// groups, and the split thread of row G g + j reads its 16 values at offset
// o_j.  Columns past K (the next row's values, or TMA's zero fill) are
// masked to zero by the thread.  Rows in the last group when the map cannot
// cover it without reading past the caller's buffer (lda > K) are loaded by
// their split thread from global memory.  With lda % 4 == 0 (G = 1) the A
// tile is the usual 64-byte-swizzled box.
//
// Roles (320 threads, 168 registers each): warp 0 TMA producer (A boxes and
// the pre-split B_hi / B_lo tiles, 256 x 16 each), warp 1 TMEM allocator and
// MMA issuer (warp-wide, one elected lane issues lo*hi, hi*lo, hi*hi per
// 8-wide K step, M = 128, N = 256, A from TMEM), warps 2..9 split A and hold
// the accumulator: warp w owns TMEM lane quarter w % 4 and column half
// (w - 2) / 4 (128 FP32 accumulators per thread); the two halves split
// alternate K blocks (a thread splits all 16 values of its row).  Epilogue:
// bias, ReLU, C staged in shared memory and stored by TMA box by box (row
// stores when C is not TMA-writable).  Launched with programmatic dependent
// launch after the B split; all waits are bounded.
#include "common.cuh"
#include "sm100.cuh"
#include "tmap.cuh"

namespace {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 16;               // K per stage: 64-byte K-major rows
constexpr int kWorkWarps = 8;        // split + accumulator + epilogue
constexpr int kThreads = 64 + 32 * kWorkWarps;
constexpr int kCPT = BN / 2;         // accumulator columns per work thread
constexpr int kTileB = BN * BK * 4;  // each of B_hi, B_lo (16 KB)
constexpr int kBoxW = 20;            // floats per row of a grouped A box (16 + up to 3 of offset)
constexpr int kStages = 5;           // shared-memory ring
constexpr int kAStages = 5;          // TMEM A ring (<= kStages, see the split loop)
constexpr int kAccCols = BN;         // one accumulator buffer
constexpr int kCBox = BM * 32 * 4;   // C staging box: 128 rows x 32 FP32, 128-byte swizzle
constexpr int kMaxChunkBlocks = 24;  // K blocks per accumulation chunk, at most

static_assert(kAccCols + kAStages * 2 * BK <= 512, "TMEM columns");

template <int G>
struct WideShape {
  static constexpr int kTileA = G == 1 ? BM * BK * 4 : BM * kBoxW * 4;
  static constexpr int kBoxA = kTileA / G;  // bytes of the box of one row offset j
  static constexpr int kStage = kTileA + 2 * kTileB;
  static constexpr int kSmem = kStages * kStage + 1024;
  static_assert(kSmem <= 227 * 1024, "stage ring exceeds shared memory");
  static_assert(kBoxA % 128 == 0, "TMA destinations need 128-byte alignment");
  static_assert((BN / 32) * kCBox <= kStages * kStage, "C staging exceeds the ring");
};

struct WideArgs {
  float *c;
  const float *bias;
  const float *a;      // raw A, for the rows the grouped map does not cover
  int64_t m, n, k, lda, ldc;
  int64_t m_grouped;   // rows [0, m_grouped) come through the map
  int num_kb;
  int chunk_blocks;    // K blocks per accumulation chunk
  int relu;
  unsigned *err;
};

template <int G, bool TMA_C>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_wide_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_bhi,
                     const __grid_constant__ CUtensorMap map_blo, const __grid_constant__ CUtensorMap map_c,
                     const WideArgs args) {
  using Shape = WideShape<G>;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[kStages];   // A boxes + B hi/lo landed
  __shared__ __align__(8) uint64_t empty_bar[kStages];  // MMAs done with the block in the stage
  __shared__ __align__(8) uint64_t a_full[kAStages];    // A hi/lo of the block stored in TMEM
  __shared__ __align__(8) uint64_t tmem_full;           // a chunk has accumulated
  __shared__ __align__(8) uint64_t tmem_empty;          // the work warps have folded it
  __shared__ __align__(8) uint64_t drain_bar;
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_word;
  __shared__ float bias_tile[BN];

  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // M-fastest raster: CTAs resident together share B column tiles.
  const int64_t m0 = (int64_t)blockIdx.x * BM;
  const int64_t n0 = (int64_t)blockIdx.y * BN;
  const int num_kb = args.num_kb;
  const int cb = args.chunk_blocks;
  const int num_chunks = (num_kb + cb - 1) / cb;
  volatile int *abort = &abort_word;

  auto a_raw = [&](int s) { return smem + s * Shape::kStage; };
  auto b_hi = [&](int s) { return smem + s * Shape::kStage + Shape::kTileA; };
  auto b_lo = [&](int s) { return smem + s * Shape::kStage + Shape::kTileA + kTileB; };

  if (threadIdx.x == 0) {
    abort_word = 0;
    for (int s = 0; s < kStages; ++s) {
      sm100::mbar_init(&full_bar[s], 1);
      sm100::mbar_init(&empty_bar[s], 1);
    }
    // a block is split by the four warps (one per lane quarter) of one half
    for (int t = 0; t < kAStages; ++t) sm100::mbar_init(&a_full[t], kWorkWarps / 2);
    sm100::mbar_init(&tmem_full, 1);
    sm100::mbar_init(&tmem_empty, kWorkWarps);
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
  const uint32_t tmem_a = tmem_base + kAccCols;  // A ring, lane 0
  // Nothing above touched global memory: under programmatic dependent
  // launch the set-up overlaps the B split kernel's tail.
  grid_dependency_wait();
  grid_dependents_launch();

  if (warp == 0) {
    if (sm100::elect_lane0()) {
      int issued = 0;
      for (int kb = 0; kb < num_kb; ++kb) {
        const int s = kb % kStages;
        if (kb >= kStages &&
            !sm100::mbar_wait(&empty_bar[s], ((kb / kStages) & 1) ^ 1, args.err, sm100::kSiteProducerEmpty, abort))
          break;
        sm100::mbar_arrive_expect_tx(&full_bar[s], Shape::kStage);
        const int kx = kb * BK;
        if constexpr (G == 1) {
          sm100::tma_load_2d(a_raw(s), &map_a, &full_bar[s], kx, (int)m0);
        } else {
#pragma unroll
          for (int j = 0; j < G; ++j) {
            // row offset j of every group: x rounded down to 16 bytes
            const int x = (int)(((int64_t)j * args.lda) & ~int64_t(3)) + kx;
            sm100::tma_load_2d(a_raw(s) + j * Shape::kBoxA, &map_a, &full_bar[s], x, (int)(m0 / G));
          }
        }
        sm100::tma_load_2d(b_hi(s), &map_bhi, &full_bar[s], kx, (int)n0);
        sm100::tma_load_2d(b_lo(s), &map_blo, &full_bar[s], kx, (int)n0);
        issued = kb + 1;
      }
      // Every issued load must land before the CTA may exit (budget only).
      int never = 0;
      for (int kb = issued > kStages ? issued - kStages : 0; kb < issued; ++kb)
        sm100::mbar_wait(&full_bar[kb % kStages], (kb / kStages) & 1, args.err, sm100::kSiteDrain, &never);
    }
  } else if (warp == 1) {
    constexpr uint32_t idesc = sm100::idesc_tf32(BM, BN);
    for (int kb = 0; kb < num_kb; ++kb) {
      const int chunk = kb / cb;
      const bool first = (kb % cb) == 0;
      const bool last = ((kb + 1) % cb) == 0 || kb + 1 == num_kb;
      // one accumulator: chunk c + 1 starts once chunk c has been folded
      if (first && chunk >= 1 &&
          !sm100::mbar_wait_warp(&tmem_empty, (chunk - 1) & 1, args.err, sm100::kSiteMmaFull, abort))
        break;
      // a_full is raised by split warps that saw full_bar complete, so it
      // also orders the stage's B loads before these MMAs.
      const int s = kb % kStages;
      const int t = kb % kAStages;
      if (!sm100::mbar_wait_warp(&a_full[t], (kb / kAStages) & 1, args.err, sm100::kSiteMmaFull, abort)) break;
      sm100::tc_fence_after();
      const uint32_t ahi = tmem_a + (uint32_t)(t * 2 * BK), alo = ahi + BK;
      const uint32_t bhi = sm100::smem_addr(b_hi(s)), blo = sm100::smem_addr(b_lo(s));
#pragma unroll
      for (int k = 0; k < BK / 8; ++k) {
        const uint64_t dbh = sm100::desc_kmajor<64>(bhi + k * 32);
        const uint64_t dbl = sm100::desc_kmajor<64>(blo + k * 32);
        sm100::mma_tf32_ts(tmem_base, alo + 8 * k, dbh, idesc, (first && k == 0) ? 0u : 1u);
        sm100::mma_tf32_ts(tmem_base, ahi + 8 * k, dbl, idesc, 1u);
        sm100::mma_tf32_ts(tmem_base, ahi + 8 * k, dbh, idesc, 1u);
      }
      sm100::mma_commit(&empty_bar[s]);
      if (last) sm100::mma_commit(&tmem_full);
    }
    // Every MMA issued must finish before TMEM is released.
    sm100::mma_commit(&drain_bar);
    int never = 0;
    sm100::mbar_wait(&drain_bar, 0, args.err, sm100::kSiteDrain, &never);
  } else {
    // Work warps 2..9: TMEM lane quarter w % 4 (A rows and accumulator rows
    // 32 q .. 32 q + 31), column half (w - 2) / 4.  The half is also the
    // split group: it splits the K blocks kb with kb % 2 == half.
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row = quarter * 32 + lane;
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    float acc[kCPT];
#pragma unroll
    for (int j = 0; j < kCPT; ++j) acc[j] = 0.0f;
    if (TMA_C && args.bias) {
      for (int i = threadIdx.x - 64; i < BN; i += 32 * kWorkWarps)
        bias_tile[i] = n0 + i < args.n ? __ldg(args.bias + n0 + i) : 0.0f;
      sm100::named_barrier(2, 32 * kWorkWarps);
    }
    // Where this thread's 16 raw values sit in a staged A tile.  G = 1: the
    // 64-byte-swizzled row (16-byte chunk c at c ^ ((row >> 1) & 3)).  G > 1:
    // row G g + j in the box of offset j, group g, at o_j floats.
    const int64_t grow = m0 + row;
    const bool direct = grow >= args.m_grouped && grow < args.m;  // loaded from global memory
    uint32_t a_off;
    if constexpr (G == 1) {
      a_off = (uint32_t)(row * 64);
    } else {
      const int j = row % G;
      const int oj = (int)(((int64_t)j * args.lda) & 3);
      a_off = (uint32_t)(j * Shape::kBoxA + (row / G) * (kBoxW * 4) + oj * 4);
    }

    // Fold the finished chunk into the FP32 registers (round-to-nearest adds)
    // and hand the accumulator back to the MMA issuer.
    auto fold = [&](int chunk) -> bool {
      if (!sm100::mbar_wait(&tmem_full, chunk & 1, args.err, sm100::kSiteEpilogueAccum, abort,
                            3 * sm100::kWaitCycles))
        return false;
      sm100::tc_fence_after();
      const uint32_t taddr = tmem_base + lane_base + (uint32_t)(half * kCPT);
#pragma unroll
      for (int j = 0; j < kCPT; j += 16) {
        uint32_t r[16];
        sm100::tmem_ld_32x32b_x16(taddr + j, r);
        sm100::tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 16; ++i) acc[j + i] = __fadd_rn(acc[j + i], __uint_as_float(r[i]));
      }
      sm100::tc_fence_before();
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(&tmem_empty);
      return true;
    };

    bool ok = true;
    int folded = 0;
    for (int kb = half; kb < num_kb && ok; kb += 2) {
      const int s = kb % kStages;
      const int t = kb % kAStages;
      if (kb >= kAStages) {
        // TMEM A stage t is free once the MMAs of block kb - kAStages are
        // done.  Those MMAs need every chunk before theirs folded, by every
        // work warp: fold them first (the MMA issuer is waiting for that).
        const int prev = kb - kAStages;
        while (folded < prev / cb) {
          if (!fold(folded)) {
            ok = false;
            break;
          }
          ++folded;
        }
        if (!ok) break;
        // Waited before the data stage: once block prev's MMAs are done, the
        // load of block kb - kStages into stage s (kStages >= kAStages) has
        // been consumed, so full_bar's parity below is unambiguous.
        if (!sm100::mbar_wait(&empty_bar[prev % kStages], (prev / kStages) & 1, args.err, sm100::kSiteConvert,
                              abort)) {
          ok = false;
          break;
        }
      }
      if (!sm100::mbar_wait(&full_bar[s], (kb / kStages) & 1, args.err, sm100::kSiteConvert, abort)) {
        ok = false;
        break;
      }
      sm100::tc_fence_after();
      const int kx = kb * BK;
      const uint32_t src = sm100::smem_addr(a_raw(s)) + a_off;
      const uint32_t dst = tmem_a + lane_base + (uint32_t)(t * 2 * BK);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float4 v;
        if (G > 1 && direct) {
          const float *arow = args.a + (m0 + row) * args.lda;
          float e[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int64_t col = kx + 4 * q + u;
            e[u] = col < args.k ? __ldg(arow + col) : 0.0f;
          }
          v = make_float4(e[0], e[1], e[2], e[3]);
        } else if constexpr (G == 1) {
          // the map's K extent is the true K: TMA zero-fills past it
          v = sm100::lds128(src + 16u * ((uint32_t)q ^ (uint32_t)((row >> 1) & 3)));
        } else {
          float e[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            float x;
            asm volatile("ld.shared.f32 %0, [%1];" : "=f"(x) : "r"(src + (uint32_t)(16 * q + 4 * u)) : "memory");
            // past K: the next row's values or TMA's zero fill
            e[u] = kx + 4 * q + u < args.k ? x : 0.0f;
          }
          v = make_float4(e[0], e[1], e[2], e[3]);
        }
        float4 h, l;
        split_tf32x4(v, h, l);
        sm100::tmem_st_32x32b_x4(dst + 4 * q, __float_as_uint(h.x), __float_as_uint(h.y), __float_as_uint(h.z),
                                 __float_as_uint(h.w));
        sm100::tmem_st_32x32b_x4(dst + BK + 4 * q, __float_as_uint(l.x), __float_as_uint(l.y),
                                 __float_as_uint(l.z), __float_as_uint(l.w));
      }
      sm100::tmem_st_wait();
      sm100::tc_fence_before();
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(&a_full[t]);
    }
    while (ok && folded < num_chunks) {
      ok = fold(folded);
      ++folded;
    }

    const int64_t col0 = n0 + half * kCPT;
    if constexpr (TMA_C) {
      // The ring is idle once the last chunk is folded (every MMA, hence
      // every load it consumed, is done): stage C there one 128 x 32 box at a
      // time per column half, the half's first thread storing each box as
      // soon as its four warps have written it.
      const bool has_bias = args.bias != nullptr;
      const bool leader = threadIdx.x == (unsigned)(64 + 128 * half);
#pragma unroll
      for (int b = 0; b < kCPT / 32; ++b) {
        if (ok) {
#pragma unroll
          for (int j = 32 * b; j < 32 * b + 32; j += 4) {
            float v[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              float x = acc[j + q];
              if (has_bias) x = __fadd_rn(x, bias_tile[half * kCPT + j + q]);
              if (args.relu) x = x > 0.0f ? x : 0.0f;
              v[q] = x;
            }
            const int col = half * kCPT + j;
            const int chunk = ((col & 31) >> 2) ^ (row & 7);
            *reinterpret_cast<float4 *>(smem + (col >> 5) * kCBox + row * 128 + chunk * 16) =
                make_float4(v[0], v[1], v[2], v[3]);
          }
        }
        sm100::fence_proxy_async_smem();
        sm100::named_barrier(3 + half * 4 + b, 128);  // this half's four warps
        if (leader && ok) {
          const int box = half * (kCPT / 32) + b;
          sm100::tma_store_2d(&map_c, smem + box * kCBox, (int)n0 + 32 * box, (int)m0);
        }
      }
      if (leader && ok) sm100::tma_store_flush();
    } else if (ok && grow < args.m && col0 < args.n) {
      float *crow = args.c + grow * args.ldc + col0;
      const bool vec = ((args.ldc & 3) == 0) && ((reinterpret_cast<uintptr_t>(args.c) & 15) == 0) &&
                       col0 + kCPT <= args.n;
      const int64_t ncols = args.n - col0;
#pragma unroll
      for (int j = 0; j < kCPT; j += 4) {
        float v[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float x = acc[j + q];
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
    sm100::tmem_dealloc(tmem_base, 512);
  }
}

template <int G, bool TMA_C>
int launch_wide(b2k_ctx *ctx, const float *a, int64_t k, int64_t lda, const b2k::SplitOperands &ops, float *c,
                int64_t m, int64_t n, int64_t ldc, const float *bias, int relu, int chunk_blocks, cudaStream_t s) {
  using Shape = WideShape<G>;
  CUtensorMap map_a, map_bhi, map_blo, map_c{};
  int64_t m_grouped = m;
  int status;
  if constexpr (G == 1) {
    // the map keeps the true K: K blocks past it read as zero
    status = b2k::make_map_2d(ctx, &map_a, a, k, m, lda, BK, BM, CU_TENSOR_MAP_SWIZZLE_64B);
  } else {
    // [m / G groups][G lda floats].  The group holding the last row is
    // covered only when lda == k: otherwise its last row's tail past k need
    // not be part of the caller's buffer, and that group's rows are loaded
    // by their split threads instead.
    const int64_t groups = lda == k ? m / G : (m - 1) / G;
    m_grouped = groups * G;
    if (groups < 1) return b2k::fail(ctx, B2K_EINVAL, "gemm (wide): too few rows for a grouped A map");
    status = b2k::make_map_2d(ctx, &map_a, a, G * lda, groups, G * lda, kBoxW, BM / G, CU_TENSOR_MAP_SWIZZLE_NONE);
  }
  if (status == B2K_OK)
    status = b2k::make_map_2d(ctx, &map_bhi, ops.b_hi, ops.kp, n, ops.kp, BK, BN, CU_TENSOR_MAP_SWIZZLE_64B);
  if (status == B2K_OK)
    status = b2k::make_map_2d(ctx, &map_blo, ops.b_lo, ops.kp, n, ops.kp, BK, BN, CU_TENSOR_MAP_SWIZZLE_64B);
  if (status == B2K_OK && TMA_C)
    status = b2k::make_map_2d(ctx, &map_c, c, n, m, ldc, 32, BM, CU_TENSOR_MAP_SWIZZLE_128B);
  if (status != B2K_OK) return status;
  const int num_kb = (int)(ops.kp / BK);
  WideArgs args{c, bias, a, m, n, k, lda, ldc, m_grouped, num_kb, chunk_blocks, relu, ctx->error_flag};
  auto kernel = gemm_wide_kernel<G, TMA_C>;
  cudaError_t err = b2k::set_max_smem(ctx, (const void *)kernel, Shape::kSmem);
  if (err != cudaSuccess) return b2k::cuda_fail(ctx, err, "gemm (wide): set smem");
  if ((n + BN - 1) / BN > 65535) return b2k::fail(ctx, B2K_EINVAL, "gemm: N exceeds %d", 65535 * BN);
  dim3 grid((unsigned)((m + BM - 1) / BM), (unsigned)((n + BN - 1) / BN), 1);
  err = b2k::launch_kernel(b2k::pdl_enabled(), kernel, grid, dim3(kThreads), Shape::kSmem, s, map_a, map_bhi, map_blo,
                           map_c, args);
  if (err != cudaSuccess) return b2k::cuda_fail(ctx, err, "gemm (wide) launch");
  return b2k::check_launch(ctx, "gemm (wide) launch");
}

// K blocks per accumulation chunk: the fewest chunks of at most
// g_wide_chunk_k / BK blocks, evened out.
int g_wide_chunk_k = 256;

int wide_chunk_blocks(int num_kb) {
  int limit = g_wide_chunk_k / BK;
  limit = limit < 1 ? 1 : (limit > kMaxChunkBlocks ? kMaxChunkBlocks : limit);
  const int chunks = (num_kb + limit - 1) / limit;
  return (num_kb + chunks - 1) / chunks;
}

}  // namespace

// Accumulation chunk of the wide kernel, in K elements (a multiple of 16 from
// 16 to 384; default 256, the chunk of the other tensor-core kernels).
extern "C" int b2k_gemm_set_wide_chunk(int k) {
  if (k < BK || k > kMaxChunkBlocks * BK || k % BK != 0) return B2K_EINVAL;
  g_wide_chunk_k = k;
  return B2K_OK;
}

namespace b2k {

// Rows grouped per TMA box row for a row stride of `lda` floats: the fewest
// consecutive rows whose stride is a multiple of 16 bytes.
int wide_row_group(int64_t lda) { return lda % 4 == 0 ? 1 : (lda % 2 == 0 ? 2 : 4); }

int gemm_wide(b2k_ctx *ctx, const float *a, int64_t k, int64_t lda, const SplitOperands &ops, float *c, int64_t m,
              int64_t n, int64_t ldc, const float *bias, int relu, cudaStream_t s) {
  PhaseTimer timer(ctx, B2K_PHASE_MMA, s);
  const int cb = wide_chunk_blocks((int)(ops.kp / BK));
  const bool tma_c = aligned16(c) && ldc % 4 == 0;
  switch (wide_row_group(lda)) {
    case 1:
      return tma_c ? launch_wide<1, true>(ctx, a, k, lda, ops, c, m, n, ldc, bias, relu, cb, s)
                   : launch_wide<1, false>(ctx, a, k, lda, ops, c, m, n, ldc, bias, relu, cb, s);
    case 2:
      return tma_c ? launch_wide<2, true>(ctx, a, k, lda, ops, c, m, n, ldc, bias, relu, cb, s)
                   : launch_wide<2, false>(ctx, a, k, lda, ops, c, m, n, ldc, bias, relu, cb, s);
    default:
      return tma_c ? launch_wide<4, true>(ctx, a, k, lda, ops, c, m, n, ldc, bias, relu, cb, s)
                   : launch_wide<4, false>(ctx, a, k, lda, ops, c, m, n, ldc, bias, relu, cb, s);
  }
}

}  // namespace b2k
