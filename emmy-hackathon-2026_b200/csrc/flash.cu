// Fused attention, O = softmax(Q K^T / scale) V, both contractions 3xTF32 on
// tcgen05, one CTA per (head, 128 query rows), streaming 128-key blocks.
//
// A tf32 tcgen05.mma with M = 128 reads its A operand (4 KB) from shared
// memory every time, so narrow MMAs are bound by shared-memory bandwidth
// (measured on B200: N = 32 runs at 35 % of the tensor rate, N = 64 at 67 %,
// N >= 128 at 100 %); every MMA here is N = 128: S_j = Q K_j^T over 128 keys
// and O_j = P_j V_j over 128 output columns.  Ring chunks are 32 wide (12
// MMAs each): 16-wide chunks in a 6-deep ring measured slower, the issuer's
// per-chunk wait and commit then costing about as much as the chunk's MMAs.
//
// The reference hoists one head's score rows into shared memory and runs the
// softmax and the P.V fold in SIMT FP32 (compile.py:7009-7966, selective exp
// 2953-2965).  Here nothing but Q, K, V and O touches HBM:
//
//   warp 0      TMA: Q once (128 x Dp, four 128-byte-swizzled column
//               blocks, resident; raw when d % 32 == 0 -- the softmax warps
//               then split it into Q_hi/Q_lo in place before the first S
//               MMA -- else the pre-split hi/lo copies), then through a 3-stage ring
//               the chunks K_j[:, 32c..] (128 keys x 32 dims) and
//               V_j^T[:, 32c..] (128 dims x 32 keys), hi and lo, in the MMA
//               issuer's order: K_0, then K_{j+1}, V_j for each j
//   warp 1      TMEM allocator and MMA issuer (warp-wide, elect.sync):
//               S_{j+1} = Q K_{j+1}^T into score buffer (j+1) % 2 while the
//               softmax works on S_j, then O_j = P_j V_j (P_j read from TMEM)
//               into the O buffer once the softmax has released P_j
//   warps 2..9  softmax, two threads per query row (warpgroup 0 takes score
//               columns 0-63 and output columns 0-63 of the row, warpgroup
//               1 the rest): S_j from TMEM, online max / sum with the
//               selective exponential (partial row max and sum exchanged
//               through shared memory), then the finished O_{j-1} folded
//               into the FP32 row accumulator O = O * alpha + O_{j-1} in
//               registers, then P_j's TF32 halves into TMEM (hi over S_j, lo
//               in its own columns: the A operand of O_j); at the end the
//               normalised O tile, staged in Q's buffer and TMA-stored box
//               by box
//
// Each key block's products accumulate in a fresh TMEM buffer, so the
// in-instruction accumulation error stays that of 48 (S) / 48 (O) MMAs.
// All mbarrier waits are bounded (sm100.cuh).
#include <cudaTypedefs.h>

#include <math.h>

#include "common.cuh"
#include "sm100.cuh"
#include "tmap.cuh"

namespace {

constexpr int BM = 128;        // query rows per CTA
constexpr int BN = 128;        // keys per block (every MMA is N = 128: full tensor rate)
constexpr int DMAX = 128;      // head dims supported (padded to 32)
constexpr int kStages = 3;     // ring of K / V chunks (single CTA)
constexpr int kThreads = 320;  // producer, MMA, 8 softmax warps (two per TMEM lane quarter)
constexpr int kQSplitBatch = 8;  // Q chunks a softmax thread loads before splitting them

constexpr int kSub = 128 * 32 * 4;          // one [128 rows x 32 fp32] swizzled block (16 KB)
constexpr int kQBytes = (DMAX / 32) * kSub; // 64 KB per half
// Q (both halves, resident) + a ring of stages, each one K chunk [128 keys x
// 32 dims] or one V^T chunk [128 dims x 32 keys], hi and lo: 128 + 96 KB.
// The row-exchange arrays and barriers are static, so the dynamic buffer is
// declared 1024-byte aligned (checked at run time) instead of carrying slack.
constexpr int kSmem = 2 * kQBytes + kStages * 2 * kSub;

// TMEM columns: two score buffers [0, 128) and [128, 256) -- S_j, then P_j's
// hi half, in buffer j % 2 -- P_j's lo half [256, 384), O_j [384, 512).  With
// two score buffers the tensor core computes S_{j+1} while the softmax warps
// turn S_j into P_j.
constexpr uint32_t kColPlo = 256, kColO = 384;
__host__ __device__ constexpr uint32_t s_col(int j) { return (uint32_t)((j & 1) * 128); }

constexpr int kChunkBytes = kSub;  // one half (hi or lo) of a ring stage

struct FlashArgs {
  int tma_o;  // O written by TMA stores from shared memory (16-byte aligned, dv % 4 == 0)
  int q_raw;  // map_qhi is raw FP32 Q: the CTA splits its Q tile in shared memory
  int q_prefetch;  // > 0: prefetch into L2 the Q tile of the CTA this many launch slots later
  float *o;
  int64_t s_q, s_kv, dv;
  int dp;          // padded head dim (multiple of 32, <= 128)
  int n_pv;        // O MMA width: round_up(dv, 16)
  float inv_scale; // 1 / scale when scale_ptr is null
  const float *scale_ptr;
  unsigned *err;
};

__global__ void __launch_bounds__(kThreads, 1)
    flash_tf32x3_kernel(const __grid_constant__ CUtensorMap map_qhi, const __grid_constant__ CUtensorMap map_qlo,
                        const __grid_constant__ CUtensorMap map_khi, const __grid_constant__ CUtensorMap map_klo,
                        const __grid_constant__ CUtensorMap map_vhi, const __grid_constant__ CUtensorMap map_vlo,
                        const __grid_constant__ CUtensorMap map_o, const FlashArgs args) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t q_full, q_ready, p_full, pv_done, drain;
  __shared__ __align__(8) uint64_t ring_full[kStages], ring_empty[kStages], s_full[2];
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_word;
  __shared__ float part_max[2][BM], part_sum[2][BM];

  uint8_t *q_hi = smem_raw, *q_lo = q_hi + kQBytes;
  uint8_t *ring = q_lo + kQBytes;  // stage i: hi at ring + 2i*chunk, lo at ring + (2i+1)*chunk
  auto st_hi = [&](int i) { return ring + (2 * i) * kChunkBytes; };
  auto st_lo = [&](int i) { return ring + (2 * i + 1) * kChunkBytes; };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int head = blockIdx.y;
  const int64_t m0 = (int64_t)blockIdx.x * BM;
  const int nblocks = (int)((args.s_kv + BN - 1) / BN);
  const int dblocks = args.dp / 32;      // K chunks per block
  constexpr int kVChunks = BN / 32;      // V chunks per block
  volatile int *abort = &abort_word;

  if (threadIdx.x == 0) {
    // swizzled tiles need 1024-byte alignment: refuse to run (error word, no
    // work) rather than compute garbage
    abort_word = (sm100::smem_addr(smem_raw) & 1023u) ? 1 : 0;
    if (abort_word) atomicOr(args.err, sm100::kSiteAttention);
    sm100::mbar_init(&q_full, 1);
    sm100::mbar_init(&q_ready, 8);             // one arrival per softmax warp (raw Q split)
    sm100::mbar_init(&p_full, 8);   // one arrival per softmax warp
    sm100::mbar_init(&pv_done, 1);
    sm100::mbar_init(&drain, 1);
    for (int i = 0; i < kStages; ++i) {
      sm100::mbar_init(&ring_full[i], 1);
      sm100::mbar_init(&ring_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) sm100::mbar_init(&s_full[i], 1);
    sm100::fence_barrier_init();
  }
  if (warp == 1) sm100::tmem_alloc(&tmem_slot, 512);
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = tmem_slot;
  // Nothing above touched global memory: under programmatic dependent
  // launch the set-up overlaps the V split kernel's tail.
  grid_dependency_wait();
  grid_dependents_launch();

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer: Q once, then K_j chunks, V_j chunks, K_{j+1} ...
      if (args.q_raw) {
        // raw Q into the hi buffer; the softmax warps split it in place
        sm100::mbar_arrive_expect_tx(&q_full, dblocks * kSub);
        for (int c = 0; c < dblocks; ++c) sm100::tma_load_3d(q_hi + c * kSub, &map_qhi, &q_full, c * 32, (int)m0, head);
      } else {
        sm100::mbar_arrive_expect_tx(&q_full, 2 * dblocks * kSub);
        for (int c = 0; c < dblocks; ++c) {
          sm100::tma_load_3d(q_hi + c * kSub, &map_qhi, &q_full, c * 32, (int)m0, head);
          sm100::tma_load_3d(q_lo + c * kSub, &map_qlo, &q_full, c * 32, (int)m0, head);
        }
      }
      if (args.q_prefetch > 0) {
        // One CTA per SM: the CTA launched q_prefetch slots later (about one
        // wave) starts on this SM or another once a CTA of this wave exits.
        // Its Q tile comes from HBM; asking L2 for it now turns that load,
        // most of a CTA's 3.6 us prologue, into an L2 hit.
        const int64_t next = (int64_t)blockIdx.y * gridDim.x + blockIdx.x + args.q_prefetch;
        if (next < (int64_t)gridDim.x * gridDim.y) {
          const int nh = (int)(next / gridDim.x), nm = (int)(next % gridDim.x) * BM;
          for (int c = 0; c < dblocks; ++c) {
            sm100::tma_prefetch_l2_3d(&map_qhi, c * 32, nm, nh);
            if (!args.q_raw) sm100::tma_prefetch_l2_3d(&map_qlo, c * 32, nm, nh);
          }
        }
      }
      // Ring order = MMA order: K_0, then for each block j, K_{j+1} and V_j.
      int n = 0;  // chunks issued through the ring
      bool ok = true;
      auto load_chunk = [&](bool is_k, int j, int c) {
        const int i = n % kStages;
        if (n >= kStages &&
            !sm100::mbar_wait(&ring_empty[i], ((n / kStages) - 1) & 1, args.err, sm100::kSiteAttention, abort))
          return false;
        sm100::mbar_arrive_expect_tx(&ring_full[i], 2 * kChunkBytes);
        if (is_k) {  // K chunk: keys j*BN.., dims c*32..
          sm100::tma_load_3d(st_hi(i), &map_khi, &ring_full[i], c * 32, j * BN, head);
          sm100::tma_load_3d(st_lo(i), &map_klo, &ring_full[i], c * 32, j * BN, head);
        } else {     // V^T chunk: all dims, keys j*BN + 32c..
          const int x = j * BN + 32 * c;
          sm100::tma_load_3d(st_hi(i), &map_vhi, &ring_full[i], x, 0, head);
          sm100::tma_load_3d(st_lo(i), &map_vlo, &ring_full[i], x, 0, head);
        }
        ++n;
        return true;
      };
      for (int c = 0; ok && c < dblocks; ++c) ok = load_chunk(true, 0, c);
      for (int j = 0; ok && j < nblocks; ++j) {
        for (int c = 0; ok && j + 1 < nblocks && c < dblocks; ++c) ok = load_chunk(true, j + 1, c);
        for (int c = 0; ok && c < kVChunks; ++c) ok = load_chunk(false, j, c);
      }
      int never = 0;  // drain loads in flight (budget only)
      sm100::mbar_wait(&q_full, 0, args.err, sm100::kSiteDrain, &never);
      for (int m = n > kStages ? n - kStages : 0; m < n; ++m)
        sm100::mbar_wait(&ring_full[m % kStages], (m / kStages) & 1, args.err, sm100::kSiteDrain, &never);
    }
  } else if (warp == 1) {
    {
      // ---------------- MMA issuer: S_0, then for each block j, S_{j+1}
      // (into the other score buffer, overlapping softmax_j) and O_j = P_j V_j.
      // S_{j+1} reuses the buffer P_{j-1} occupied; O_{j-1}'s MMAs, which read
      // it, were issued earlier and tcgen05 MMAs of one issuer run in order.
      const uint32_t id_s = sm100::idesc_tf32(BM, BN);
      const uint32_t id_o = sm100::idesc_tf32(BM, args.n_pv);
      const uint32_t qh = sm100::smem_addr(q_hi), ql = sm100::smem_addr(q_lo);
      auto mma_ss = [&](uint32_t d, uint64_t a, uint64_t b, uint32_t id, uint32_t acc) {
        sm100::mma_tf32(d, a, b, id, acc);
      };
      auto mma_ts = [&](uint32_t d, uint32_t a, uint64_t b, uint32_t id, uint32_t acc) {
        sm100::mma_tf32_ts(d, a, b, id, acc);
      };
      auto commit = [&](uint64_t *bar) { sm100::mma_commit(bar); };
      auto stage_ready = [&](int i, int n_) {
        return sm100::mbar_wait_warp(&ring_full[i], (n_ / kStages) & 1, args.err, sm100::kSiteAttention, abort);
      };
      bool ok = args.q_raw ? sm100::mbar_wait_warp(&q_ready, 0, args.err, sm100::kSiteAttention, abort)
                           : sm100::mbar_wait_warp(&q_full, 0, args.err, sm100::kSiteAttention, abort);
      int n = 0;  // ring chunks consumed
      auto issue_s = [&](int j) {
        for (int c = 0; ok && c < dblocks; ++c, ++n) {
          const int i = n % kStages;
          if (!(ok = stage_ready(i, n))) break;
          sm100::tc_fence_after();
          const uint32_t kh = sm100::smem_addr(st_hi(i)), kl = sm100::smem_addr(st_lo(i));
          for (int k = 0; k < 4; ++k) {
            const uint32_t qa = (uint32_t)(c * kSub + k * 32), ka = (uint32_t)(k * 32);
            const uint64_t dqh = sm100::desc_kmajor<128>(qh + qa), dql = sm100::desc_kmajor<128>(ql + qa);
            const uint64_t dkh = sm100::desc_kmajor<128>(kh + ka), dkl = sm100::desc_kmajor<128>(kl + ka);
            mma_ss(tmem + s_col(j), dql, dkh, id_s, (c == 0 && k == 0) ? 0u : 1u);
            mma_ss(tmem + s_col(j), dqh, dkl, id_s, 1u);
            mma_ss(tmem + s_col(j), dqh, dkh, id_s, 1u);
          }
          commit(&ring_empty[i]);
        }
        if (ok) commit(&s_full[j & 1]);
      };
      auto issue_pv = [&](int j) {
        // once the softmax has written P_j into TMEM and folded O_{j-1}
        if (!(ok = sm100::mbar_wait_warp(&p_full, j & 1, args.err, sm100::kSiteAttention, abort))) return;
        sm100::tc_fence_after();
        for (int c = 0; ok && c < kVChunks; ++c, ++n) {
          const int i = n % kStages;
          if (!(ok = stage_ready(i, n))) break;
          sm100::tc_fence_after();
          const uint32_t vh = sm100::smem_addr(st_hi(i)), vl = sm100::smem_addr(st_lo(i));
          for (int k = 0; k < 4; ++k) {
            const uint32_t pcol = (uint32_t)(c * 32 + k * 8);
            const uint64_t dvh = sm100::desc_kmajor<128>(vh + k * 32), dvl = sm100::desc_kmajor<128>(vl + k * 32);
            mma_ts(tmem + kColO, tmem + kColPlo + pcol, dvh, id_o, (c == 0 && k == 0) ? 0u : 1u);
            mma_ts(tmem + kColO, tmem + s_col(j) + pcol, dvl, id_o, 1u);
            mma_ts(tmem + kColO, tmem + s_col(j) + pcol, dvh, id_o, 1u);
          }
          commit(&ring_empty[i]);
        }
        if (ok) commit(&pv_done);
      };
      if (ok) issue_s(0);
      for (int j = 0; ok && j < nblocks; ++j) {
        if (j + 1 < nblocks) issue_s(j + 1);
        if (ok) issue_pv(j);
      }
      sm100::mma_commit(&drain);
      int never = 0;
      sm100::mbar_wait(&drain, 0, args.err, sm100::kSiteDrain, &never);
    }
  } else {
    // ---------------- softmax + O accumulation: two threads per query row
    const int quarter = warp & 3;
    const int wg = (warp - 2) >> 2;        // column half of the row
    const int r = quarter * 32 + lane;     // row within the tile == TMEM lane
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    const float inv_scale = args.scale_ptr ? __frcp_rn(__ldg(args.scale_ptr)) : args.inv_scale;
    constexpr int SC = BN / 2;   // score columns per thread
    constexpr int OC = 64;       // output columns per thread
    const int sc0 = wg * SC, oc0 = wg * OC;
    float o_acc[OC];
#pragma unroll
    for (int i = 0; i < OC; ++i) o_acc[i] = 0.0f;
    float m_run = -INFINITY, l_run = 0.0f;
    float alpha_prev = 1.0f;  // exp(m_{j-2} - m_{j-1}): the rescale O_{j-1} is folded with
    bool ok = true;
    // Fold O_{j-1} = P_{j-1} V_{j-1} (TMEM) into the register accumulator once
    // its MMAs are done; O's TMEM buffer is then free for O_j.
    auto fold_o = [&](int jm1) {
      ok = ok && sm100::mbar_wait(&pv_done, jm1 & 1, args.err, sm100::kSiteAttention, abort,
                                          3 * sm100::kWaitCycles);
      if (!ok) return;
      sm100::tc_fence_after();
      if (oc0 < args.n_pv) {  // warp-uniform
        uint32_t o0[32], o1[32];
        const uint32_t ta = tmem + lane_base + kColO + (uint32_t)oc0;
        sm100::tmem_ld_32x32b_x32(ta, o0);
        sm100::tmem_ld_32x32b_x32(ta + 32, o1);
        sm100::tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          o_acc[i] = __fadd_rn(__fmul_rn(o_acc[i], alpha_prev), __uint_as_float(o0[i]));
          o_acc[32 + i] = __fadd_rn(__fmul_rn(o_acc[32 + i], alpha_prev), __uint_as_float(o1[i]));
        }
      }
    };
    if (args.q_raw) {
      // Split the raw Q tile in place: Q_hi over the raw values, Q_lo in its
      // own buffer, the same 128-byte-swizzled [128 rows x 32] boxes the
      // MMAs read.  Warpgroup wg takes boxes wg, wg + 2, ...; each thread its
      // row's eight 16-byte chunks of a box (chunk c of row r sits at
      // c ^ (r & 7): conflict-free across the warp).
      ok = sm100::mbar_wait(&q_full, 0, args.err, sm100::kSiteAttention, abort);
      if (ok) {
        const uint32_t qh = sm100::smem_addr(q_hi), ql = sm100::smem_addr(q_lo);
        for (int c = wg; c < dblocks; c += 2) {
          // All eight chunks of a row are loaded before any is split and
          // stored, so the loads are in flight together; one at a time, each
          // behind the previous chunk's stores, the split took 2 us of a
          // CTA's prologue and the whole attention step 0.5 % longer.
#pragma unroll
          for (int g = 0; g < 8; g += kQSplitBatch) {
            float4 v[kQSplitBatch];
#pragma unroll
            for (int u = 0; u < kQSplitBatch; ++u)
              v[u] = sm100::lds128(qh + (uint32_t)(c * kSub + r * 128 + (((g + u) ^ (r & 7)) << 4)));
#pragma unroll
            for (int u = 0; u < kQSplitBatch; ++u) {
              const uint32_t off = (uint32_t)(c * kSub + r * 128 + (((g + u) ^ (r & 7)) << 4));
              float4 hv, lv;
              split_tf32x4(v[u], hv, lv);
              sm100::sts128_relaxed(qh + off, hv);
              sm100::sts128_relaxed(ql + off, lv);
            }
          }
        }
        sm100::fence_proxy_async_smem();  // the MMAs read Q through the async proxy
      }
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(&q_ready);
    }
    // Every thread runs every iteration and reaches both named barriers even
    // after a failed wait (ok == false), so the two warpgroups never wait on
    // each other forever; failed waits only skip work.
    for (int j = 0; j < nblocks; ++j) {
      ok = ok && sm100::mbar_wait(&s_full[j & 1], (j >> 1) & 1, args.err, sm100::kSiteAttention, abort);
      sm100::tc_fence_after();
      uint32_t sr[SC];
      {
        uint32_t (&a)[32] = *reinterpret_cast<uint32_t(*)[32]>(&sr[0]);
        uint32_t (&b)[32] = *reinterpret_cast<uint32_t(*)[32]>(&sr[32]);
        sm100::tmem_ld_32x32b_x32(tmem + lane_base + s_col(j) + (uint32_t)sc0, a);
        sm100::tmem_ld_32x32b_x32(tmem + lane_base + s_col(j) + (uint32_t)sc0 + 32, b);
        sm100::tmem_ld_wait();
      }
      float mx = -INFINITY;
      const int64_t c0 = (int64_t)j * BN + sc0;
#pragma unroll
      for (int i = 0; i < SC; ++i) {
        const float x = (c0 + i < args.s_kv) ? __fmul_rn(__uint_as_float(sr[i]), inv_scale) : -INFINITY;
        sr[i] = __float_as_uint(x);
        mx = fmaxf(mx, x);
      }
      part_max[wg][r] = mx;
      sm100::named_barrier(1, 256);
      mx = fmaxf(fmaxf(mx, part_max[wg ^ 1][r]), m_run);
      const float alpha = b2k_exp(__fsub_rn(m_run, mx));
      float sum = 0.0f;
      uint32_t pl[SC];
#pragma unroll
      for (int i = 0; i < SC; ++i) {
        const float v = b2k_exp(__fsub_rn(__uint_as_float(sr[i]), mx));
        sum += v;
        // probabilities are finite and in [0, 1]: the split needs no range guards
        const uint32_t hv = (__float_as_uint(v) + 0x1000u) & 0xFFFFE000u;
        sr[i] = hv;
        pl[i] = (__float_as_uint(__fsub_rn(v, __uint_as_float(hv))) + 0x1000u) & 0xFFFFE000u;
      }
      part_sum[wg][r] = sum;
      // O_{j-1} must leave TMEM (and P_{j-1}'s lo half be consumed) before
      // P_j's lo half and, later, O_j are written.
      if (j >= 1) fold_o(j - 1);
      if (ok) {
        // P_j's halves into TMEM: hi over S_j, lo in its own columns (the A operand of O_j)
        uint32_t (&h0)[32] = *reinterpret_cast<uint32_t(*)[32]>(&sr[0]);
        uint32_t (&h1)[32] = *reinterpret_cast<uint32_t(*)[32]>(&sr[32]);
        uint32_t (&l0)[32] = *reinterpret_cast<uint32_t(*)[32]>(&pl[0]);
        uint32_t (&l1)[32] = *reinterpret_cast<uint32_t(*)[32]>(&pl[32]);
        sm100::tmem_st_32x32b_x32(tmem + lane_base + s_col(j) + (uint32_t)sc0, h0);
        sm100::tmem_st_32x32b_x32(tmem + lane_base + s_col(j) + (uint32_t)sc0 + 32, h1);
        sm100::tmem_st_32x32b_x32(tmem + lane_base + kColPlo + (uint32_t)sc0, l0);
        sm100::tmem_st_32x32b_x32(tmem + lane_base + kColPlo + (uint32_t)sc0 + 32, l1);
        sm100::tmem_st_wait();
      }
      sm100::tc_fence_before();
      __syncwarp();
      if (lane == 0 && ok) sm100::mbar_arrive(&p_full);
      sm100::named_barrier(2, 256);
      l_run = __fadd_rn(__fmul_rn(l_run, alpha), __fadd_rn(part_sum[0][r], part_sum[1][r]));
      m_run = mx;
      alpha_prev = alpha;
    }
    if (nblocks > 0) fold_o(nblocks - 1);
    const int64_t row = m0 + r;
    const float inv_l = __frcp_rn(l_run);
    if (args.tma_o) {
      // Q's buffer is idle after the last block: stage the normalised O tile
      // there as 128-byte-swizzled boxes of 128 rows x 32 columns and write it
      // with TMA stores (coalesced, rows past s_q clipped).  Each warpgroup
      // stages its two boxes one at a time; its first thread stores a box as
      // soon as the group's four warps have written it.
      const bool leader = threadIdx.x == (unsigned)(64 + 128 * wg);
#pragma unroll
      for (int b = 0; b < OC / 32; ++b) {
        const int box = oc0 / 32 + b;
        if (ok) {
#pragma unroll
          for (int i = 32 * b; i < 32 * b + 32; i += 4) {
            const int col = oc0 + i;
            const uint32_t chunk = (uint32_t)((col & 31) >> 2) ^ (uint32_t)(r & 7);
            sm100::sts128_relaxed(sm100::smem_addr(q_hi + (col >> 5) * kSub + r * 128 + chunk * 16),
                                  make_float4(__fmul_rn(o_acc[i], inv_l), __fmul_rn(o_acc[i + 1], inv_l),
                                              __fmul_rn(o_acc[i + 2], inv_l), __fmul_rn(o_acc[i + 3], inv_l)));
          }
        }
        sm100::fence_proxy_async_smem();
        sm100::named_barrier(4 + 2 * wg + b, 128);  // this warpgroup's four warps
        if (leader && ok && box * 32 < args.dv)
          sm100::tma_store_3d(&map_o, q_hi + box * kSub, 32 * box, (int)m0, head);
      }
      if (leader && ok) sm100::tma_store_flush();
    } else if (ok && row < args.s_q && oc0 < args.dv) {
      float *orow = args.o + ((int64_t)head * args.s_q + row) * args.dv;
      const bool vec = (args.dv % 4 == 0) && ((reinterpret_cast<uintptr_t>(args.o) & 15) == 0);
      if (vec) {
#pragma unroll
        for (int i = 0; i < OC; i += 4)
          if (oc0 + i < args.dv)
            *reinterpret_cast<float4 *>(orow + oc0 + i) =
                make_float4(__fmul_rn(o_acc[i], inv_l), __fmul_rn(o_acc[i + 1], inv_l), __fmul_rn(o_acc[i + 2], inv_l),
                            __fmul_rn(o_acc[i + 3], inv_l));
      } else {
#pragma unroll
        for (int i = 0; i < OC; ++i)
          if (oc0 + i < args.dv) orow[oc0 + i] = __fmul_rn(o_acc[i], inv_l);
      }
    }
  }
  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, 512);
  }
}

// [batch][rows][inner] FP32, box [1][box_rows][32] with the 128-byte swizzle.
int make_map(b2k_ctx *ctx, CUtensorMap *map, const float *base, int64_t inner, int64_t rows, int64_t batch,
             int box_rows) {
  auto encode = b2k::tensor_map_encoder();
  if (!encode) return b2k::fail(ctx, B2K_ECUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[3] = {(cuuint64_t)inner, (cuuint64_t)rows, (cuuint64_t)batch};
  cuuint64_t strides[2] = {(cuuint64_t)inner * 4, (cuuint64_t)(rows * inner * 4)};
  cuuint32_t box[3] = {32, (cuuint32_t)box_rows, 1};
  cuuint32_t elem[3] = {1, 1, 1};
  CUresult res = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float *>(base), dims, strides, box, elem,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (res != CUDA_SUCCESS) return b2k::fail(ctx, B2K_ECUDA, "cuTensorMapEncodeTiled failed (%d)", (int)res);
  return B2K_OK;
}

}  // namespace

namespace b2k {

bool flash_supported(int64_t d, int64_t dv) { return d >= 1 && d <= DMAX && dv >= 1 && dv <= 128; }

size_t flash_workspace_floats(int64_t bh, int64_t s_q, int64_t s_kv, int64_t d, int64_t dv) {
  const int64_t dp = gemm_kpad(d), sp = gemm_kpad(s_kv);
  return (size_t)(2 * bh * s_q * dp + 2 * bh * s_kv * dp + 2 * bh * dv * sp);
}

// Fused path: split Q, K, V into `ws`, then one kernel per (head, 128 rows).
int flash_attention(b2k_ctx *ctx, const float *q, const float *k, const float *v, float *o, int64_t bh, int64_t s_q,
                    int64_t s_kv, int64_t d, int64_t dv, float scale_div, const float *scale_div_ptr, int k_layout,
                    float *ws, cudaStream_t s) {
  const int64_t dp = gemm_kpad(d), sp = gemm_kpad(s_kv);
  float *q_hi = ws, *q_lo = q_hi + bh * s_q * dp;
  float *k_hi = q_lo + bh * s_q * dp, *k_lo = k_hi + bh * s_kv * dp;
  float *v_hi = k_lo + bh * s_kv * dp, *v_lo = v_hi + bh * dv * sp;
  int status;
  const int64_t tiles = (s_q + BM - 1) / BM;
  // A single CTA loads its Q tile once and can split it in shared memory:
  // that needs raw Q TMA-readable with whole 32-column boxes (d % 32 == 0,
  // 16-byte aligned) and saves the pre-pass writing and the kernel reading
  // Q's hi/lo copies.  Otherwise Q is split by the pre-pass like K.
  const bool q_raw = d % 32 == 0 && aligned16(q);
  const RowSplit sq{q, s_q, d, d, s_q * d, bh, q_hi, q_lo};
  const RowSplit sk{k, s_kv, d, d, s_kv * d, bh, k_hi, k_lo};
  if (k_layout == B2K_K_SD) {
    // Q (unless split in the kernel) and K in one launch
    status = q_raw ? split_rows2(ctx, sk, nullptr, dp, s) : split_rows2(ctx, sq, &sk, dp, s);
  } else if ((status = q_raw ? B2K_OK : split_rows2(ctx, sq, nullptr, dp, s)) == B2K_OK) {
    status = split_transpose(ctx, k, d, s_kv, s_kv, d * s_kv, bh, dp, k_hi, k_lo, s);
  }
  if (status != B2K_OK) return status;
  if ((status = split_transpose(ctx, v, s_kv, dv, dv, s_kv * dv, bh, sp, v_hi, v_lo, s)) != B2K_OK) return status;
  CUtensorMap maps[6];
  if ((status = make_map(ctx, &maps[0], q_raw ? q : q_hi, q_raw ? d : dp, s_q, bh, BM)) != B2K_OK) return status;
  if ((status = make_map(ctx, &maps[1], q_lo, dp, s_q, bh, BM)) != B2K_OK) return status;
  if ((status = make_map(ctx, &maps[2], k_hi, dp, s_kv, bh, BN)) != B2K_OK) return status;
  if ((status = make_map(ctx, &maps[3], k_lo, dp, s_kv, bh, BN)) != B2K_OK) return status;
  if ((status = make_map(ctx, &maps[4], v_hi, sp, dv, bh, 128)) != B2K_OK) return status;
  if ((status = make_map(ctx, &maps[5], v_lo, sp, dv, bh, 128)) != B2K_OK) return status;
  // O through TMA stores when it is TMA-writable, else row stores by the threads.
  CUtensorMap map_o{};
  const int tma_o = aligned16(o) && dv % 4 == 0;
  if (tma_o && (status = make_map(ctx, &map_o, o, dv, s_q, bh, BM)) != B2K_OK) return status;
  FlashArgs args{tma_o, (int)q_raw, ctx->sm_count, o, s_q, s_kv, dv, (int)dp, (int)((dv + 15) / 16 * 16),
                 1.0f / scale_div, scale_div_ptr, ctx->error_flag};
  auto kernel = flash_tf32x3_kernel;
  cudaError_t err = set_max_smem(ctx, (const void *)kernel, kSmem);
  if (err != cudaSuccess) return cuda_fail(ctx, err, "flash: set smem");
  PhaseTimer timer(ctx, B2K_PHASE_FLASH, s);
  err = launch_kernel(pdl_enabled(), kernel, dim3((unsigned)tiles, (unsigned)bh), dim3(kThreads), kSmem, s, maps[0],
                      maps[1], maps[2], maps[3], maps[4], maps[5], map_o, args);
  if (err != cudaSuccess) return cuda_fail(ctx, err, "flash: launch");
  return check_launch(ctx, "flash launch");
}

}  // namespace b2k
