// Fused attention, O = softmax(Q K^T / scale) V, both contractions 3xTF32 on
// tcgen05, one CTA per (head, 128 query rows), streaming 32-key blocks.
//
// The reference hoists one head's score rows into shared memory and runs the
// softmax and the P.V fold in SIMT FP32 (compile.py:7009-7966, selective exp
// 2953-2965).  Here nothing but Q, K, V and O touches HBM:
//
//   warp 0      TMA: Q_hi/Q_lo once (128 x Dp, four 128-byte-swizzled
//               column blocks each), then per key block j the K_j tiles
//               (32 keys x Dp) and the V_j^T tiles (Dv x 32 keys)
//   warp 1      TMEM allocator and MMA issuer: S_j = Q K_j^T (three TF32
//               products per 8-wide step) into TMEM buffer j % 2, and
//               O_j = P_j V_j into TMEM buffer j % 2; issue order
//               S_0, S_1, O_0, S_2, O_1, ... so QK^T of the next block
//               overlaps the softmax of this one
//   warps 2..5  softmax, one thread per query row: S_j from TMEM, online max /
//               sum with the selective exponential, P_j's TF32 halves into
//               swizzled shared memory (the A operand of O_j), then the
//               finished O_{j-1} from TMEM folded into the FP32 row
//               accumulator O = O * alpha + O_{j-1} in registers (which also
//               keeps the tensor core's accumulation error per block small)
//
// Each key block's products accumulate in a fresh TMEM buffer, so the
// in-instruction accumulation error stays that of 48 (S) / 12 (O) MMAs.
// All mbarrier waits are bounded (sm100.cuh).
#include <cudaTypedefs.h>

#include <math.h>

#include "common.cuh"
#include "sm100.cuh"

namespace {

constexpr int BM = 128;        // query rows per CTA
constexpr int BN = 32;         // keys per block
constexpr int DMAX = 128;      // head dims supported (padded to 32)
constexpr int kThreads = 192;  // producer, MMA, 4 softmax warps

constexpr int kSub = 128 * 32 * 4;                 // one [128 rows x 32 fp32] swizzled block (16 KB)
constexpr int kQBytes = (DMAX / 32) * kSub;        // 64 KB per half
constexpr int kKBytes = (DMAX / 32) * BN * 128;    // 16 KB per half
constexpr int kVBytes = kSub;                      // Dv <= 128 rows x 32 keys: 16 KB per half
constexpr int kPBytes = kSub;                      // 128 rows x 32 keys: 16 KB per half
constexpr int kSmem = 2 * (kQBytes + kKBytes + kVBytes + kPBytes) + 1024;

struct FlashArgs {
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
                        const FlashArgs args) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t q_full, k_full, k_empty, v_full, v_empty, p_full, p_empty, drain;
  __shared__ __align__(8) uint64_t s_full[2], s_empty[2], o_full[2], o_empty[2];
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_word;

  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *q_hi = smem, *q_lo = q_hi + kQBytes;
  uint8_t *k_hi = q_lo + kQBytes, *k_lo = k_hi + kKBytes;
  uint8_t *v_hi = k_lo + kKBytes, *v_lo = v_hi + kVBytes;
  uint8_t *p_hi = v_lo + kVBytes, *p_lo = p_hi + kPBytes;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int head = blockIdx.y;
  const int64_t m0 = (int64_t)blockIdx.x * BM;
  const int nblocks = (int)((args.s_kv + BN - 1) / BN);
  const int dblocks = args.dp / 32;
  volatile int *abort = &abort_word;

  if (threadIdx.x == 0) {
    abort_word = 0;
    uint64_t *singles[] = {&q_full, &k_full, &k_empty, &v_full, &v_empty, &p_empty, &drain};
    for (uint64_t *b : singles) sm100::mbar_init(b, 1);
    for (int i = 0; i < 2; ++i) {
      sm100::mbar_init(&s_full[i], 1);
      sm100::mbar_init(&s_empty[i], 4);  // one arrival per softmax warp
      sm100::mbar_init(&o_full[i], 1);
      sm100::mbar_init(&o_empty[i], 4);
    }
    sm100::mbar_init(&p_full, 4);
    sm100::fence_barrier_init();
  }
  if (warp == 1) sm100::tmem_alloc(&tmem_slot, 512);
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = tmem_slot;
  // TMEM columns: S buffers at [0, 32) and [32, 64); O buffers at [128, 256) and [256, 384).
  auto s_col = [](int b) { return (uint32_t)(b * BN); };
  auto o_col = [](int b) { return (uint32_t)(128 + b * 128); };

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer
      sm100::mbar_arrive_expect_tx(&q_full, 2 * dblocks * kSub);
      for (int c = 0; c < dblocks; ++c) {
        sm100::tma_load_3d(q_hi + c * kSub, &map_qhi, &q_full, c * 32, (int)m0, head);
        sm100::tma_load_3d(q_lo + c * kSub, &map_qlo, &q_full, c * 32, (int)m0, head);
      }
      int k_issued = 0, v_issued = 0;
      for (int j = 0; j < nblocks; ++j) {
        if (j > 0 && !sm100::mbar_wait(&k_empty, (j - 1) & 1, args.err, sm100::kSiteAttention, abort)) break;
        sm100::mbar_arrive_expect_tx(&k_full, 2 * dblocks * BN * 128);
        for (int c = 0; c < dblocks; ++c) {
          sm100::tma_load_3d(k_hi + c * BN * 128, &map_khi, &k_full, c * 32, j * BN, head);
          sm100::tma_load_3d(k_lo + c * BN * 128, &map_klo, &k_full, c * 32, j * BN, head);
        }
        k_issued = j + 1;
        if (j > 0 && !sm100::mbar_wait(&v_empty, (j - 1) & 1, args.err, sm100::kSiteAttention, abort)) break;
        sm100::mbar_arrive_expect_tx(&v_full, 2 * kVBytes);
        sm100::tma_load_3d(v_hi, &map_vhi, &v_full, j * BN, 0, head);
        sm100::tma_load_3d(v_lo, &map_vlo, &v_full, j * BN, 0, head);
        v_issued = j + 1;
      }
      // drain loads in flight (budget only)
      int never = 0;
      sm100::mbar_wait(&q_full, 0, args.err, sm100::kSiteDrain, &never);
      if (k_issued) sm100::mbar_wait(&k_full, (k_issued - 1) & 1, args.err, sm100::kSiteDrain, &never);
      if (v_issued) sm100::mbar_wait(&v_full, (v_issued - 1) & 1, args.err, sm100::kSiteDrain, &never);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer
      const uint32_t id_s = sm100::idesc_tf32(BM, BN);
      const uint32_t id_o = sm100::idesc_tf32(BM, args.n_pv);
      const uint32_t qh = sm100::smem_addr(q_hi), ql = sm100::smem_addr(q_lo);
      const uint32_t kh = sm100::smem_addr(k_hi), kl = sm100::smem_addr(k_lo);
      const uint32_t vh = sm100::smem_addr(v_hi), vl = sm100::smem_addr(v_lo);
      const uint32_t ph = sm100::smem_addr(p_hi), pl = sm100::smem_addr(p_lo);
      bool ok = sm100::mbar_wait(&q_full, 0, args.err, sm100::kSiteAttention, abort);
      auto issue_s = [&](int j) -> bool {
        const int b = j & 1;
        if (j >= 2 && !sm100::mbar_wait(&s_empty[b], ((j >> 1) - 1) & 1, args.err, sm100::kSiteAttention, abort))
          return false;
        if (!sm100::mbar_wait(&k_full, j & 1, args.err, sm100::kSiteAttention, abort)) return false;
        sm100::tc_fence_after();
        const uint32_t d = tmem + s_col(b);
        for (int k = 0; k < dblocks * 4; ++k) {
          const uint32_t qa = (uint32_t)((k >> 2) * kSub + (k & 3) * 32);
          const uint32_t ka = (uint32_t)((k >> 2) * BN * 128 + (k & 3) * 32);
          const uint64_t dqh = sm100::desc_kmajor<128>(qh + qa), dql = sm100::desc_kmajor<128>(ql + qa);
          const uint64_t dkh = sm100::desc_kmajor<128>(kh + ka), dkl = sm100::desc_kmajor<128>(kl + ka);
          sm100::mma_tf32(d, dql, dkh, id_s, k == 0 ? 0u : 1u);
          sm100::mma_tf32(d, dqh, dkl, id_s, 1u);
          sm100::mma_tf32(d, dqh, dkh, id_s, 1u);
        }
        sm100::mma_commit(&k_empty);
        sm100::mma_commit(&s_full[b]);
        return true;
      };
      auto issue_o = [&](int j) -> bool {
        const int b = j & 1;
        if (j >= 2 && !sm100::mbar_wait(&o_empty[b], ((j >> 1) - 1) & 1, args.err, sm100::kSiteAttention, abort))
          return false;
        if (!sm100::mbar_wait(&p_full, j & 1, args.err, sm100::kSiteAttention, abort)) return false;
        if (!sm100::mbar_wait(&v_full, j & 1, args.err, sm100::kSiteAttention, abort)) return false;
        sm100::tc_fence_after();
        const uint32_t d = tmem + o_col(b);
        for (int k = 0; k < BN / 8; ++k) {
          const uint32_t off = (uint32_t)(k * 32);
          const uint64_t dph = sm100::desc_kmajor<128>(ph + off), dpl = sm100::desc_kmajor<128>(pl + off);
          const uint64_t dvh = sm100::desc_kmajor<128>(vh + off), dvl = sm100::desc_kmajor<128>(vl + off);
          sm100::mma_tf32(d, dpl, dvh, id_o, k == 0 ? 0u : 1u);
          sm100::mma_tf32(d, dph, dvl, id_o, 1u);
          sm100::mma_tf32(d, dph, dvh, id_o, 1u);
        }
        sm100::mma_commit(&p_empty);
        sm100::mma_commit(&v_empty);
        sm100::mma_commit(&o_full[b]);
        return true;
      };
      for (int j = 0; ok && j <= nblocks; ++j) {
        if (j < nblocks) ok = issue_s(j);
        if (ok && j >= 1) ok = issue_o(j - 1);
      }
      sm100::mma_commit(&drain);
      int never = 0;
      sm100::mbar_wait(&drain, 0, args.err, sm100::kSiteDrain, &never);
    }
  } else {
    // ---------------- softmax + O accumulation: thread = query row
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // row within the tile == TMEM lane
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    const float inv_scale = args.scale_ptr ? __frcp_rn(__ldg(args.scale_ptr)) : args.inv_scale;
    constexpr int OC = 128;  // O columns held per thread (>= n_pv)
    float o_acc[OC];
#pragma unroll
    for (int i = 0; i < OC; ++i) o_acc[i] = 0.0f;
    float m_run = -INFINITY, l_run = 0.0f, alpha_prev = 0.0f;
    bool ok = true;
    uint8_t *prow_hi = p_hi + r * 128, *prow_lo = p_lo + r * 128;
    for (int j = 0; j <= nblocks && ok; ++j) {
      float alpha = 1.0f;
      if (j < nblocks) {
        const int b = j & 1;
        ok = sm100::mbar_wait(&s_full[b], (j >> 1) & 1, args.err, sm100::kSiteAttention, abort);
        if (!ok) break;
        sm100::tc_fence_after();
        uint32_t sr[32];
        sm100::tmem_ld_32x32b_x32(tmem + lane_base + s_col(b), sr);
        sm100::tmem_ld_wait();
        sm100::tc_fence_before();
        __syncwarp();
        if (lane == 0) sm100::mbar_arrive(&s_empty[b]);
        float x[32];
        float mx = m_run;
        const int64_t c0 = (int64_t)j * BN;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          x[i] = (c0 + i < args.s_kv) ? __fmul_rn(__uint_as_float(sr[i]), inv_scale) : -INFINITY;
          mx = fmaxf(mx, x[i]);
        }
        alpha = b2k_exp(__fsub_rn(m_run, mx));
        float sum = 0.0f;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          x[i] = b2k_exp(__fsub_rn(x[i], mx));
          sum += x[i];
        }
        l_run = __fadd_rn(__fmul_rn(l_run, alpha), sum);
        m_run = mx;
        // P_j into the swizzled A tile once O_{j-1}'s MMA has released it
        if (j > 0) {
          ok = sm100::mbar_wait(&p_empty, (j - 1) & 1, args.err, sm100::kSiteAttention, abort);
          if (!ok) break;
        }
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          float4 h, l;
          split_tf32(x[4 * c + 0], h.x, l.x);
          split_tf32(x[4 * c + 1], h.y, l.y);
          split_tf32(x[4 * c + 2], h.z, l.z);
          split_tf32(x[4 * c + 3], h.w, l.w);
          const int pos = (c ^ (r & 7)) * 16;
          *reinterpret_cast<float4 *>(prow_hi + pos) = h;
          *reinterpret_cast<float4 *>(prow_lo + pos) = l;
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) sm100::mbar_arrive(&p_full);
      }
      if (j >= 1) {
        // fold the finished O_{j-1} = P_{j-1} V_{j-1}
        const int jb = j - 1, b = jb & 1;
        ok = sm100::mbar_wait(&o_full[b], (jb >> 1) & 1, args.err, sm100::kSiteAttention, abort,
                              3 * sm100::kWaitCycles);
        if (!ok) break;
        sm100::tc_fence_after();
#pragma unroll
        for (int c = 0; c < OC; c += 32) {
          if (c >= args.n_pv) break;  // warp-uniform
          uint32_t orr[32];
          sm100::tmem_ld_32x32b_x32(tmem + lane_base + o_col(b) + (uint32_t)c, orr);
          sm100::tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) o_acc[c + i] = __fadd_rn(__fmul_rn(o_acc[c + i], alpha_prev), __uint_as_float(orr[i]));
        }
        sm100::tc_fence_before();
        __syncwarp();
        if (lane == 0) sm100::mbar_arrive(&o_empty[b]);
      }
      alpha_prev = alpha;
    }
    const int64_t row = m0 + r;
    if (ok && row < args.s_q) {
      const float inv_l = __frcp_rn(l_run);
      float *orow = args.o + ((int64_t)head * args.s_q + row) * args.dv;
      const bool vec = (args.dv % 4 == 0) && ((reinterpret_cast<uintptr_t>(args.o) & 15) == 0);
      if (vec) {
#pragma unroll
        for (int i = 0; i < OC; i += 4)
          if (i < args.dv)
            *reinterpret_cast<float4 *>(orow + i) =
                make_float4(__fmul_rn(o_acc[i], inv_l), __fmul_rn(o_acc[i + 1], inv_l), __fmul_rn(o_acc[i + 2], inv_l),
                            __fmul_rn(o_acc[i + 3], inv_l));
      } else {
#pragma unroll
        for (int i = 0; i < OC; ++i)
          if (i < args.dv) orow[i] = __fmul_rn(o_acc[i], inv_l);
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

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void *p = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// [batch][rows][inner] FP32, box [1][box_rows][32] with the 128-byte swizzle.
int make_map(b2k_ctx *ctx, CUtensorMap *map, const float *base, int64_t inner, int64_t rows, int64_t batch,
             int box_rows) {
  auto encode = encode_fn();
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
  if ((status = split_rows(ctx, q, s_q, d, d, s_q * d, bh, dp, q_hi, q_lo, s)) != B2K_OK) return status;
  status = k_layout == B2K_K_SD ? split_rows(ctx, k, s_kv, d, d, s_kv * d, bh, dp, k_hi, k_lo, s)
                                : split_transpose(ctx, k, d, s_kv, s_kv, d * s_kv, bh, dp, k_hi, k_lo, s);
  if (status != B2K_OK) return status;
  if ((status = split_transpose(ctx, v, s_kv, dv, dv, s_kv * dv, bh, sp, v_hi, v_lo, s)) != B2K_OK) return status;
  CUtensorMap maps[6];
  if ((status = make_map(ctx, &maps[0], q_hi, dp, s_q, bh, BM)) != B2K_OK) return status;
  if ((status = make_map(ctx, &maps[1], q_lo, dp, s_q, bh, BM)) != B2K_OK) return status;
  if ((status = make_map(ctx, &maps[2], k_hi, dp, s_kv, bh, BN)) != B2K_OK) return status;
  if ((status = make_map(ctx, &maps[3], k_lo, dp, s_kv, bh, BN)) != B2K_OK) return status;
  if ((status = make_map(ctx, &maps[4], v_hi, sp, dv, bh, 128)) != B2K_OK) return status;
  if ((status = make_map(ctx, &maps[5], v_lo, sp, dv, bh, 128)) != B2K_OK) return status;
  FlashArgs args{o, s_q, s_kv, dv, (int)dp, (int)((dv + 15) / 16 * 16), 1.0f / scale_div, scale_div_ptr,
                 ctx->error_flag};
  cudaError_t err = cudaFuncSetAttribute(flash_tf32x3_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
  if (err != cudaSuccess) return cuda_fail(ctx, err, "flash: set smem");
  dim3 grid((unsigned)((s_q + BM - 1) / BM), (unsigned)bh);
  PhaseTimer timer(ctx, B2K_PHASE_FLASH, s);
  flash_tf32x3_kernel<<<grid, kThreads, kSmem, s>>>(maps[0], maps[1], maps[2], maps[3], maps[4], maps[5], args);
  return check_launch(ctx, "flash launch");
}

}  // namespace b2k
