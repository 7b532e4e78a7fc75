// Attention O = softmax(Q K^T / scale) V with both contractions as 3xTF32 on
// the tensor cores, batched over batch*heads.
//
// The reference fuses this per head in SIMT FP32 (compile.py:7009-7966:
// hoisted score rows in shared memory, softmax with the selective exp, then
// the P.V fold).  Here the work is three batched passes over HBM:
//   1. split Q and K once into TF32 hi/lo halves (K-major),
//      S = (Q K^T) / scale on tcgen05 with the divide in the GEMM epilogue;
//   2. row softmax of S (selective exp) written directly as the hi/lo halves
//      of P, the A operand of the next contraction;
//   3. split V (transposed to K-major) and O = P V on tcgen05.
// Every score row is complete before its softmax, so no online rescaling is
// needed; the cost is S and P round-tripping HBM.
#include "common.cuh"

namespace {

inline int64_t round32(int64_t x) { return (x + 31) / 32 * 32; }

// 1 = fused kernel, one CTA per query tile (default), 0 = three passes
// (tests and benchmarks compare them).
int g_attention_mode = 1;

}  // namespace

int b2k::attention_mode() { return g_attention_mode; }

extern "C" int b2k_attention_set_fused(int mode) {
  if (mode < 0 || mode > 1) return B2K_EINVAL;
  g_attention_mode = mode;
  return B2K_OK;
}

size_t b2k_attention_workspace_floats(int64_t bh, int64_t s_q, int64_t s_kv, int64_t d, int64_t dv) {
  const int64_t dp = b2k::gemm_kpad(d), sp = b2k::gemm_kpad(s_kv);
  return (size_t)(2 * bh * s_q * dp + 2 * bh * s_kv * dp + round32(bh * s_q * s_kv) + 2 * bh * s_q * sp +
                  2 * bh * dv * sp);
}

extern "C" int b2k_attention_tf32x3(b2k_ctx *ctx, const float *q, const float *k, const float *v, float *o,
                                    int64_t bh, int64_t s_q, int64_t s_kv, int64_t d, int64_t dv, float scale_div,
                                    const float *scale_div_ptr, int32_t k_layout, void *stream) {
  B2K_CHECK_CTX(ctx);
  if (bh < 0 || s_q < 0 || s_kv < 0 || d < 0 || dv < 0) return b2k::fail(ctx, B2K_EINVAL, "attention: negative extent");
  if (k_layout != B2K_K_SD && k_layout != B2K_K_DS) return b2k::fail(ctx, B2K_EINVAL, "attention: bad k_layout");
  if (bh == 0 || s_q == 0 || dv == 0) return B2K_OK;
  if (!q || !k || !v || !o) return b2k::fail(ctx, B2K_EINVAL, "attention: null buffer");
  if (s_kv == 0 || d == 0) return b2k::fail(ctx, B2K_EUNSUPPORTED, "attention: empty key or head dimension");
  if (bh > 65535) return b2k::fail(ctx, B2K_EINVAL, "attention: batch*heads exceeds 65535");
  if (s_q > INT32_MAX - 256 || s_kv > INT32_MAX - 256 || d > INT32_MAX - 64 || dv > INT32_MAX - 256)
    return b2k::fail(ctx, B2K_EINVAL, "attention: extent exceeds 32-bit TMA coordinates");
  if (!scale_div_ptr && !(scale_div != 0.0f)) return b2k::fail(ctx, B2K_EINVAL, "attention: zero scale divisor");
  cudaStream_t s = (cudaStream_t)stream;
  if (b2k::flash_supported(d, dv) && g_attention_mode != 0) {
    int status = b2k::reserve_workspace(ctx, b2k::flash_workspace_floats(bh, s_q, s_kv, d, dv) * sizeof(float), s);
    if (status != B2K_OK) return status;
    b2k::PhaseTimer timer(ctx, B2K_PHASE_ATTENTION, s);
    return b2k::flash_attention(ctx, q, k, v, o, bh, s_q, s_kv, d, dv, scale_div, scale_div_ptr, k_layout,
                                static_cast<float *>(ctx->workspace), s);
  }
  int status = b2k::reserve_workspace(ctx, b2k_attention_workspace_floats(bh, s_q, s_kv, d, dv) * sizeof(float), s);
  if (status != B2K_OK) return status;
  const int64_t dp = b2k::gemm_kpad(d), sp = b2k::gemm_kpad(s_kv);
  float *w = static_cast<float *>(ctx->workspace);
  float *q_hi = w, *q_lo = q_hi + bh * s_q * dp;
  float *k_hi = q_lo + bh * s_q * dp, *k_lo = k_hi + bh * s_kv * dp;
  float *scores = k_lo + bh * s_kv * dp;
  float *p_hi = scores + round32(bh * s_q * s_kv), *p_lo = p_hi + bh * s_q * sp;
  float *v_hi = p_lo + bh * s_q * sp, *v_lo = v_hi + bh * dv * sp;
  b2k::PhaseTimer timer(ctx, B2K_PHASE_ATTENTION, s);
  // 1. S = Q K^T / scale
  if ((status = b2k::split_rows(ctx, q, s_q, d, d, s_q * d, bh, dp, q_hi, q_lo, s)) != B2K_OK) return status;
  status = k_layout == B2K_K_SD ? b2k::split_rows(ctx, k, s_kv, d, d, s_kv * d, bh, dp, k_hi, k_lo, s)
                                : b2k::split_transpose(ctx, k, d, s_kv, s_kv, d * s_kv, bh, dp, k_hi, k_lo, s);
  if (status != B2K_OK) return status;
  b2k::SplitOperands qk{q_hi, q_lo, k_hi, k_lo, dp};
  status = b2k::gemm_main(ctx, qk, s_q, s_kv, bh, scores, s_kv, s_q * s_kv, nullptr, 0, scale_div_ptr, scale_div, s);
  if (status != B2K_OK) return status;
  // 2. P = softmax(S), written as its TF32 halves
  if ((status = b2k::softmax_split_rows(ctx, scores, bh * s_q, s_kv, s_kv, p_hi, p_lo, sp, s)) != B2K_OK)
    return status;
  // 3. O = P V
  if ((status = b2k::split_transpose(ctx, v, s_kv, dv, dv, s_kv * dv, bh, sp, v_hi, v_lo, s)) != B2K_OK)
    return status;
  b2k::SplitOperands pv{p_hi, p_lo, v_hi, v_lo, sp};
  return b2k::gemm_main(ctx, pv, s_q, dv, bh, o, dv, s_q * dv, nullptr, 0, nullptr, 1.0f, s);
}
