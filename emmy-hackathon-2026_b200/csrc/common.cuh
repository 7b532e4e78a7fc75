// Shared definitions of the B200 backend: the context object, error plumbing
// and device helpers used by more than one kernel file.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <string>
#include <utility>
#include <vector>

#include "b200k.h"

struct b2k_ctx {
  int device = 0;
  int sm_count = 0;
  int max_smem_optin = 0;
  std::string error;
  // Context-owned scratch arena (grown on demand, never shrunk).
  void *workspace = nullptr;
  size_t workspace_bytes = 0;
  // Raw per-chunk accumulators of the chunk-split GEMM (grown on demand).
  void *partials = nullptr;
  size_t partials_bytes = 0;
  // Set on the stack contexts of the allocation-free entry points: nothing
  // may grow an arena, so paths that need one more (chunk split) are off.
  bool fixed_scratch = false;
  // Device-side error word written by kernels whose bounded waits expire.
  unsigned int *error_flag = nullptr;
  // Kernels enqueued through this context (b2k_kernel_launches).
  int64_t kernel_launches = 0;
  // Pipelined host-array calls (host.cu): copy streams, dependency events
  // (reused across calls) and the device staging arena.
  cudaStream_t copy_in = nullptr, copy_out = nullptr;
  // Compute streams of the pipelined GEMM: slab GEMMs run round-robin on
  // these so that short slabs (a few tiles each) fill the GPU together.
  static constexpr int kComputeStreams = 3;
  cudaStream_t compute[kComputeStreams] = {};
  std::vector<cudaEvent_t> sync_events;
  void *staging = nullptr;
  size_t staging_bytes = 0;
  // Optional per-phase CUDA-event timing (b2k_timing_*), for the phases
  // whose bit is set in timing_mask.
  bool timing = false;
  uint32_t timing_mask = ~0u;
  std::vector<cudaEvent_t> event_pool;
  std::vector<std::pair<cudaEvent_t, cudaEvent_t>> phase_events[B2K_PHASE_COUNT];
};

namespace b2k {

// Record a formatted reason on the context and return `code`.
inline int fail(b2k_ctx *ctx, int code, const char *fmt, ...) {
  char buffer[512];
  va_list args;
  va_start(args, fmt);
  vsnprintf(buffer, sizeof buffer, fmt, args);
  va_end(args);
  if (ctx) ctx->error = buffer;
  return code;
}

inline int cuda_fail(b2k_ctx *ctx, cudaError_t err, const char *what) {
  return fail(ctx, B2K_ECUDA, "%s: %s (%s)", what, cudaGetErrorName(err), cudaGetErrorString(err));
}

// Check the `launches` kernel launches just enqueued (configuration errors
// only; the kernels themselves run asynchronously) and count them.
inline int check_launch(b2k_ctx *ctx, const char *what, int launches = 1) {
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return cuda_fail(ctx, err, what);
  ctx->error.clear();
  ctx->kernel_launches += launches;
  return B2K_OK;
}

inline int make_current(b2k_ctx *ctx) {
  cudaError_t err = cudaSetDevice(ctx->device);
  if (err != cudaSuccess) return cuda_fail(ctx, err, "cudaSetDevice");
  return B2K_OK;
}

// Grow the context's scratch arena to at least `bytes`.
int reserve_workspace(b2k_ctx *ctx, size_t bytes, cudaStream_t stream);
// The same for the chunk-split GEMM's partial-accumulator arena.
int reserve_partials(b2k_ctx *ctx, size_t bytes, cudaStream_t stream);

// Raise a kernel's dynamic shared-memory limit once per (kernel, device):
// cudaFuncSetAttribute costs about a microsecond and a half of host time per
// call, a noticeable share of a short GEMM's enqueue cost.
inline cudaError_t set_max_smem(b2k_ctx *ctx, const void *kernel, int bytes) {
  static std::mutex mu;
  static std::vector<std::pair<const void *, int>> done;
  std::lock_guard<std::mutex> lock(mu);
  for (const auto &e : done)
    if (e.first == kernel && e.second == ctx->device) return cudaSuccess;
  cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (err == cudaSuccess) done.emplace_back(kernel, ctx->device);
  return err;
}

// Programmatic dependent launch (b2k_set_pdl, on by default): the kernels of
// one operation (operand split, then the tensor-core kernel) are launched
// with the programmatic-serialization attribute, so a kernel's CTAs may be
// scheduled and run their set-up (barrier init, TMEM allocation, tensor-map
// prefetch) while the previous kernel in the stream drains.  Every kernel
// launched this way executes grid_dependency_wait() before it touches global
// memory, which orders it after the previous kernel's completion and makes
// that kernel's writes visible.
bool pdl_enabled();

template <typename... KArgs, typename... Args>
inline cudaError_t launch_kernel(bool pdl, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                 cudaStream_t s, Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// --- 3xTF32 operand split and tensor-core GEMM (gemm.cu) ---------------------
// K is zero-padded to a multiple of 32 in the split operands.
inline int64_t gemm_kpad(int64_t k) { return (k + 31) / 32 * 32; }

// Split operands of a (batched) GEMM: A_hi/A_lo [batch][m][kp] and
// B_hi/B_lo [batch][n][kp], all K-major.
struct SplitOperands {
  float *a_hi, *a_lo, *b_hi, *b_lo;
  int64_t kp;
};

// In-kernel split GEMM (gemm_fused.cu).  gemm_split_mode returns the path a
// call takes under the b2k_gemm_set_fused_split switch: 0 = pre-pass split of
// both operands; kSplitDirect = A split into TMEM inside the kernel, B
// pre-split into `ops` (A TMA-readable: 16-byte aligned, row stride a
// multiple of 4 elements, K >= 16, not stored transposed); kSplitTransposed =
// C^T = B^T A^T with B split into TMEM inside the kernel and A pre-split (B
// TMA-readable).  Under the default switch the path with the lowest
// estimated time over `sms` SMs is taken.
constexpr int kSplitDirect = 1;
constexpr int kSplitTransposed = 2;
int gemm_split_mode(const float *a, const float *b, int64_t m, int64_t n, int64_t k, int64_t lda, int64_t ldb,
                    int layout, int sms, bool chunks_ok = true);
// Estimated microseconds of the chunk-split pre-pass GEMM (one 256-wide K
// chunk of one 128 x 128 tile per CTA, then an in-order fold of the chunks)
// for an m x n output with kp K elements on `sms` SMs; a huge value where it
// does not apply (fewer than two chunks, or b2k_gemm_set_chunk_split(0)).
double chunked_cost_us(int64_t m, int64_t n, int64_t kp, int sms);
// Tile width (columns) of the pre-pass kernel gemm_main picks for a [batch]
// m x n output with kp K elements on `sms` SMs, and that kernel's estimated time.
int main_tile_width(int64_t m, int64_t n, int64_t batch, int64_t kp, int sms);
double prepass_cost_us(int64_t tiles, int bn, int64_t kp, int sms);
// The tile variant selected with b2k_gemm_set_variant (2 = 128-wide tiles).
int gemm_variant();
int gemm_tmem_a(b2k_ctx *ctx, const float *a, int64_t k, int64_t lda, const SplitOperands &ops, float *c, int64_t m,
                int64_t n, int64_t ldc, const float *bias, int relu, cudaStream_t s);
// The transposed orientation: raw B ([k][n] row-major, or [n][k] when b_nk)
// split inside the kernel, the caller's A pre-split into ops.b_hi / b_lo
// ([m][kp]); C is the caller's [m][n].  `bn` is the tile width over m (128 or
// 192; 0 = gemm_transposed_tile_width(m, n, SMs)).
int gemm_tmem_b(b2k_ctx *ctx, const float *b, int64_t k, int64_t ldb, bool b_nk, const SplitOperands &ops, float *c,
                int64_t m, int64_t n, int64_t ldc, const float *bias, int relu, cudaStream_t s, int bn = 0);
int gemm_transposed_tile_width(int64_t m, int64_t n, int sms);
// Tile width of the direct orientation's kernel (128 or 192).
int gemm_direct_tile_width(int64_t n);
// Whether gemm_main runs a batch-1 m x n pre-pass GEMM (kp K elements, `sms`
// SMs) as the chunk split, under the current variant and chunk settings.
bool gemm_takes_chunks(int64_t m, int64_t n, int64_t kp, int sms);

// Row-major [batch][rows, k] -> hi/lo [batch][rows][kp].
int split_rows(b2k_ctx *ctx, const float *src, int64_t rows, int64_t k, int64_t ld, int64_t bs, int64_t batch,
               int64_t kp, float *hi, float *lo, cudaStream_t s);
// One row-major operand [batch][rows, k] (row stride ld, batch stride bs)
// and its hi/lo destination [batch][rows][kp].
struct RowSplit {
  const float *src;
  int64_t rows, k, ld, bs, batch;
  float *hi, *lo;
};
// Splits `a` and, when `b` is not null, `b` (same kp) in one launch.
int split_rows2(b2k_ctx *ctx, const RowSplit &a, const RowSplit *b, int64_t kp, cudaStream_t s);
// Row-major [batch][k, n] -> transposed hi/lo [batch][n][kp].
int split_transpose(b2k_ctx *ctx, const float *src, int64_t k, int64_t n, int64_t ld, int64_t bs, int64_t batch,
                    int64_t kp, float *hi, float *lo, cudaStream_t s);

// Row softmax of x [rows, cols] written as TF32 hi/lo halves [rows][kp] (softmax.cu).
int softmax_split_rows(b2k_ctx *ctx, const float *x, int64_t rows, int64_t cols, int64_t ld_x, float *hi,
                       float *lo, int64_t kp, cudaStream_t s);

// Attention path chosen with b2k_attention_set_fused (attention.cu).
int attention_mode();
// Fused attention (flash.cu): supported head dims, scratch, launch.
bool flash_supported(int64_t d, int64_t dv);
size_t flash_workspace_floats(int64_t bh, int64_t s_q, int64_t s_kv, int64_t d, int64_t dv);
int flash_attention(b2k_ctx *ctx, const float *q, const float *k, const float *v, float *o, int64_t bh, int64_t s_q,
                    int64_t s_kv, int64_t d, int64_t dv, float scale_div, const float *scale_div_ptr, int k_layout,
                    float *ws, cudaStream_t s);

// C[z] = epilogue(A[z] * B[z]^T) for z < batch on pre-split operands; the
// epilogue divides by *div_ptr (or div_value), adds bias[n], applies ReLU.
int gemm_main(b2k_ctx *ctx, const SplitOperands &ops, int64_t m, int64_t n, int64_t batch, float *c, int64_t ldc,
              int64_t batch_stride_c, const float *bias, int relu, const float *div_ptr, float div_value,
              cudaStream_t s, bool allow_chunks = false);

inline bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Brackets the kernels of one phase with CUDA events on `stream` when the
// context's timing is enabled; a no-op otherwise.
class PhaseTimer {
 public:
  PhaseTimer(b2k_ctx *ctx, int phase, cudaStream_t stream);
  ~PhaseTimer();

 private:
  b2k_ctx *ctx_;
  int phase_;
  cudaStream_t stream_;
  cudaEvent_t start_ = nullptr;
};

}  // namespace b2k

#define B2K_CHECK_CTX(ctx)                                   \
  do {                                                       \
    if (!(ctx)) return B2K_EINVAL;                           \
    int b2k_status_ = b2k::make_current(ctx);                \
    if (b2k_status_ != B2K_OK) return b2k_status_;           \
  } while (0)

// ---------------------------------------------------------------------------
// Device helpers
// ---------------------------------------------------------------------------

// Selective subnormal-preserving exponential (the reference's method,
// compile.py:2953-2965): t = x*log2(e) in FP32; arguments with t < -125 are
// shifted by +126 into the normal range of the flush-to-zero ex2, and the
// result is scaled back by an exact 2^-126 multiply that is NOT flushed, so
// results in the subnormal range survive.  Relies on this library being
// compiled without -ftz / --use_fast_math.
__device__ __forceinline__ float b2k_exp(float x) {
  float t = __fmul_rn(x, 1.44269502162933349609375f);  // f32(log2(e))
  const bool tiny = t < -125.0f;
  if (tiny) t = __fadd_rn(t, 126.0f);
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(t));
  if (tiny) r = __fmul_rn(r, 1.17549435082228750797e-38f);  // exact 2^-126
  return r;
}

// TF32 split of one FP32 value: hi = rna(x) with the bit rule of
// tf32_emitter.py:22-29 ((bits + 0x1000) & 0xFFFFE000), lo = rna(x - hi), so
// hi + lo carries x to about 2^-22 and both halves are exact TF32 values.
// Deviation from the reference model, on purpose: when rounding a finite x
// overflows to infinity (|x| near FLT_MAX) hi falls back to truncation, so
// max-finite * 0 stays 0 instead of inf * 0 = NaN (the bundled
// maxfinite-times-zero witness expects 0).  Non-finite x gives hi = x, lo = 0.
__device__ __forceinline__ void split_tf32(float x, float &hi, float &lo) {
  const uint32_t bits = __float_as_uint(x);
  if (!isfinite(x)) {
    hi = x;
    lo = 0.0f;
    return;
  }
  float h = __uint_as_float((bits + 0x1000u) & 0xFFFFE000u);
  if (!isfinite(h)) h = __uint_as_float(bits & 0xFFFFE000u);
  const float r = __fsub_rn(x, h);
  hi = h;
  lo = __uint_as_float((__float_as_uint(r) + 0x1000u) & 0xFFFFE000u);
}

// split_tf32 of four values.  When every |x| is below 0x7F7FF000 (bit
// pattern: finite, and rounding cannot carry into the exponent's all-ones
// value) the special cases cannot arise and the split is two integer ops per
// half; otherwise each value takes split_tf32.  Results are bit-identical.
__device__ __forceinline__ void split_tf32x4(const float4 &x, float4 &hi, float4 &lo) {
  const uint32_t b0 = __float_as_uint(x.x), b1 = __float_as_uint(x.y);
  const uint32_t b2 = __float_as_uint(x.z), b3 = __float_as_uint(x.w);
  const uint32_t mag = max(max(b0 & 0x7FFFFFFFu, b1 & 0x7FFFFFFFu), max(b2 & 0x7FFFFFFFu, b3 & 0x7FFFFFFFu));
  if (mag < 0x7F7FF000u) {
    hi.x = __uint_as_float((b0 + 0x1000u) & 0xFFFFE000u);
    hi.y = __uint_as_float((b1 + 0x1000u) & 0xFFFFE000u);
    hi.z = __uint_as_float((b2 + 0x1000u) & 0xFFFFE000u);
    hi.w = __uint_as_float((b3 + 0x1000u) & 0xFFFFE000u);
    lo.x = __uint_as_float((__float_as_uint(__fsub_rn(x.x, hi.x)) + 0x1000u) & 0xFFFFE000u);
    lo.y = __uint_as_float((__float_as_uint(__fsub_rn(x.y, hi.y)) + 0x1000u) & 0xFFFFE000u);
    lo.z = __uint_as_float((__float_as_uint(__fsub_rn(x.z, hi.z)) + 0x1000u) & 0xFFFFE000u);
    lo.w = __uint_as_float((__float_as_uint(__fsub_rn(x.w, hi.w)) + 0x1000u) & 0xFFFFE000u);
  } else {
    split_tf32(x.x, hi.x, lo.x);
    split_tf32(x.y, hi.y, lo.y);
    split_tf32(x.z, hi.z, lo.z);
    split_tf32(x.w, hi.w, lo.w);
  }
}

// Programmatic dependent launch, device side (see launch_kernel): wait until
// the previous kernel in the stream has completed and its writes are
// visible; allow the next kernel's CTAs to be scheduled.  Both are no-ops in
// a kernel launched without the programmatic-serialization attribute.
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dependents_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int offset = 16; offset > 0; offset >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, offset));
  return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int offset = 16; offset > 0; offset >>= 1) v += __shfl_xor_sync(0xffffffffu, v, offset);
  return v;
}

__device__ __forceinline__ float4 ld_stream(const float4 *p) {
  float4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ void st_stream(float4 *p, float4 v) {
  asm volatile("st.global.cs.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(v.x), "f"(v.y), "f"(v.z),
               "f"(v.w)
               : "memory");
}
