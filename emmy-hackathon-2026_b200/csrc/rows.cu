// Row reductions and row norms: the rest of the reference's row family.
//
// The reference lowers these through its merged vector row reduction
// (compile.py:4987-5165: thread-strided fold with v4 loads, shfl.sync
// butterfly, shared halving tree) and, for norms, a second pass over the row
// that reuses the reduction's loads (row map reuse, compile.py:5511-5665).
// Here one CTA owns a row: for rows that fit (<= 16,384 columns, 16-byte
// aligned) the row stays in registers between the reduction and the map, so
// HBM sees one read (+ one write for norms); longer rows re-read through L2.
// A whole-array sum (one very long row) is split over many CTAs whose partial
// sums are combined in a fixed order by a second launch (deterministic).
#include <math.h>

#include "common.cuh"

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;

struct RowArgs {
  int op;
  float sum_div;
  const float *sum_div_ptr;
  float ms_div;
  const float *ms_div_ptr;
  float eps;
  const float *eps_ptr;
  const float *w;
};

__device__ __forceinline__ float block_sum(float v, float *scratch) {
  v = warp_sum(v);
  if ((threadIdx.x & 31) == 0) scratch[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = 0.0f;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) r += scratch[w];
  return r;
}

__device__ __forceinline__ float row_scale(const RowArgs &a, float acc) {
  if (a.op == B2K_ROW_SUM) return __fdiv_rn(acc, a.sum_div_ptr ? __ldg(a.sum_div_ptr) : a.sum_div);
  const float count = a.ms_div_ptr ? __ldg(a.ms_div_ptr) : a.ms_div;
  const float eps = a.eps_ptr ? __ldg(a.eps_ptr) : a.eps;
  const float ms = a.op == B2K_ROW_RMSNORM ? __fmul_rn(acc, __frcp_rn(count)) : acc;
  return __frcp_rn(__fsqrt_rn(__fadd_rn(ms, eps)));
}

template <int VPT>
__global__ void __launch_bounds__(kThreads) rows_vec(const RowArgs a, const float *__restrict__ x, float *__restrict__ y,
                                                     int64_t cols4, int64_t ldx, int64_t ldy) {
  grid_dependency_wait();
  grid_dependents_launch();
  __shared__ float red[kWarps];
  const int64_t row = blockIdx.x;
  const float4 *xr = reinterpret_cast<const float4 *>(x + row * ldx);
  float4 v[VPT];
  float acc = 0.0f;
  const bool squares = a.op != B2K_ROW_SUM;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int64_t c = threadIdx.x + (int64_t)k * kThreads;
    if (c < cols4) {
      v[k] = ld_stream(xr + c);
      acc += squares ? (v[k].x * v[k].x + v[k].y * v[k].y) + (v[k].z * v[k].z + v[k].w * v[k].w)
                     : (v[k].x + v[k].y) + (v[k].z + v[k].w);
    }
  }
  acc = block_sum(acc, red);
  const float s = row_scale(a, acc);
  if (a.op == B2K_ROW_SUM) {
    if (threadIdx.x == 0) y[row] = s;
    return;
  }
  float4 *yr = reinterpret_cast<float4 *>(y + row * ldy);
  const float4 *wr = reinterpret_cast<const float4 *>(a.w);
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int64_t c = threadIdx.x + (int64_t)k * kThreads;
    if (c < cols4) {
      float4 o = make_float4(__fmul_rn(v[k].x, s), __fmul_rn(v[k].y, s), __fmul_rn(v[k].z, s), __fmul_rn(v[k].w, s));
      if (wr) {
        const float4 w = __ldg(wr + c);
        o = make_float4(__fmul_rn(o.x, w.x), __fmul_rn(o.y, w.y), __fmul_rn(o.z, w.z), __fmul_rn(o.w, w.w));
      }
      st_stream(yr + c, o);
    }
  }
}

__global__ void __launch_bounds__(kThreads) rows_generic(const RowArgs a, const float *__restrict__ x,
                                                         float *__restrict__ y, int64_t cols, int64_t ldx,
                                                         int64_t ldy) {
  grid_dependency_wait();
  grid_dependents_launch();
  __shared__ float red[kWarps];
  const int64_t row = blockIdx.x;
  const float *xr = x + row * ldx;
  const bool squares = a.op != B2K_ROW_SUM;
  float acc = 0.0f;
  for (int64_t c = threadIdx.x; c < cols; c += kThreads) {
    const float v = __ldg(xr + c);
    acc += squares ? v * v : v;
  }
  acc = block_sum(acc, red);
  const float s = row_scale(a, acc);
  if (a.op == B2K_ROW_SUM) {
    if (threadIdx.x == 0) y[row] = s;
    return;
  }
  for (int64_t c = threadIdx.x; c < cols; c += kThreads) {
    float o = __fmul_rn(__ldg(xr + c), s);
    if (a.w) o = __fmul_rn(o, __ldg(a.w + c));
    y[row * ldy + c] = o;
  }
}

// Whole-array sum, stage 1: CTA b folds elements b, b + stride, ... in a
// fixed order and writes one partial.
__global__ void __launch_bounds__(kThreads) sum_partials(const float *__restrict__ x, int64_t n,
                                                         float *__restrict__ partials) {
  grid_dependency_wait();
  grid_dependents_launch();
  __shared__ float red[kWarps];
  float acc = 0.0f;
  const int64_t stride = (int64_t)gridDim.x * kThreads;
  for (int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x; i < n; i += stride) acc += __ldg(x + i);
  acc = block_sum(acc, red);
  if (threadIdx.x == 0) partials[blockIdx.x] = acc;
}

// Stage 2: one CTA sums the partials in index order.
__global__ void __launch_bounds__(kThreads) sum_finish(const RowArgs a, const float *__restrict__ partials, int count,
                                                       float *__restrict__ y) {
  grid_dependency_wait();
  grid_dependents_launch();
  __shared__ float red[kWarps];
  float acc = 0.0f;
  for (int i = threadIdx.x; i < count; i += kThreads) acc += partials[i];
  acc = block_sum(acc, red);
  if (threadIdx.x == 0) y[0] = row_scale(a, acc);
}

// Row folds with a non-additive operator (max, min, product), one CTA per
// row: thread-strided fold, shfl.xor butterfly, then the warps' partials in
// warp order -- a fixed order, so repeated runs are bit-identical.
template <int OP>
__device__ __forceinline__ float fold_op(float a, float b) {
  if constexpr (OP == B2K_ROW_MAX) return fmaxf(a, b);
  else if constexpr (OP == B2K_ROW_MIN) return fminf(a, b);
  else return __fmul_rn(a, b);
}

template <int OP>
__device__ __forceinline__ float fold_identity() {
  if constexpr (OP == B2K_ROW_MAX) return -INFINITY;
  else if constexpr (OP == B2K_ROW_MIN) return INFINITY;
  else return 1.0f;
}

template <int OP>
__global__ void __launch_bounds__(kThreads) rows_fold(const float *__restrict__ x, float *__restrict__ y,
                                                      int64_t cols, int64_t ldx) {
  grid_dependency_wait();
  grid_dependents_launch();
  __shared__ float red[kWarps];
  const float *xr = x + (int64_t)blockIdx.x * ldx;
  float acc = fold_identity<OP>();
  for (int64_t c = threadIdx.x; c < cols; c += kThreads) acc = fold_op<OP>(acc, __ldg(xr + c));
#pragma unroll
  for (int offset = 16; offset > 0; offset >>= 1) acc = fold_op<OP>(acc, __shfl_xor_sync(0xffffffffu, acc, offset));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float r = red[0];
#pragma unroll
    for (int w = 1; w < kWarps; ++w) r = fold_op<OP>(r, red[w]);
    y[blockIdx.x] = r;
  }
}

// Fold over the middle axis of [batch][s][cols]: one thread per output
// column j, folding i = 0 .. s-1 in order (the IR's serial Loop + Accum over
// that axis).  Consecutive threads hold consecutive columns, so every step of
// every fold is one coalesced read of a row segment.  Each thread loads
// kAxisAhead rows before folding them in order: with few output columns (a
// long fold over few cells) the loads in flight, not the threads, carry the
// bandwidth: [8, 8192, 4096] ran at 1.7 TB/s with 8 rows ahead, 3.1 with 32
// and 3.8 with 64 (no spills; other shapes unchanged).
constexpr int kAxisAhead = 64;

template <int OP>
__global__ void __launch_bounds__(kThreads) axis_fold(const float *__restrict__ x, float *__restrict__ y,
                                                      int64_t batch, int64_t s_len, int64_t cols,
                                                      const float *div_ptr, float div) {
  grid_dependency_wait();
  grid_dependents_launch();
  const int64_t j = (int64_t)blockIdx.x * kThreads + threadIdx.x;
  if (j >= cols) return;
  for (int64_t b = blockIdx.y; b < batch; b += gridDim.y) {
    const float *xb = x + b * s_len * cols + j;
    float acc = OP == B2K_ROW_SUM ? 0.0f : fold_identity<OP>();
    auto fold = [&](float v) { acc = OP == B2K_ROW_SUM ? __fadd_rn(acc, v) : fold_op<OP>(acc, v); };
    int64_t i = 0;
    for (; i + kAxisAhead <= s_len; i += kAxisAhead) {
      float v[kAxisAhead];
#pragma unroll
      for (int u = 0; u < kAxisAhead; ++u) v[u] = __ldg(xb + (i + u) * cols);
#pragma unroll
      for (int u = 0; u < kAxisAhead; ++u) fold(v[u]);
    }
    for (; i < s_len; ++i) fold(__ldg(xb + i * cols));
    if (OP == B2K_ROW_SUM) {
      const float d = div_ptr ? __ldg(div_ptr) : div;
      if (div_ptr || d != 1.0f) acc = __fdiv_rn(acc, d);
    }
    y[b * cols + j] = acc;
  }
}

}  // namespace

extern "C" int b2k_axis_reduce_f32(b2k_ctx *ctx, int32_t op, const float *x, float *y, int64_t batch, int64_t s,
                                   int64_t cols, float div, const float *div_ptr, void *stream) {
  B2K_CHECK_CTX(ctx);
  if (op != B2K_ROW_SUM && op != B2K_ROW_MAX && op != B2K_ROW_MIN && op != B2K_ROW_PROD)
    return b2k::fail(ctx, B2K_EINVAL, "axis_reduce: op %d is not a fold", op);
  if (batch < 0 || s < 0 || cols < 0) return b2k::fail(ctx, B2K_EINVAL, "axis_reduce: negative extent");
  if (batch == 0 || cols == 0) return B2K_OK;
  if (!y || (s > 0 && !x)) return b2k::fail(ctx, B2K_EINVAL, "axis_reduce: null buffer");
  if ((cols + kThreads - 1) / kThreads > INT32_MAX) return b2k::fail(ctx, B2K_EINVAL, "axis_reduce: too many columns");
  cudaStream_t st = (cudaStream_t)stream;
  b2k::PhaseTimer timer(ctx, B2K_PHASE_ROWS, st);
  const dim3 g((unsigned)((cols + kThreads - 1) / kThreads), (unsigned)std::min<int64_t>(batch, 65535)), b(kThreads);
  const bool pdl = b2k::pdl_enabled();
  switch (op) {
    case B2K_ROW_SUM: b2k::launch_kernel(pdl, axis_fold<B2K_ROW_SUM>, g, b, 0, st, x, y, batch, s, cols, div_ptr, div); break;
    case B2K_ROW_MAX: b2k::launch_kernel(pdl, axis_fold<B2K_ROW_MAX>, g, b, 0, st, x, y, batch, s, cols, div_ptr, div); break;
    case B2K_ROW_MIN: b2k::launch_kernel(pdl, axis_fold<B2K_ROW_MIN>, g, b, 0, st, x, y, batch, s, cols, div_ptr, div); break;
    default: b2k::launch_kernel(pdl, axis_fold<B2K_ROW_PROD>, g, b, 0, st, x, y, batch, s, cols, div_ptr, div); break;
  }
  return b2k::check_launch(ctx, "axis_reduce launch");
}

extern "C" int b2k_row_op_f32(b2k_ctx *ctx, const b2k_row_params *params, const float *x, float *y, int64_t rows,
                              int64_t cols, int64_t ld_x, int64_t ld_y, void *stream) {
  B2K_CHECK_CTX(ctx);
  if (!params) return b2k::fail(ctx, B2K_EINVAL, "row_op: null params");
  if (params->op < B2K_ROW_SUM || params->op > B2K_ROW_PROD)
    return b2k::fail(ctx, B2K_EINVAL, "row_op: unknown op %d", params->op);
  const bool reduction = params->op == B2K_ROW_SUM || params->op >= B2K_ROW_MAX;  // one value per row
  if (rows < 0 || cols < 0) return b2k::fail(ctx, B2K_EINVAL, "row_op: negative extent");
  if (rows == 0) return B2K_OK;
  if (!x || !y) return b2k::fail(ctx, B2K_EINVAL, "row_op: null buffer");
  if (ld_x < cols || (!reduction && ld_y < cols))
    return b2k::fail(ctx, B2K_EINVAL, "row_op: leading dimension < cols");
  if (rows > INT32_MAX) return b2k::fail(ctx, B2K_EINVAL, "row_op: too many rows");
  if (params->op >= B2K_ROW_MAX) {
    cudaStream_t s = (cudaStream_t)stream;
    b2k::PhaseTimer timer(ctx, B2K_PHASE_ROWS, s);
    const int grid = (int)rows;
    const bool pdl = b2k::pdl_enabled();
    const dim3 g((unsigned)grid), b(kThreads);
    if (params->op == B2K_ROW_MAX) b2k::launch_kernel(pdl, rows_fold<B2K_ROW_MAX>, g, b, 0, s, x, y, cols, ld_x);
    else if (params->op == B2K_ROW_MIN) b2k::launch_kernel(pdl, rows_fold<B2K_ROW_MIN>, g, b, 0, s, x, y, cols, ld_x);
    else b2k::launch_kernel(pdl, rows_fold<B2K_ROW_PROD>, g, b, 0, s, x, y, cols, ld_x);
    return b2k::check_launch(ctx, "row_op fold launch");
  }
  const RowArgs a{params->op,  params->sum_div, params->sum_div_ptr, params->ms_div,
                  params->ms_div_ptr, params->eps, params->eps_ptr,     params->w};
  cudaStream_t s = (cudaStream_t)stream;
  b2k::PhaseTimer timer(ctx, B2K_PHASE_ROWS, s);
  if (params->op == B2K_ROW_SUM && rows == 1 && cols > 65536) {
    const int parts = ctx->sm_count * 4;
    int status = b2k::reserve_workspace(ctx, (size_t)parts * sizeof(float), s);
    if (status != B2K_OK) return status;
    float *partials = static_cast<float *>(ctx->workspace);
    b2k::launch_kernel(b2k::pdl_enabled(), sum_partials, dim3(parts), dim3(kThreads), 0, s, x, cols, partials);
    b2k::launch_kernel(b2k::pdl_enabled(), sum_finish, dim3(1), dim3(kThreads), 0, s, a, (const float *)partials,
                       parts, y);
    return b2k::check_launch(ctx, "row_op sum launch", 2);
  }
  const bool vec = (cols % 4 == 0) && (ld_x % 4 == 0) && b2k::aligned16(x) &&
                   (params->op == B2K_ROW_SUM || ((ld_y % 4 == 0) && b2k::aligned16(y) &&
                                                  (!params->w || b2k::aligned16(params->w))));
  const int64_t cols4 = cols / 4;
  const int grid = (int)rows;
  const bool pdl = b2k::pdl_enabled();
  const dim3 g((unsigned)grid), b(kThreads);
  if (vec && cols4 <= kThreads) b2k::launch_kernel(pdl, rows_vec<1>, g, b, 0, s, a, x, y, cols4, ld_x, ld_y);
  else if (vec && cols4 <= kThreads * 2) b2k::launch_kernel(pdl, rows_vec<2>, g, b, 0, s, a, x, y, cols4, ld_x, ld_y);
  else if (vec && cols4 <= kThreads * 4) b2k::launch_kernel(pdl, rows_vec<4>, g, b, 0, s, a, x, y, cols4, ld_x, ld_y);
  else if (vec && cols4 <= kThreads * 8) b2k::launch_kernel(pdl, rows_vec<8>, g, b, 0, s, a, x, y, cols4, ld_x, ld_y);
  else if (vec && cols4 <= kThreads * 16) b2k::launch_kernel(pdl, rows_vec<16>, g, b, 0, s, a, x, y, cols4, ld_x, ld_y);
  else b2k::launch_kernel(pdl, rows_generic, g, b, 0, s, a, x, y, cols, ld_x, ld_y);
  return b2k::check_launch(ctx, "row_op launch");
}
