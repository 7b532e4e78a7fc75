// Row softmax: one CTA per row, the row held in registers between the max,
// exp-sum and normalise phases so HBM sees exactly one read and one write.
//
// The reference's f02 IR is an online max/sum recurrence that its emitter
// rewrites into a known-max form (compile.py:1656-1711 online_max_carriers,
// 6492-6539 two_pass_softmax, 6570-6644 fused_softmax_pass), combined across
// lanes with a shfl.sync butterfly (8958-9035) and across warps with a shared
// halving tree (9175-9268); exponentials use the selective subnormal method
// (2953-2965) and the normalisation is reciprocal-then-multiply.
#include <math.h>

#include "common.cuh"

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;

__device__ __forceinline__ float block_max(float v, float *scratch) {
  v = warp_max(v);
  if ((threadIdx.x & 31) == 0) scratch[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = scratch[0];
#pragma unroll
  for (int w = 1; w < kWarps; ++w) r = fmaxf(r, scratch[w]);
  return r;
}

__device__ __forceinline__ float block_sum(float v, float *scratch) {
  v = warp_sum(v);
  if ((threadIdx.x & 31) == 0) scratch[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = 0.0f;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) r += scratch[w];
  return r;
}

// Where a normalised row goes: a plain FP32 row, or (for the attention path)
// the TF32 hi/lo halves of the row, zero padded to `pad4` float4 chunks, in
// the K-major layout the 3xTF32 GEMM reads as its A operand.
struct PlainSink {
  float *y;
  int64_t ldy;
  __device__ __forceinline__ void put4(int64_t row, int64_t c4, float4 o) const {
    st_stream(reinterpret_cast<float4 *>(y + row * ldy) + c4, o);
  }
  __device__ __forceinline__ void put(int64_t row, int64_t c, float o) const { y[row * ldy + c] = o; }
  __device__ __forceinline__ void finish_row(int64_t, int64_t) const {}
};

struct SplitSink {
  float *hi, *lo;
  int64_t kp;  // padded row length (multiple of 32)
  __device__ __forceinline__ void put4(int64_t row, int64_t c4, float4 o) const {
    float4 h, l;
    split_tf32(o.x, h.x, l.x);
    split_tf32(o.y, h.y, l.y);
    split_tf32(o.z, h.z, l.z);
    split_tf32(o.w, h.w, l.w);
    st_stream(reinterpret_cast<float4 *>(hi + row * kp) + c4, h);
    st_stream(reinterpret_cast<float4 *>(lo + row * kp) + c4, l);
  }
  __device__ __forceinline__ void put(int64_t row, int64_t c, float o) const {
    float h, l;
    split_tf32(o, h, l);
    hi[row * kp + c] = h;
    lo[row * kp + c] = l;
  }
  // zero the padding columns [cols, kp) of the row
  __device__ __forceinline__ void finish_row(int64_t row, int64_t cols) const {
    for (int64_t c = cols + threadIdx.x; c < kp; c += blockDim.x) {
      hi[row * kp + c] = 0.0f;
      lo[row * kp + c] = 0.0f;
    }
  }
};

// VPT float4 chunks per thread; the row (cols4 = cols/4 chunks) must satisfy
// cols4 <= kThreads * VPT.  Rows are 16-byte aligned.
template <int VPT, class Sink>
__global__ void __launch_bounds__(kThreads) softmax_rows_vec(const float *__restrict__ x, const Sink sink,
                                                             int64_t cols4, int64_t ldx) {
  __shared__ float red_max[kWarps];
  __shared__ float red_sum[kWarps];
  grid_dependency_wait();
  grid_dependents_launch();
  const int64_t row = blockIdx.x;
  const float4 *xr = reinterpret_cast<const float4 *>(x + row * ldx);
  float4 v[VPT];
  float m = -INFINITY;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int64_t c = threadIdx.x + (int64_t)k * kThreads;
    if (c < cols4) {
      v[k] = ld_stream(xr + c);
      m = fmaxf(m, fmaxf(fmaxf(v[k].x, v[k].y), fmaxf(v[k].z, v[k].w)));
    }
  }
  m = block_max(m, red_max);
  float s = 0.0f;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int64_t c = threadIdx.x + (int64_t)k * kThreads;
    if (c < cols4) {
      v[k].x = b2k_exp(__fsub_rn(v[k].x, m));
      v[k].y = b2k_exp(__fsub_rn(v[k].y, m));
      v[k].z = b2k_exp(__fsub_rn(v[k].z, m));
      v[k].w = b2k_exp(__fsub_rn(v[k].w, m));
      s += (v[k].x + v[k].y) + (v[k].z + v[k].w);
    }
  }
  s = block_sum(s, red_sum);
  const float r = __frcp_rn(s);
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int64_t c = threadIdx.x + (int64_t)k * kThreads;
    if (c < cols4) {
      float4 o;
      o.x = __fmul_rn(v[k].x, r);
      o.y = __fmul_rn(v[k].y, r);
      o.z = __fmul_rn(v[k].z, r);
      o.w = __fmul_rn(v[k].w, r);
      sink.put4(row, c, o);
    }
  }
  sink.finish_row(row, cols4 * 4);
}

// Any row length / alignment: three passes over the row (max, exp-sum,
// normalise) with scalar coalesced accesses; later passes hit L2 for rows
// that fit there.
template <class Sink>
__global__ void __launch_bounds__(kThreads) softmax_rows_generic(const float *__restrict__ x, const Sink sink,
                                                                 int64_t cols, int64_t ldx) {
  grid_dependency_wait();
  grid_dependents_launch();
  __shared__ float red_max[kWarps];
  __shared__ float red_sum[kWarps];
  const int64_t row = blockIdx.x;
  const float *xr = x + row * ldx;
  float m = -INFINITY;
  for (int64_t c = threadIdx.x; c < cols; c += kThreads) m = fmaxf(m, __ldg(xr + c));
  m = block_max(m, red_max);
  float s = 0.0f;
  for (int64_t c = threadIdx.x; c < cols; c += kThreads) s += b2k_exp(__fsub_rn(__ldg(xr + c), m));
  s = block_sum(s, red_sum);
  const float r = __frcp_rn(s);
  for (int64_t c = threadIdx.x; c < cols; c += kThreads) sink.put(row, c, __fmul_rn(b2k_exp(__fsub_rn(__ldg(xr + c), m)), r));
  sink.finish_row(row, cols);
}

template <class Sink>
void launch_rows(const float *x, const Sink &sink, int64_t rows, int64_t cols, int64_t ld_x, bool vec,
                 cudaStream_t s) {
  const int64_t cols4 = cols / 4;
  const int grid = (int)rows;
  // programmatic dependent launch: back-to-back launches hide each other's
  // launch latency and tail (each kernel waits for its predecessor first)
  const bool pdl = b2k::pdl_enabled();
  const dim3 g((unsigned)grid), b(kThreads);
  if (vec && cols4 <= kThreads * 1) b2k::launch_kernel(pdl, softmax_rows_vec<1, Sink>, g, b, 0, s, x, sink, cols4, ld_x);
  else if (vec && cols4 <= kThreads * 2) b2k::launch_kernel(pdl, softmax_rows_vec<2, Sink>, g, b, 0, s, x, sink, cols4, ld_x);
  else if (vec && cols4 <= kThreads * 4) b2k::launch_kernel(pdl, softmax_rows_vec<4, Sink>, g, b, 0, s, x, sink, cols4, ld_x);
  else if (vec && cols4 <= kThreads * 8) b2k::launch_kernel(pdl, softmax_rows_vec<8, Sink>, g, b, 0, s, x, sink, cols4, ld_x);
  else if (vec && cols4 <= kThreads * 16) b2k::launch_kernel(pdl, softmax_rows_vec<16, Sink>, g, b, 0, s, x, sink, cols4, ld_x);
  else b2k::launch_kernel(pdl, softmax_rows_generic<Sink>, g, b, 0, s, x, sink, cols, ld_x);
}

__global__ void selective_exp_kernel(const float *__restrict__ x, float *__restrict__ y, int64_t n) {
  grid_dependency_wait();
  grid_dependents_launch();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) y[i] = b2k_exp(x[i]);
}

}  // namespace

extern "C" int b2k_row_softmax_f32(b2k_ctx *ctx, const float *x, float *y, int64_t rows, int64_t cols,
                                   int64_t ld_x, int64_t ld_y, void *stream) {
  B2K_CHECK_CTX(ctx);
  if (rows < 0 || cols < 0) return b2k::fail(ctx, B2K_EINVAL, "row_softmax: negative extent");
  if (rows == 0 || cols == 0) return B2K_OK;
  if (!x || !y) return b2k::fail(ctx, B2K_EINVAL, "row_softmax: null buffer");
  if (ld_x < cols || ld_y < cols) return b2k::fail(ctx, B2K_EINVAL, "row_softmax: leading dimension < cols");
  if (rows > INT32_MAX) return b2k::fail(ctx, B2K_EINVAL, "row_softmax: too many rows");
  cudaStream_t s = (cudaStream_t)stream;
  const bool vec = (cols % 4 == 0) && (ld_x % 4 == 0) && (ld_y % 4 == 0) && b2k::aligned16(x) && b2k::aligned16(y);
  b2k::PhaseTimer timer(ctx, B2K_PHASE_SOFTMAX, s);
  launch_rows(x, PlainSink{y, ld_y}, rows, cols, ld_x, vec, s);
  return b2k::check_launch(ctx, "row_softmax launch");
}

namespace b2k {

// Row softmax whose output is written as the TF32 hi/lo split [rows][kp]
// (zero padded), ready to be the A operand of the 3xTF32 GEMM.
int softmax_split_rows(b2k_ctx *ctx, const float *x, int64_t rows, int64_t cols, int64_t ld_x, float *hi,
                       float *lo, int64_t kp, cudaStream_t s) {
  if (rows > INT32_MAX) return fail(ctx, B2K_EINVAL, "softmax_split: too many rows");
  const bool vec = (cols % 4 == 0) && (ld_x % 4 == 0) && aligned16(x) && aligned16(hi) && aligned16(lo);
  launch_rows(x, SplitSink{hi, lo, kp}, rows, cols, ld_x, vec, s);
  return check_launch(ctx, "softmax_split launch");
}

}  // namespace b2k

extern "C" int b2k_selective_exp_f32(b2k_ctx *ctx, const float *x, float *y, int64_t n, void *stream) {
  B2K_CHECK_CTX(ctx);
  if (n < 0) return b2k::fail(ctx, B2K_EINVAL, "selective_exp: negative extent");
  if (n == 0) return B2K_OK;
  if (!x || !y) return b2k::fail(ctx, B2K_EINVAL, "selective_exp: null buffer");
  const int64_t blocks = (n + 255) / 256;
  if (blocks > INT32_MAX) return b2k::fail(ctx, B2K_EINVAL, "selective_exp: extent too large");
  b2k::launch_kernel(b2k::pdl_enabled(), selective_exp_kernel, dim3((unsigned)blocks), dim3(256), 0,
                     (cudaStream_t)stream, x, y, n);
  return b2k::check_launch(ctx, "selective_exp launch");
}
