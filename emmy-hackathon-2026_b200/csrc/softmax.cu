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

// VPT float4 chunks per thread; the row (cols4 = cols/4 chunks) must satisfy
// cols4 <= kThreads * VPT.  Rows are 16-byte aligned.
template <int VPT>
__global__ void __launch_bounds__(kThreads) softmax_rows_vec(const float *__restrict__ x, float *__restrict__ y,
                                                             int64_t cols4, int64_t ldx, int64_t ldy) {
  __shared__ float red_max[kWarps];
  __shared__ float red_sum[kWarps];
  const int64_t row = blockIdx.x;
  const float4 *xr = reinterpret_cast<const float4 *>(x + row * ldx);
  float4 *yr = reinterpret_cast<float4 *>(y + row * ldy);
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
      st_stream(yr + c, o);
    }
  }
}

// Any row length / alignment: three passes over the row (max, exp-sum,
// normalise) with scalar coalesced accesses; later passes hit L2 for rows
// that fit there.
__global__ void __launch_bounds__(kThreads) softmax_rows_generic(const float *__restrict__ x, float *__restrict__ y,
                                                                 int64_t cols, int64_t ldx, int64_t ldy) {
  __shared__ float red_max[kWarps];
  __shared__ float red_sum[kWarps];
  const int64_t row = blockIdx.x;
  const float *xr = x + row * ldx;
  float *yr = y + row * ldy;
  float m = -INFINITY;
  for (int64_t c = threadIdx.x; c < cols; c += kThreads) m = fmaxf(m, __ldg(xr + c));
  m = block_max(m, red_max);
  float s = 0.0f;
  for (int64_t c = threadIdx.x; c < cols; c += kThreads) s += b2k_exp(__fsub_rn(__ldg(xr + c), m));
  s = block_sum(s, red_sum);
  const float r = __frcp_rn(s);
  for (int64_t c = threadIdx.x; c < cols; c += kThreads) yr[c] = __fmul_rn(b2k_exp(__fsub_rn(__ldg(xr + c), m)), r);
}

__global__ void selective_exp_kernel(const float *__restrict__ x, float *__restrict__ y, int64_t n) {
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
  const int64_t cols4 = cols / 4;
  const int grid = (int)rows;
  b2k::PhaseTimer timer(ctx, B2K_PHASE_SOFTMAX, s);
  if (vec && cols4 <= kThreads * 1) softmax_rows_vec<1><<<grid, kThreads, 0, s>>>(x, y, cols4, ld_x, ld_y);
  else if (vec && cols4 <= kThreads * 2) softmax_rows_vec<2><<<grid, kThreads, 0, s>>>(x, y, cols4, ld_x, ld_y);
  else if (vec && cols4 <= kThreads * 4) softmax_rows_vec<4><<<grid, kThreads, 0, s>>>(x, y, cols4, ld_x, ld_y);
  else if (vec && cols4 <= kThreads * 8) softmax_rows_vec<8><<<grid, kThreads, 0, s>>>(x, y, cols4, ld_x, ld_y);
  else if (vec && cols4 <= kThreads * 16) softmax_rows_vec<16><<<grid, kThreads, 0, s>>>(x, y, cols4, ld_x, ld_y);
  else softmax_rows_generic<<<grid, kThreads, 0, s>>>(x, y, cols, ld_x, ld_y);
  return b2k::check_launch(ctx, "row_softmax launch");
}

extern "C" int b2k_selective_exp_f32(b2k_ctx *ctx, const float *x, float *y, int64_t n, void *stream) {
  B2K_CHECK_CTX(ctx);
  if (n < 0) return b2k::fail(ctx, B2K_EINVAL, "selective_exp: negative extent");
  if (n == 0) return B2K_OK;
  if (!x || !y) return b2k::fail(ctx, B2K_EINVAL, "selective_exp: null buffer");
  const int64_t blocks = (n + 255) / 256;
  if (blocks > INT32_MAX) return b2k::fail(ctx, B2K_EINVAL, "selective_exp: extent too large");
  selective_exp_kernel<<<(int)blocks, 256, 0, (cudaStream_t)stream>>>(x, y, n);
  return b2k::check_launch(ctx, "selective_exp launch");
}
