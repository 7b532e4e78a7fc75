// Pipelined host-array entry points: copy in, compute and copy out as one
// call, in slabs, with both copy directions and the kernels overlapped.
//
// The reference's runner does one launch request as three serial steps --
// cuMemcpyHtoD of every input, cuLaunchKernel, cuMemcpyDtoH of every output
// (tools/local_runner.py:287-338) -- so the host link idles while the GPU
// computes and the GPU idles while the link moves data.  Here the inputs are
// cut into slabs along an axis the operation is independent over (rows of
// the softmax, elements of a pointwise program, rows of A for the GEMM,
// batch*heads of attention).  Slab i is copied in on the context's
// host-to-device stream; the caller's stream waits for it (event) and runs
// the slab's kernels; the device-to-host stream waits for those and copies
// slab i's output out while slab i+1 computes and slab i+2 is copied in.
// The host link is full duplex and the B200 has copy engines per direction
// (measured on the B200 box: 55 GB/s one way, 42 GB/s each way when both
// run), so the call costs about the link time of its bytes plus one slab of
// compute and copy-out, instead of the sum of copy-in, compute and copy-out.
//
// The GEMM's slab kernels run round-robin on three context-owned compute
// streams: a slab of 256 rows of A is only a few dozen tiles, so one slab's
// kernel alone would leave most SMs idle.  Measured on B200, the 4096^3
// host-array GEMM then takes 2.99 ms against 2.79 ms for the same copies
// with no kernels at all: the call is bound by the host link.
//
// Device memory for the staged operands is a context-owned arena; the split
// operands of the GEMM use the context workspace as the device entry points
// do.  Every call is ordered after earlier work on the caller's stream (the
// copy streams wait for an event recorded there) and the caller's stream
// waits for the last copy-out, so the host results are complete once the
// caller's stream is synchronised -- the same contract as the device
// entry points.  Host buffers should be page-locked (b2k_host_alloc); with
// pageable memory the copies are correct but partly synchronous.
#include <algorithm>

#include "common.cuh"

namespace b2k {

namespace {

constexpr size_t kAlign = 256;
constexpr int kMaxSlabs = 32;
// Target input bytes per slab, per operation, measured on B200 (4 / 8 / 16 /
// 32 MB tried): small GEMM slabs shorten the exposed last slab (the compute
// of 256 rows of A and their copy-out); attention wants slabs of at least
// six heads of 2048 queries (96 CTAs) per launch; the streaming kernels are
// flat between 8 and 16 MB.
constexpr size_t kSlabStream = size_t(8) << 20;
constexpr size_t kSlabAttention = size_t(16) << 20;
// GEMM slabs of A: a sixteenth of A, but no less than 2 MB and no more than
// 4 MB (then at most kMaxSlabs of them). Measured end to end on B200 with 1,
// 2 and 4 MB slabs: 4097 x 1000 x 777 (A 12.7 MB) took 0.545, 0.495 and
// 0.546 ms (7 slabs of 2 MB best); 4096^3 (A 64 MB) took 3.08, 3.07 and
// 2.98 ms (16 slabs of 4 MB best: more slabs add per-slab launch and event
// overhead that the shorter last slab does not pay back).
size_t gemm_slab_target(size_t a_bytes) {
  return std::min(size_t(4) << 20, std::max(size_t(2) << 20, a_bytes / 16));
}

size_t round_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Slabs of about `target` bytes for `total_in` input bytes, at least 1, at
// most min(kMaxSlabs, units).
int64_t slab_count(size_t total_in, int64_t units, size_t target) {
  const int64_t s = (int64_t)((total_in + target - 1) / target);
  return std::max<int64_t>(1, std::min<int64_t>({s, (int64_t)kMaxSlabs, units}));
}

int reserve_staging(b2k_ctx *ctx, size_t bytes, cudaStream_t s) {
  if (bytes <= ctx->staging_bytes) return B2K_OK;
  // Earlier calls may still read the old arena on any of the three streams;
  // their last copy-out is ordered before the caller's stream.
  cudaError_t err = cudaStreamSynchronize(s);
  if (err != cudaSuccess) return cuda_fail(ctx, err, "staging: stream sync");
  if (ctx->staging) {
    err = cudaFree(ctx->staging);
    ctx->staging = nullptr;
    ctx->staging_bytes = 0;
    if (err != cudaSuccess) return cuda_fail(ctx, err, "staging: cudaFree");
  }
  const size_t rounded = round_up(bytes, size_t(1) << 21);
  err = cudaMalloc(&ctx->staging, rounded);
  if (err != cudaSuccess) {
    ctx->staging = nullptr;
    return cuda_fail(ctx, err, "staging: cudaMalloc");
  }
  ctx->staging_bytes = rounded;
  return B2K_OK;
}

// Carves 256-byte aligned device buffers out of the staging arena.
struct Carve {
  size_t used = 0;
  size_t take(size_t bytes) {
    const size_t off = used;
    used += round_up(std::max<size_t>(bytes, 1), kAlign);
    return off;
  }
};

// The copy streams and dependency events of one pipelined call.
class Pipe {
 public:
  Pipe(b2k_ctx *ctx, cudaStream_t s) : ctx_(ctx), s_(s) {}

  int begin() {
    if (!ctx_->copy_in) {
      cudaError_t err = cudaStreamCreateWithFlags(&ctx_->copy_in, cudaStreamNonBlocking);
      if (err == cudaSuccess) err = cudaStreamCreateWithFlags(&ctx_->copy_out, cudaStreamNonBlocking);
      if (err != cudaSuccess) return cuda_fail(ctx_, err, "pipeline: stream creation");
    }
    cudaEvent_t entry = nullptr;
    int status = mark(s_, &entry);
    if (status == B2K_OK) status = wait(ctx_->copy_in, entry);
    if (status == B2K_OK) status = wait(ctx_->copy_out, entry);
    return status;
  }

  // host -> device on the copy-in stream: `rows` rows of `width` bytes.
  int in(void *dst, size_t dpitch, const void *src, size_t spitch, size_t width, size_t rows) {
    return copy(dst, dpitch, src, spitch, width, rows, cudaMemcpyHostToDevice, ctx_->copy_in);
  }
  int out(void *dst, size_t dpitch, const void *src, size_t spitch, size_t width, size_t rows) {
    return copy(dst, dpitch, src, spitch, width, rows, cudaMemcpyDeviceToHost, ctx_->copy_out);
  }

  // The compute stream waits for everything copied in so far.
  int landed() { return landed_on(s_); }
  // The copy-out stream waits for everything computed so far.
  int computed() { return computed_on(s_); }
  // The same for one of the context's compute streams (compute_stream).
  int landed_on(cudaStream_t st) {
    cudaEvent_t e = nullptr;
    int status = mark(ctx_->copy_in, &e);
    return status == B2K_OK ? wait(st, e) : status;
  }
  int computed_on(cudaStream_t st) {
    cudaEvent_t e = nullptr;
    int status = mark(st, &e);
    return status == B2K_OK ? wait(ctx_->copy_out, e) : status;
  }
  // Compute stream i, created on first use; it waits for everything issued
  // so far on the caller's stream (the call's earlier kernels).
  int compute_stream(int i, cudaStream_t *out) {
    cudaStream_t &st = ctx_->compute[i];
    if (!st) {
      cudaError_t err = cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking);
      if (err != cudaSuccess) return cuda_fail(ctx_, err, "pipeline: compute stream creation");
    }
    cudaEvent_t e = nullptr;
    int status = mark(s_, &e);
    if (status == B2K_OK) status = wait(st, e);
    *out = st;
    return status;
  }
  // The caller's stream waits for the last copy-out.
  int end() {
    cudaEvent_t e = nullptr;
    int status = mark(ctx_->copy_out, &e);
    return status == B2K_OK ? wait(s_, e) : status;
  }

 private:
  int copy(void *dst, size_t dpitch, const void *src, size_t spitch, size_t width, size_t rows, cudaMemcpyKind kind,
           cudaStream_t st) {
    if (!width || !rows) return B2K_OK;
    cudaError_t err = (dpitch == width && spitch == width) || rows == 1
                          ? cudaMemcpyAsync(dst, src, width * rows, kind, st)
                          : cudaMemcpy2DAsync(dst, dpitch, src, spitch, width, rows, kind, st);
    if (err != cudaSuccess) return cuda_fail(ctx_, err, "pipeline: copy");
    return B2K_OK;
  }
  // Events are reused across calls: a wait binds to the record made before it.
  int mark(cudaStream_t st, cudaEvent_t *out) {
    if (next_ == ctx_->sync_events.size()) {
      cudaEvent_t e = nullptr;
      cudaError_t err = cudaEventCreateWithFlags(&e, cudaEventDisableTiming);
      if (err != cudaSuccess) return cuda_fail(ctx_, err, "pipeline: event creation");
      ctx_->sync_events.push_back(e);
    }
    *out = ctx_->sync_events[next_++];
    cudaError_t err = cudaEventRecord(*out, st);
    if (err != cudaSuccess) return cuda_fail(ctx_, err, "pipeline: event record");
    return B2K_OK;
  }
  int wait(cudaStream_t st, cudaEvent_t e) {
    cudaError_t err = cudaStreamWaitEvent(st, e, 0);
    if (err != cudaSuccess) return cuda_fail(ctx_, err, "pipeline: stream wait");
    return B2K_OK;
  }

  b2k_ctx *ctx_;
  cudaStream_t s_;
  size_t next_ = 0;
};

#define B2K_TRY(expr)                        \
  do {                                       \
    int b2k_try_ = (expr);                   \
    if (b2k_try_ != B2K_OK) return b2k_try_; \
  } while (0)

}  // namespace

}  // namespace b2k

extern "C" {

int b2k_row_softmax_f32_host(b2k_ctx *ctx, const float *x, float *y, int64_t rows, int64_t cols, int64_t ld_x,
                             int64_t ld_y, void *stream) {
  B2K_CHECK_CTX(ctx);
  if (rows < 0 || cols < 0) return b2k::fail(ctx, B2K_EINVAL, "row_softmax_host: negative extent");
  if (rows == 0 || cols == 0) return B2K_OK;
  if (!x || !y) return b2k::fail(ctx, B2K_EINVAL, "row_softmax_host: null buffer");
  if (ld_x < cols || ld_y < cols) return b2k::fail(ctx, B2K_EINVAL, "row_softmax_host: leading dimension < cols");
  cudaStream_t s = (cudaStream_t)stream;
  const size_t row_bytes = (size_t)cols * 4;
  b2k::Carve carve;
  const size_t ox = carve.take(row_bytes * rows), oy = carve.take(row_bytes * rows);
  B2K_TRY(b2k::reserve_staging(ctx, carve.used, s));
  char *base = static_cast<char *>(ctx->staging);
  float *dx = reinterpret_cast<float *>(base + ox), *dy = reinterpret_cast<float *>(base + oy);
  const int64_t slabs = b2k::slab_count(row_bytes * rows, rows, b2k::kSlabStream);
  const int64_t per = (rows + slabs - 1) / slabs;
  b2k::Pipe pipe(ctx, s);
  B2K_TRY(pipe.begin());
  for (int64_t r0 = 0; r0 < rows; r0 += per) {
    const int64_t nr = std::min(per, rows - r0);
    B2K_TRY(pipe.in(dx + r0 * cols, row_bytes, x + r0 * ld_x, (size_t)ld_x * 4, row_bytes, nr));
    B2K_TRY(pipe.landed());
    B2K_TRY(b2k_row_softmax_f32(ctx, dx + r0 * cols, dy + r0 * cols, nr, cols, cols, cols, stream));
    B2K_TRY(pipe.computed());
    B2K_TRY(pipe.out(y + r0 * ld_y, (size_t)ld_y * 4, dy + r0 * cols, row_bytes, row_bytes, nr));
  }
  return pipe.end();
}

int b2k_pointwise_f32_host(b2k_ctx *ctx, const b2k_pw_program *program, const float *const *inputs, float *out,
                           int64_t n, void *stream) {
  B2K_CHECK_CTX(ctx);
  if (!program || (program->n_inputs > 0 && !inputs) || !out)
    return b2k::fail(ctx, B2K_EINVAL, "pointwise_host: null argument");
  if (program->n_inputs < 0 || program->n_inputs > B2K_PW_MAX_INPUTS)
    return b2k::fail(ctx, B2K_EINVAL, "pointwise_host: bad input count");
  if (n < 0) return b2k::fail(ctx, B2K_EINVAL, "pointwise_host: negative extent");
  if (n == 0) return B2K_OK;
  for (int i = 0; i < program->n_inputs; ++i)
    if (!inputs[i]) return b2k::fail(ctx, B2K_EINVAL, "pointwise_host: null input %d", i);
  for (int i = 0; i < program->n_inputs; ++i)
    if (!program->broadcast[i] && program->offset[i] < 0)
      return b2k::fail(ctx, B2K_EINVAL, "pointwise_host: input %d has a negative offset", i);
  cudaStream_t s = (cudaStream_t)stream;
  const int ni = program->n_inputs;
  // Shifted windows are applied on the host side: each stream's slab is
  // copied from its shifted start into compact device staging, and the
  // device program reads the staging at offset 0.
  b2k_pw_program staged = *program;
  const float *src[B2K_PW_MAX_INPUTS] = {};
  for (int i = 0; i < ni; ++i) {
    src[i] = program->broadcast[i] ? inputs[i] : inputs[i] + program->offset[i];
    staged.offset[i] = 0;
  }
  b2k::Carve carve;
  size_t off_in[B2K_PW_MAX_INPUTS];
  size_t streamed = 0;
  for (int i = 0; i < ni; ++i) {
    const bool scalar = program->broadcast[i] != 0;
    off_in[i] = carve.take(scalar ? 4 : (size_t)n * 4);
    if (!scalar) streamed += (size_t)n * 4;
  }
  const size_t off_out = carve.take((size_t)n * 4);
  B2K_TRY(b2k::reserve_staging(ctx, carve.used, s));
  char *base = static_cast<char *>(ctx->staging);
  // Slabs of a multiple of 1024 elements keep every slab 16-byte aligned.
  const int64_t slabs =
      b2k::slab_count(std::max<size_t>(streamed, (size_t)n * 4), (n + 1023) / 1024, b2k::kSlabStream);
  const int64_t per = ((n + slabs - 1) / slabs + 1023) / 1024 * 1024;
  b2k::Pipe pipe(ctx, s);
  B2K_TRY(pipe.begin());
  for (int i = 0; i < ni; ++i)
    if (program->broadcast[i]) B2K_TRY(pipe.in(base + off_in[i], 4, src[i], 4, 4, 1));
  for (int64_t e0 = 0; e0 < n; e0 += per) {
    const int64_t ne = std::min(per, n - e0);
    const float *dev_in[B2K_PW_MAX_INPUTS];
    for (int i = 0; i < ni; ++i) {
      float *d = reinterpret_cast<float *>(base + off_in[i]);
      if (program->broadcast[i]) {
        dev_in[i] = d;
      } else {
        B2K_TRY(pipe.in(d + e0, (size_t)ne * 4, src[i] + e0, (size_t)ne * 4, (size_t)ne * 4, 1));
        dev_in[i] = d + e0;
      }
    }
    B2K_TRY(pipe.landed());
    float *dout = reinterpret_cast<float *>(base + off_out) + e0;
    B2K_TRY(b2k_pointwise_f32(ctx, &staged, dev_in, dout, ne, stream));
    B2K_TRY(pipe.computed());
    B2K_TRY(pipe.out(out + e0, (size_t)ne * 4, dout, (size_t)ne * 4, (size_t)ne * 4, 1));
  }
  return pipe.end();
}

int b2k_gemm_tf32x3_host(b2k_ctx *ctx, const float *a, const float *b, float *c, int64_t m, int64_t n, int64_t k,
                         int64_t lda, int64_t ldb, int64_t ldc, int32_t b_layout, const float *bias, int32_t relu,
                         void *stream) {
  B2K_CHECK_CTX(ctx);
  if (m < 0 || n < 0 || k < 0) return b2k::fail(ctx, B2K_EINVAL, "gemm_host: negative extent");
  if (b_layout != B2K_B_KN && b_layout != B2K_B_NK) return b2k::fail(ctx, B2K_EINVAL, "gemm_host: bad b_layout");
  if (m == 0 || n == 0) return B2K_OK;
  if (!a || !b || !c) return b2k::fail(ctx, B2K_EINVAL, "gemm_host: null buffer");
  const bool b_nk = b_layout == B2K_B_NK;
  if (lda < k || ldc < n || ldb < (b_nk ? k : n))
    return b2k::fail(ctx, B2K_EINVAL, "gemm_host: leading dimension too small");
  cudaStream_t s = (cudaStream_t)stream;
  // Device copies are compact: A [m][k], B [k][n] or [n][k], C [m][n].
  const int64_t b_rows = b_nk ? n : k, b_cols = b_nk ? k : n;
  b2k::Carve carve;
  const size_t oa = carve.take((size_t)m * k * 4), ob = carve.take((size_t)b_rows * b_cols * 4);
  const size_t oc = carve.take((size_t)m * n * 4), obias = carve.take(bias ? (size_t)n * 4 : 4);
  B2K_TRY(b2k::reserve_staging(ctx, carve.used, s));
  char *base = static_cast<char *>(ctx->staging);
  float *da = reinterpret_cast<float *>(base + oa), *db = reinterpret_cast<float *>(base + ob);
  float *dc = reinterpret_cast<float *>(base + oc);
  const float *dbias = bias ? reinterpret_cast<float *>(base + obias) : nullptr;
  // Slabs of rows of A (multiples of the 128-row tile).
  const size_t a_bytes = (size_t)m * k * 4;
  const int64_t slabs = b2k::slab_count(a_bytes, (m + 127) / 128, b2k::gemm_slab_target(a_bytes));
  const int64_t per = ((m + slabs - 1) / slabs + 127) / 128 * 128;
  b2k::Pipe pipe(ctx, s);
  // The kernel is chosen for the whole call's m, as b2k_gemm_tf32x3 chooses
  // it, so that the result equals the device entry point's bit for bit.
  // (slab calls run concurrently on three streams and share no partial
  // arena, so the chunk split is not among the choices here)
  const int mode = k == 0 ? 0 : b2k::gemm_split_mode(da, db, m, n, k, k, b_cols, b_layout, ctx->sm_count, false);
  if (k == 0) {
    // No split operands to share between slabs: each slab is a whole GEMM.
    B2K_TRY(pipe.begin());
    B2K_TRY(pipe.in(db, (size_t)b_cols * 4, b, (size_t)ldb * 4, (size_t)b_cols * 4, b_rows));
    if (bias) B2K_TRY(pipe.in(const_cast<float *>(dbias), 4, bias, 4, (size_t)n * 4, 1));
    for (int64_t r0 = 0; r0 < m; r0 += per) {
      const int64_t nr = std::min(per, m - r0);
      B2K_TRY(pipe.in(da + r0 * k, (size_t)k * 4, a + r0 * lda, (size_t)lda * 4, (size_t)k * 4, nr));
      B2K_TRY(pipe.landed());
      B2K_TRY(b2k_gemm_tf32x3(ctx, da + r0 * k, db, dc + r0 * n, nr, n, k, k, b_cols, n, b_layout, dbias, relu, stream));
      B2K_TRY(pipe.computed());
      B2K_TRY(pipe.out(c + r0 * ldc, (size_t)ldc * 4, dc + r0 * n, (size_t)n * 4, (size_t)n * 4, nr));
    }
    return pipe.end();
  }
  const int64_t kp = b2k::gemm_kpad(k);
  if (mode == b2k::kSplitTransposed) {
    // B is read raw by the kernel (split into TMEM); each slab splits its rows
    // of A into the workspace.  The tile width is the whole call's.
    const int bn = b2k::gemm_transposed_tile_width(m, n, ctx->sm_count);
    // one split region for A's slab per compute stream
    constexpr int kStreams = b2k_ctx::kComputeStreams;
    B2K_TRY(b2k::reserve_workspace(ctx, (size_t)(kStreams * 2 * per * kp) * 4, s));
    float *ws = static_cast<float *>(ctx->workspace);
    B2K_TRY(pipe.begin());
    cudaStream_t cs[kStreams];
    for (int i = 0; i < kStreams; ++i) B2K_TRY(pipe.compute_stream(i, &cs[i]));
    B2K_TRY(pipe.in(db, (size_t)b_cols * 4, b, (size_t)ldb * 4, (size_t)b_cols * 4, b_rows));
    if (bias) B2K_TRY(pipe.in(const_cast<float *>(dbias), 4, bias, 4, (size_t)n * 4, 1));
    int slab = 0;
    for (int64_t r0 = 0; r0 < m; r0 += per, ++slab) {
      const int64_t nr = std::min(per, m - r0);
      const int i = slab % kStreams;
      float *wi = ws + (int64_t)i * 2 * per * kp;
      b2k::SplitOperands ops{nullptr, nullptr, wi, wi + per * kp, kp};
      B2K_TRY(pipe.in(da + r0 * k, (size_t)k * 4, a + r0 * lda, (size_t)lda * 4, (size_t)k * 4, nr));
      B2K_TRY(pipe.landed_on(cs[i]));
      {
        b2k::PhaseTimer timer(ctx, B2K_PHASE_SPLIT, cs[i]);
        B2K_TRY(b2k::split_rows(ctx, da + r0 * k, nr, k, k, nr * k, 1, kp, ops.b_hi, ops.b_lo, cs[i]));
      }
      B2K_TRY(b2k::gemm_tmem_b(ctx, db, k, b_cols, b_nk, ops, dc + r0 * n, nr, n, n, dbias, relu, cs[i], bn));
      B2K_TRY(pipe.computed_on(cs[i]));
      B2K_TRY(pipe.out(c + r0 * ldc, (size_t)ldc * 4, dc + r0 * n, (size_t)n * 4, (size_t)n * 4, nr));
    }
    return pipe.end();
  }
  // B is split once into the workspace; each slab then splits its rows of A
  // (pre-pass path) or reads them raw (A split into TMEM inside the kernel).
  const bool tmem_a = mode == b2k::kSplitDirect;
  // B's split once, then one split region for A's slab per compute stream
  // (pre-pass path); the slab GEMMs run round-robin on the compute streams.
  constexpr int kStreams = b2k_ctx::kComputeStreams;
  B2K_TRY(b2k::reserve_workspace(ctx, (size_t)(2 * n * kp + (tmem_a ? 0 : kStreams * 2 * per * kp)) * 4, s));
  float *ws = static_cast<float *>(ctx->workspace);
  float *b_hi = ws, *b_lo = ws + n * kp;
  B2K_TRY(pipe.begin());
  B2K_TRY(pipe.in(db, (size_t)b_cols * 4, b, (size_t)ldb * 4, (size_t)b_cols * 4, b_rows));
  if (bias) B2K_TRY(pipe.in(const_cast<float *>(dbias), 4, bias, 4, (size_t)n * 4, 1));
  B2K_TRY(pipe.landed());
  {
    b2k::PhaseTimer timer(ctx, B2K_PHASE_SPLIT, s);
    B2K_TRY(b_nk ? b2k::split_rows(ctx, db, n, k, k, n * k, 1, kp, b_hi, b_lo, s)
                 : b2k::split_transpose(ctx, db, k, n, n, k * n, 1, kp, b_hi, b_lo, s));
  }
  // the compute streams start after B's split
  cudaStream_t cs[kStreams];
  for (int i = 0; i < kStreams; ++i) B2K_TRY(pipe.compute_stream(i, &cs[i]));
  int slab = 0;
  for (int64_t r0 = 0; r0 < m; r0 += per, ++slab) {
    const int64_t nr = std::min(per, m - r0);
    const int i = slab % kStreams;
    float *wi = ws + 2 * n * kp + (int64_t)i * 2 * per * kp;
    b2k::SplitOperands ops{wi, wi + per * kp, b_hi, b_lo, kp};
    B2K_TRY(pipe.in(da + r0 * k, (size_t)k * 4, a + r0 * lda, (size_t)lda * 4, (size_t)k * 4, nr));
    B2K_TRY(pipe.landed_on(cs[i]));
    if (tmem_a) {
      B2K_TRY(b2k::gemm_tmem_a(ctx, da + r0 * k, k, k, ops, dc + r0 * n, nr, n, n, dbias, relu, cs[i]));
    } else {
      {
        b2k::PhaseTimer timer(ctx, B2K_PHASE_SPLIT, cs[i]);
        B2K_TRY(b2k::split_rows(ctx, da + r0 * k, nr, k, k, nr * k, 1, kp, ops.a_hi, ops.a_lo, cs[i]));
      }
      B2K_TRY(b2k::gemm_main(ctx, ops, nr, n, 1, dc + r0 * n, n, nr * n, dbias, relu, nullptr, 1.0f, cs[i]));
    }
    B2K_TRY(pipe.computed_on(cs[i]));
    B2K_TRY(pipe.out(c + r0 * ldc, (size_t)ldc * 4, dc + r0 * n, (size_t)n * 4, (size_t)n * 4, nr));
  }
  return pipe.end();
}

int b2k_attention_tf32x3_host(b2k_ctx *ctx, const float *q, const float *k, const float *v, float *o, int64_t bh,
                              int64_t s_q, int64_t s_kv, int64_t d, int64_t dv, float scale_div, int32_t k_layout,
                              void *stream) {
  B2K_CHECK_CTX(ctx);
  if (bh < 0 || s_q < 0 || s_kv < 0 || d < 0 || dv < 0)
    return b2k::fail(ctx, B2K_EINVAL, "attention_host: negative extent");
  if (bh == 0 || s_q == 0 || dv == 0) return B2K_OK;
  if (!q || !k || !v || !o) return b2k::fail(ctx, B2K_EINVAL, "attention_host: null buffer");
  cudaStream_t s = (cudaStream_t)stream;
  // Per head: Q [s_q][d], K [s_kv][d] (or [d][s_kv]), V [s_kv][dv], O [s_q][dv].
  const size_t hq = (size_t)s_q * d, hk = (size_t)s_kv * d, hv = (size_t)s_kv * dv, ho = (size_t)s_q * dv;
  b2k::Carve carve;
  const size_t oq = carve.take(hq * bh * 4), ok = carve.take(hk * bh * 4);
  const size_t ov = carve.take(hv * bh * 4), oo = carve.take(ho * bh * 4);
  B2K_TRY(b2k::reserve_staging(ctx, carve.used, s));
  char *base = static_cast<char *>(ctx->staging);
  float *dq = reinterpret_cast<float *>(base + oq), *dk = reinterpret_cast<float *>(base + ok);
  float *dvv = reinterpret_cast<float *>(base + ov), *dout = reinterpret_cast<float *>(base + oo);
  const int64_t slabs = b2k::slab_count((hq + hk + hv) * bh * 4, bh, b2k::kSlabAttention);
  const int64_t per = (bh + slabs - 1) / slabs;
  b2k::Pipe pipe(ctx, s);
  B2K_TRY(pipe.begin());
  for (int64_t h0 = 0; h0 < bh; h0 += per) {
    const int64_t nh = std::min(per, bh - h0);
    B2K_TRY(pipe.in(dq + h0 * hq, hq * nh * 4, q + h0 * hq, hq * nh * 4, hq * nh * 4, 1));
    B2K_TRY(pipe.in(dk + h0 * hk, hk * nh * 4, k + h0 * hk, hk * nh * 4, hk * nh * 4, 1));
    B2K_TRY(pipe.in(dvv + h0 * hv, hv * nh * 4, v + h0 * hv, hv * nh * 4, hv * nh * 4, 1));
    B2K_TRY(pipe.landed());
    B2K_TRY(b2k_attention_tf32x3(ctx, dq + h0 * hq, dk + h0 * hk, dvv + h0 * hv, dout + h0 * ho, nh, s_q, s_kv, d,
                                 dv, scale_div, nullptr, k_layout, stream));
    B2K_TRY(pipe.computed());
    B2K_TRY(pipe.out(o + h0 * ho, ho * nh * 4, dout + h0 * ho, ho * nh * 4, ho * nh * 4, 1));
  }
  return pipe.end();
}

}  // extern "C"
