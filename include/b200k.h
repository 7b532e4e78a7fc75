/*
 * b200k.h -- C ABI of the B200 (sm_100a) kernel backend for Emmy Kernel IR.
 *
 * The reference compiler turns each recognised Kernel-IR kernel into PTX text
 * (compile.py:9628-9724 compile_path) which a runner assembles and launches
 * with cuLaunchKernel, passing positional arguments in meta.json's arg_order
 * (tools/local_runner.py:246-342, launch at :309-324).  This library replaces
 * that emitted PTX: a front end recognises the kernel and calls one of the
 * entry points below with the same device buffers.
 *
 * Conventions shared by every entry point:
 *   - Plain C types only: device pointers, 64-bit extents, a cudaStream_t
 *     passed as void* (NULL = the legacy default stream).
 *   - The caller owns every buffer; the library only reads inputs and writes
 *     outputs.  Scratch memory (the GEMM's TF32 operand split) belongs to the
 *     context and is reused across calls.
 *   - Return value: B2K_OK, a positive validation code (nothing was
 *     launched), or a negative device-side code.  b2k_last_error() gives a
 *     human-readable reason.
 *   - A context is not thread-safe: use one per (host thread, device).
 */
#ifndef B200K_H
#define B200K_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define B2K_OK 0
#define B2K_EINVAL 1       /* invalid argument; nothing launched */
#define B2K_EUNSUPPORTED 2 /* valid request outside this build's kernels */
#define B2K_ECUDA (-1)     /* CUDA runtime/driver error */
#define B2K_ETIMEOUT (-2)  /* a device-side bounded wait expired (kernel error flag) */
#define B2K_ESCRATCH 3     /* problem needs more than the fixed no-alloc scratch array */
#define B2K_ENCCL (-3)     /* NCCL error; the multi-GPU handle is aborted and must be destroyed */

typedef struct b2k_ctx b2k_ctx;

/* ABI version of this header (major*100 + minor). */
int b2k_version(void);

/* Create a context on CUDA device `device_ordinal` (makes it current on this
 * thread).  Replaces the runner's per-worker context set-up
 * (tools/local_runner.py:258-280). */
int b2k_init(int device_ordinal, b2k_ctx **out);
int b2k_destroy(b2k_ctx *ctx);
/* Reason for the last non-OK return on this context ("" if none). */
const char *b2k_last_error(const b2k_ctx *ctx);
/* Streaming multiprocessor count of the context's device. */
int b2k_sm_count(const b2k_ctx *ctx);

/* --- device memory helpers for callers without their own allocator ------
 * (the runner's cuMemAlloc / cuMemcpyHtoD / cuMemcpyDtoH / cuMemsetD8 calls,
 * tools/local_runner.py:287-300, 320-322, 333-338). */
int b2k_malloc(b2k_ctx *ctx, void **ptr, size_t bytes);
int b2k_free(b2k_ctx *ctx, void *ptr);
int b2k_memcpy_htod(b2k_ctx *ctx, void *dst, const void *src, size_t bytes, void *stream);
int b2k_memcpy_dtoh(b2k_ctx *ctx, void *dst, const void *src, size_t bytes, void *stream);
int b2k_memset(b2k_ctx *ctx, void *dst, int value, size_t bytes, void *stream);
/* Page-locked host memory, so host<->device copies run asynchronously at
 * full PCIe/C2C bandwidth. */
int b2k_host_alloc(b2k_ctx *ctx, void **ptr, size_t bytes);
int b2k_host_free(b2k_ctx *ctx, void *ptr);
int b2k_stream_sync(b2k_ctx *ctx, void *stream);
/* Failure-detection self test: launches one kernel whose mbarrier wait can
 * never complete and gives up after `budget_cycles` SM cycles (at most the
 * kernels' own ~2 s budget), exactly as a stalled tensor-core kernel would.
 * The following b2k_stream_sync returns B2K_ETIMEOUT and clears the device
 * error word; the context stays usable.  No counterpart in the reference
 * (its runner retires a worker process on any CUDA error,
 * tools/local_runner.py:246-342). */
int b2k_selftest_wait_timeout(b2k_ctx *ctx, int64_t budget_cycles, void *stream);

/* --- per-phase timing -------------------------------------------------------
 * When enabled, every entry point brackets the kernels of each of its phases
 * with CUDA events recorded on the caller's stream (the runner's event
 * timing, tools/local_runner.py:318-332, per kernel instead of per launch
 * request).  b2k_timing_read synchronises and sums the recorded intervals of
 * one phase (`launches` = intervals: one per entry-point call of the phase,
 * which may cover more than one kernel); b2k_timing_reset forgets them.
 * b2k_kernel_launches returns how many kernels the context has enqueued
 * since b2k_init (every launch is counted, timing enabled or not). */
#define B2K_PHASE_SPLIT 0     /* 3xTF32 operand split pre-pass */
#define B2K_PHASE_MMA 1       /* tcgen05 GEMM main kernel */
#define B2K_PHASE_POINTWISE 2 /* pointwise programs */
#define B2K_PHASE_SOFTMAX 3   /* row softmax */
#define B2K_PHASE_ATTENTION 4 /* attention (all of its passes) */
#define B2K_PHASE_ROWS 5      /* row reductions / norms */
#define B2K_PHASE_FLASH 6     /* fused attention kernel */
#define B2K_PHASE_COUNT 7
int b2k_timing_enable(b2k_ctx *ctx, int on);
/* Restrict timing to the phases whose bit (1 << B2K_PHASE_*) is set in
 * `phase_mask` (default: all).  Each timed phase costs two event records
 * per call, and an event between two kernels of one call serialises them
 * (see b2k_set_pdl), so a caller timing one kernel should select only its
 * phase. */
int b2k_timing_select(b2k_ctx *ctx, uint32_t phase_mask);
int b2k_timing_read(b2k_ctx *ctx, int phase, double *total_ms, int64_t *launches);
int b2k_timing_reset(b2k_ctx *ctx);
int b2k_kernel_launches(b2k_ctx *ctx, int64_t *count);

/* --- launch overlap -----------------------------------------------------------
 * Process-wide switch (default on): the kernels of a split-then-multiply
 * operation (GEMM, fused attention) are launched with programmatic
 * dependent launch, so the tensor-core kernel's CTAs are scheduled and run
 * their set-up while the split kernel drains, and the next call's split
 * overlaps this call's tail.  Results are identical either way; the switch
 * exists for comparisons.  No counterpart in the reference. */
int b2k_set_pdl(int on);

/* --- pointwise programs ---------------------------------------------------
 * Replaces the SIMT Emitter's pointwise lowering: Tile decode
 * (compile.py:8473-8585), 16-byte vector load/store groups
 * (compile.py:1425-1600, 5865-5942, 8586-8661) and scalar arithmetic
 * (compile.py:2645-2965).  A program is a straight-line list of FP32
 * operations over up to B2K_PW_MAX_INPUTS input streams; register r < n_inputs
 * holds input r's element, later registers hold instruction results. */
#define B2K_PW_MAX_INPUTS 8
#define B2K_PW_MAX_INSNS 48
#define B2K_PW_MAX_REGS (B2K_PW_MAX_INPUTS + B2K_PW_MAX_INSNS)

enum b2k_pw_opcode {
  B2K_OP_CONST = 0,      /* dst = imm */
  B2K_OP_COPY = 1,       /* dst = a */
  B2K_OP_ADD = 2,        /* dst = a + b (round to nearest) */
  B2K_OP_SUB = 3,
  B2K_OP_MUL = 4,
  B2K_OP_DIV = 5,        /* IEEE division, round to nearest */
  B2K_OP_MAX = 6,
  B2K_OP_MIN = 7,
  B2K_OP_NEG = 8,
  B2K_OP_RCP = 9,        /* 1/a, round to nearest */
  B2K_OP_SQRT = 10,      /* round to nearest */
  B2K_OP_RSQRT = 11,     /* 1/sqrt(a) */
  B2K_OP_EXP = 12,       /* selective subnormal-preserving exp (compile.py:2953-2965) */
  B2K_OP_RELU = 13,      /* max(a, 0) */
  B2K_OP_ABS = 14,
  B2K_OP_FMA = 15,       /* dst = a * b + c, single rounding */
  B2K_OP_GT = 16,        /* dst = (a > b) ? 1 : 0 */
  B2K_OP_GE = 17,
  B2K_OP_LT = 18,
  B2K_OP_LE = 19,
  B2K_OP_WHERE = 20,     /* dst = (a != 0) ? b : c */
  B2K_OP_LOG = 21,       /* natural log via lg2.approx * ln2 (compile.py:2938-2942) */
  B2K_OP_COUNT = 22
};

typedef struct b2k_pw_insn {
  int32_t op;       /* enum b2k_pw_opcode */
  int32_t a, b, c;  /* source registers (unused ones ignored) */
  float imm;        /* B2K_OP_CONST value */
} b2k_pw_insn;

typedef struct b2k_pw_program {
  int32_t n_inputs;                        /* input streams, registers 0..n_inputs-1 */
  int32_t n_insns;                         /* instructions; insn i writes register n_inputs+i */
  int32_t result;                          /* register stored to the output */
  int32_t broadcast[B2K_PW_MAX_INPUTS];    /* 1: input is a scalar buffer read at element 0 */
  int32_t offset[B2K_PW_MAX_INPUTS];       /* >= 0: input i is read at element i + offset[i]
                                              (a shifted window; ignored for broadcast inputs) */
  b2k_pw_insn insns[B2K_PW_MAX_INSNS];
} b2k_pw_program;

/* out[i] = program(inputs[0][i + offset[0]], inputs[1][i + offset[1]], ...)
 * for i in [0, n).  Non-broadcast input r must hold n + offset[r] FP32
 * elements, out n; 16-byte vector accesses are used when every stream (its
 * base plus offset) is 16-byte aligned, element accesses otherwise -- the
 * runtime alignment fallback of the reference's vector groups
 * (compile.py:1425-1600, 8586-8661). */
int b2k_pointwise_f32(b2k_ctx *ctx, const b2k_pw_program *program, const float *const *inputs,
                      float *out, int64_t n, void *stream);

/* --- row softmax ----------------------------------------------------------
 * Replaces the Emitter's row-reduction softmax passes: online/two-pass
 * max+sum (compile.py:1656-1711, 6492-6644), warp-shuffle and shared-tree
 * combine (compile.py:8958-9035, 9175-9268), selective exp
 * (compile.py:2953-2965) and the reciprocal-multiply normalisation.
 * y[r, :] = exp(x[r, :] - max_r) / sum_r for a row-major rows x cols matrix
 * with leading dimensions ld_x / ld_y (elements). */
int b2k_row_softmax_f32(b2k_ctx *ctx, const float *x, float *y, int64_t rows, int64_t cols,
                        int64_t ld_x, int64_t ld_y, void *stream);

/* --- row reductions and row norms -------------------------------------------
 * Replaces the Emitter's merged vector row reduction (compile.py:4987-5165,
 * shuffles and trees 8958-9268) and row-map reuse (compile.py:5511-5665) for
 * the reduction / rmsnorm / l2norm kernels:
 *   B2K_ROW_SUM      y[r]    = (sum_c x[r,c]) / div                 (div = *sum_div_ptr or sum_div)
 *   B2K_ROW_RMSNORM  y[r,c]  = x[r,c] * w[c] / sqrt(sum_c x^2 / count + eps)
 *   B2K_ROW_L2NORM   y[r,c]  = x[r,c] * w[c] / sqrt(sum_c x^2 + eps)
 *   B2K_ROW_MAX      y[r]    = max_c x[r,c]    (IEEE maxNum: a NaN loses to a number)
 *   B2K_ROW_MIN      y[r]    = min_c x[r,c]    (IEEE minNum)
 *   B2K_ROW_PROD     y[r]    = prod_c x[r,c]   (FP32 products in a fixed tree order)
 * count = *ms_div_ptr or ms_div, eps = *eps_ptr or eps; w may be NULL (1).
 * A single row longer than 65,536 (a whole-array sum) is reduced by many CTAs
 * and a fixed-order second pass. */
#define B2K_ROW_SUM 0
#define B2K_ROW_RMSNORM 1
#define B2K_ROW_L2NORM 2
#define B2K_ROW_MAX 3
#define B2K_ROW_MIN 4
#define B2K_ROW_PROD 5
typedef struct b2k_row_params {
  int32_t op;
  float sum_div;
  const float *sum_div_ptr;
  float ms_div;
  const float *ms_div_ptr;
  float eps;
  const float *eps_ptr;
  const float *w;
} b2k_row_params;
/* Fold over the middle axis of x [batch][s][cols] (contiguous):
 *   y[b][j] = fold_{i < s} x[b][i][j]      (y [batch][cols], contiguous)
 * op: B2K_ROW_SUM (the sum divided by *div_ptr when non-NULL, else by div:
 * a mean for div = s), B2K_ROW_MAX, B2K_ROW_MIN (IEEE maxNum / minNum) or
 * B2K_ROW_PROD.  Each output folds i = 0, 1, ... in order, as the IR's serial
 * Loop + Accum over that axis (the reference interpreter,
 * tests/test_research_cases.py:103-160).  s = 0 gives the fold's identity. */
int b2k_axis_reduce_f32(b2k_ctx *ctx, int32_t op, const float *x, float *y, int64_t batch, int64_t s, int64_t cols,
                        float div, const float *div_ptr, void *stream);
int b2k_row_op_f32(b2k_ctx *ctx, const b2k_row_params *params, const float *x, float *y, int64_t rows,
                   int64_t cols, int64_t ld_x, int64_t ld_y, void *stream);

/* Elementwise selective exponential (compile.py:2953-2965); exposed for the
 * subnormal-range accuracy tests. */
int b2k_selective_exp_f32(b2k_ctx *ctx, const float *x, float *y, int64_t n, void *stream);

/* --- 3xTF32 GEMM -----------------------------------------------------------
 * Replaces the reference's dense-contraction back ends: the 3xTF32
 * mma.sync emitter tf32_emitter.production_ptx (tf32_emitter.py:291-710,
 * arithmetic model :22-96) and the exact-FP32 SIMT plan emitter
 * compile.plan_simt_ptx (compile.py:9326-9611) selected for proven plans
 * (compile.py:9614-9625, tensor_core.py MatmulPlan :232-330).
 *
 * C[m, n] = relu?(A[m, k] * B + bias[n]) with every product expanded as
 * hi*hi + hi*lo + lo*hi of TF32 halves and FP32 accumulation.
 * A is row-major with leading dimension lda.  b_layout B2K_B_KN: B is
 * row-major [k, n] (ldb >= n); B2K_B_NK: B is stored transposed, row-major
 * [n, k] (ldb >= k).  Or-ing B2K_A_KM into b_layout says A is stored
 * transposed, row-major [k, m] (lda >= m; the pre-pass split transposes it;
 * not accepted by the host-array and batched calls).  bias may be NULL; relu
 * is 0 or 1.  C is row-major (ldc >= n).  Uses 2 * (m + n) * round_up(k, 32)
 * * 4 bytes of context scratch for the split operands, and, when the call
 * takes the K-chunk split (b2k_gemm_set_chunk_split, b2k_gemm_plan), a
 * second context arena of chunks * m * round_up(n, 4) * 4 bytes (chunks =
 * round_up(k, 32) / 256 rounded up) for the chunks' raw accumulators.  Both
 * arenas grow on first need (a synchronising cudaMalloc) and are then
 * reused. */
#define B2K_B_KN 0
#define B2K_B_NK 1
#define B2K_A_KM 2
int b2k_gemm_tf32x3(b2k_ctx *ctx, const float *a, const float *b, float *c, int64_t m, int64_t n, int64_t k,
                    int64_t lda, int64_t ldb, int64_t ldc, int32_t b_layout, const float *bias, int32_t relu,
                    void *stream);

/* b2k_gemm_tf32x3 with the product divided before the epilogue:
 *   C = relu?((A B) / div + bias),  div = *div_ptr (a one-element device
 *   buffer, read on the device) when div_ptr is non-NULL, else div_value.
 * The division is FP32 round-to-nearest of each accumulated element, as the
 * IR's `divide` of a contraction result (the scaled-score kernel of an
 * attention pipeline: scores = x @ y / scale[0]).  Takes the pre-pass split
 * path.  K = 0 returns B2K_EUNSUPPORTED. */
int b2k_gemm_tf32x3_scaled(b2k_ctx *ctx, const float *a, const float *b, float *c, int64_t m, int64_t n, int64_t k,
                           int64_t lda, int64_t ldb, int64_t ldc, int32_t b_layout, const float *bias, int32_t relu,
                           const float *div_ptr, float div_value, void *stream);

/* A batch of independent GEMMs with the arithmetic and epilogue of
 * b2k_gemm_tf32x3: C[i] = relu?(A[i] B[i] + bias) for i < batch, A[i] at
 * a + i * stride_a (elements), B[i] at b + i * stride_b, C[i] at
 * c + i * stride_c; bias (optional, n columns) is shared by the batch.  Each
 * stride must cover its matrix (stride_a >= m * lda, ...).  Replaces the
 * batched contractions the reference's tensor-core plan rejects
 * (tensor_core.py:284).  batch <= 65535; takes the pre-pass split path. */
int b2k_gemm_tf32x3_batched(b2k_ctx *ctx, const float *a, const float *b, float *c, int64_t batch, int64_t m,
                            int64_t n, int64_t k, int64_t lda, int64_t ldb, int64_t ldc, int64_t stride_a,
                            int64_t stride_b, int64_t stride_c, int32_t b_layout, const float *bias, int32_t relu,
                            void *stream);

/* --- attention ----------------------------------------------------------------
 * Replaces the reference's fused SIMT attention lowering (compile.py:7009-7966:
 * hoisted score rows, selective-exp softmax, P.V fold) for every head of a
 * batch: O[h] = softmax(Q[h] K[h]^T / scale) V[h] for h < bh, both contractions
 * as 3xTF32 on the tensor cores.  Q is [bh][s_q][d], V is [bh][s_kv][dv], O
 * is [bh][s_q][dv] (all row-major, contiguous).  k_layout B2K_K_SD: K is
 * [bh][s_kv][d]; B2K_K_DS: K is given transposed as [bh][d][s_kv] (the IR's
 * `kt`).  The divisor is *scale_div_ptr when that device pointer is non-NULL
 * (the IR's one-element `div_c1` buffer), else scale_div.  Head dims up to
 * 128 (d and dv) run one fused kernel (S and P never leave the SM); larger
 * ones run three batched passes through context scratch. */
#define B2K_K_SD 0
#define B2K_K_DS 1
int b2k_attention_tf32x3(b2k_ctx *ctx, const float *q, const float *k, const float *v, float *o, int64_t bh,
                         int64_t s_q, int64_t s_kv, int64_t d, int64_t dv, float scale_div,
                         const float *scale_div_ptr, int32_t k_layout, void *stream);
/* Process-wide choice of attention path where head dims allow the fused
 * kernel: 1 (default) the fused kernel with one CTA per query tile; 0 the
 * three-pass path (for comparisons).  Other values return B2K_EINVAL. */
int b2k_attention_set_fused(int mode);

/* --- launch by descriptor ----------------------------------------------------
 * The reference's runner launches a compiled kernel with
 * cuLaunchKernel(fn, grid, block, smem, stream, params, NULL), `params` being
 * pointers to the values of the positional meta.json arguments in arg_order
 * (tools/local_runner.py:296-324; Emitter ABI binding compile.py:1995-2213).
 * b2k_launch takes that same `args` array -- a device-pointer argument's slot
 * points at its 64-bit address, an f32 scalar's slot at its value -- plus a
 * descriptor naming the B200 kernel and which positional arguments feed it.
 * The front end (frontend.py) fills the descriptor when it recognises an IR
 * kernel; meta's grid/block are validated there, not obeyed (the sm_89
 * geometry is not a B200 geometry).  zero_outputs stay with the caller, as in
 * the reference's runner.  Every failure is reported before launching. */
#define B2K_KIND_POINTWISE 1
#define B2K_KIND_ROW_SOFTMAX 2
#define B2K_KIND_ROW_OP 3
#define B2K_KIND_GEMM_3XTF32 4
#define B2K_KIND_ATTENTION_3XTF32 5
#define B2K_KIND_AXIS_REDUCE 6
#define B2K_KIND_GEMM_BATCHED 7
#define B2K_MAX_ROLES 12
#define B2K_NO_ARG (-1)
#define B2K_ROLE_PW_OUT 8
typedef struct b2k_kernel_desc {
  int32_t kind;
  /* Positional argument index of each operand role (B2K_NO_ARG if absent):
   *   POINTWISE   roles 0..n_inputs-1 input streams, B2K_ROLE_PW_OUT output
   *   ROW_SOFTMAX 0 x, 1 y
   *   ROW_OP      0 x, 1 y, 2 weight, 3 sum-divisor buffer,
   *               4 mean-square-divisor buffer, 5 epsilon buffer
   *   GEMM_3XTF32 0 A, 1 B, 2 C, 3 bias, 4 divisor buffer (b2k_gemm_tf32x3_scaled)
   *   ATTENTION   0 Q, 1 K, 2 V, 3 O, 4 divisor buffer
   *   AXIS_REDUCE 0 x, 1 y, 3 divisor buffer
   *   GEMM_BATCHED 0 A, 1 B, 2 C, 3 bias (contiguous [batch][rows][cols] operands) */
  int32_t role[B2K_MAX_ROLES];
  /* POINTWISE: n | ROW_*: rows, cols, ld_x, ld_y | GEMM: m, n, k, lda, ldb, ldc |
   * ATTENTION: bh, s_q, s_kv, d, dv | AXIS_REDUCE: batch, s, cols | GEMM_BATCHED: batch, m, n, k */
  int64_t dims[6];
  /* GEMM, GEMM_BATCHED: b_layout, relu | ATTENTION: k_layout | ROW_OP, AXIS_REDUCE: op */
  int32_t flags[4];
  /* ROW_OP: sum_div, ms_div, eps | ATTENTION: scale_div (when no buffer) |
   * AXIS_REDUCE: sum divisor (when no buffer) */
  float values[4];
  const b2k_pw_program *program; /* POINTWISE */
} b2k_kernel_desc;
int b2k_launch(b2k_ctx *ctx, const b2k_kernel_desc *desc, void *const *args, int32_t nargs, void *stream);

/* The same GEMM for callers that cannot allocate device memory: embedders
 * whose device memory belongs to another allocator or a pre-sized pool,
 * runtimes that plan every buffer up front, and code in a host callback or
 * library hook where a synchronising cudaMalloc is not allowed.  No
 * counterpart in the reference.  It takes no context and
 * allocates nothing: the operand split goes to a fixed scratch array inside
 * the library image (B2K_NOALLOC_SCRATCH_BYTES per device that loads the
 * library, kept until exit).  Problems with 2 * (m + n) * round_up(k, 32) * 4
 * bytes of split operands above that size return B2K_ESCRATCH and launch
 * nothing; extents beyond the 32-bit limits of b2k_gemm_tf32x3 return
 * B2K_EINVAL; K = 0 returns B2K_EUNSUPPORTED.  Runs on the calling thread's
 * current device and the given stream.  The first call on a device looks up
 * the scratch array's device address (cudaGetSymbolAddress) and keeps it;
 * make that first call on each device before any stream capture begins.
 * Every call on a device shares the one
 * array, so calls that overlap on the GPU (different streams, no ordering)
 * race and corrupt each other's results; calls on one stream are safe.  Each
 * call rewrites all the scratch it reads, so nothing needs clearing.  A
 * device-side bounded-wait expiry is not returned by this entry point (its
 * kernels are still running when it returns): the kernels record it in a
 * per-device word that b2k_gemm_noalloc_status reads.
 * Other return codes as b2k_gemm_tf32x3 (B2K_EINVAL, B2K_ECUDA). */
#define B2K_NOALLOC_SCRATCH_BYTES (32u << 20)
int b2k_gemm_tf32x3_noalloc(const float *a, const float *b, float *c, int64_t m, int64_t n, int64_t k,
                            int64_t lda, int64_t ldb, int64_t ldc, int32_t b_layout, const float *bias,
                            int32_t relu, void *stream);

/* Read and clear the device error word of b2k_gemm_tf32x3_noalloc on
 * `device`: B2K_ETIMEOUT when a bounded wait of one of its kernels expired
 * since the last query (the word is then cleared), B2K_OK when none did,
 * B2K_EINVAL for a device index out of range, B2K_ECUDA on a CUDA error.
 * Synchronise the streams of the calls to be checked first; the calling
 * thread's current device is left as it was.  No counterpart in the
 * reference (its runner retires a worker on any CUDA error). */
int b2k_gemm_noalloc_status(int32_t device);

/* --- multi-GPU: one problem over the GPUs of a node -------------------------
 * One process per GPU, each with its own b2k_ctx and one NCCL communicator
 * (NCCL is opened at run time; without it these calls return
 * B2K_EUNSUPPORTED and everything else works).  The reference is single-GPU
 * (tools/local_runner.py:246-342 drives one device); each workload of its hot
 * path splits into independent units, so a call takes this rank's shard of
 * the inputs and returns the whole output on every rank:
 *   shard of `units` for rank r = b2k_mgpu_partition(units, world, r, align):
 *   contiguous, every shard but the last a multiple of `align`, the last
 *   taking the remainder (4097 rows over 8 ranks: seven of 512, one of 513).
 * Collectives run on a stream of the handle's own and overlap the compute on
 * the caller's stream; the caller's stream waits for them at the end of each
 * call.  Calls on one handle are ordered like any other stream work.  Every
 * rank must make the same calls in the same order.  Returns B2K_ENCCL after
 * an NCCL error and B2K_ETIMEOUT when a bounded wait expires; the handle is
 * then aborted and only b2k_mgpu_destroy remains valid. */
typedef struct b2k_mgpu b2k_mgpu;
#define B2K_MGPU_ID_BYTES 128
int b2k_mgpu_partition(int64_t units, int32_t world, int32_t rank, int64_t align, int64_t *start, int64_t *count);
/* Rendezvous token: one rank makes it; the caller hands the 128 bytes to
 * every rank by its own channel (a file, a socket, a process-group broadcast). */
int b2k_mgpu_unique_id(void *id);
/* Join the communicator of `world` ranks as `rank` on ctx's device.  Returns
 * B2K_ETIMEOUT (nothing left behind) if the ranks have not all joined within
 * timeout_ms. */
int b2k_mgpu_init(b2k_ctx *ctx, int32_t world, int32_t rank, const void *id, int64_t timeout_ms, b2k_mgpu **out);
int b2k_mgpu_destroy(b2k_mgpu *mg);
/* Wait for the work issued on `stream` (the calls' collectives included),
 * at most timeout_ms: a collective whose peer has gone (a rank that exited
 * or stopped calling) ends in B2K_ETIMEOUT or B2K_ENCCL, not a hang. */
int b2k_mgpu_sync(b2k_mgpu *mg, void *stream, int64_t timeout_ms);
/* C = relu?(A B + bias) for C [m][n] (row-major, complete on every rank).
 * a_rows: this rank's rows of A, partition(m, world, rank, align), row-major
 * [rows][k] contiguous.  b: B on rank 0 only (other ranks may pass NULL),
 * [k][n] (B2K_B_KN) or [n][k] (B2K_B_NK), contiguous.  bias: [n] on every
 * rank, or NULL.  B is broadcast in `panels` column panels (1..16): panel
 * p's GEMM waits only for panel p, and panel p's C is gathered while panel
 * p + 1 computes; with one panel rank 0 broadcasts from `b` itself (read
 * only, never written).  Replaces a launch of the reference's GEMM plan
 * (tensor_core.py:232-330) by its row-partitioned form. */
int b2k_mgpu_gemm_tf32x3(b2k_mgpu *mg, const float *a_rows, const float *b, float *c, int64_t m, int64_t n,
                         int64_t k, int64_t align, int32_t b_layout, const float *bias, int32_t relu, int32_t panels,
                         void *stream);
/* Row softmax of a [rows][cols] matrix: x_rows is this rank's rows
 * (partition(rows, world, rank, 1)), y the whole output.  The gathers run
 * per piece (1..16; equal shards only, else one piece), piece i while piece
 * i + 1 computes. */
int b2k_mgpu_row_softmax_f32(b2k_mgpu *mg, const float *x_rows, float *y, int64_t rows, int64_t cols,
                             int32_t pieces, void *stream);
/* A pointwise program over n elements: non-broadcast input r holds this
 * rank's elements, partition(n, world, rank, align) (plus offset[r] elements
 * of window), broadcast inputs their one element; out is the whole output. */
int b2k_mgpu_pointwise_f32(b2k_mgpu *mg, const b2k_pw_program *program, const float *const *inputs, float *out,
                           int64_t n, int64_t align, int32_t pieces, void *stream);
/* Attention over bh heads: q, k ([heads][s_kv][d]) and v are this rank's
 * heads, partition(bh, world, rank, 1); o [bh][s_q][dv] the whole output. */
int b2k_mgpu_attention_tf32x3(b2k_mgpu *mg, const float *q, const float *k, const float *v, float *o, int64_t bh,
                              int64_t s_q, int64_t s_kv, int64_t d, int64_t dv, float scale_div, int32_t pieces,
                              void *stream);

/* Select the GEMM kernel variant for subsequent calls (process-wide; for
 * tuning and benchmarking): 0 = 128x256 tile, 128-byte swizzle, 2 stages;
 * 1 (default) = 128x256, 64-byte swizzle, 4 stages, or the tile of variant 3
 * or 2 when its tiles cover the output in clearly less estimated time (fewer
 * waves over the SMs: a row shard of a multi-GPU GEMM); every width gives the
 * same bits; 2 = 128x128, 128-byte
 * swizzle, 3 stages; 3 = 128x192, 64-byte swizzle, 5 stages.  Outputs at
 * most 128 columns wide always use 2.  For the in-kernel split kernels
 * (b2k_gemm_set_fused_split) variant 2 selects 128-wide tiles and every
 * other variant 192-wide ones.  No counterpart in the reference, whose plan
 * geometry comes from the IR. */
int b2k_gemm_set_variant(int variant);

/* Chunk split of the pre-pass GEMM kernel (process-wide; for tuning and
 * tests): 1 (default) = where the estimate says it is faster, 0 = never,
 * 2 = wherever it applies.  It applies to single (not batched) calls with at
 * least two 256-wide K chunks, made through a context: every 128 x 128 output
 * tile is computed as one CTA per K chunk, each storing its chunk's raw
 * accumulator in a context-owned arena, and a second kernel folds the chunks
 * in order and applies the epilogue -- the fold the unsplit kernel makes --
 * so the result is the same bits.  It fills the GPU when the output has few
 * tiles and K is long (a row shard of the ragged GEMM on eight GPUs, a
 * 256 x 512 x 4096 product).  The allocation-free entry point and the
 * host-array calls never take it.  No counterpart in the reference (its
 * split-K variant uses atomics, whose order is not fixed). */
int b2k_gemm_set_chunk_split(int mode);

/* Which kernel path b2k_gemm_tf32x3 takes for a call with these operands on
 * a GPU of `sms` SMs, under the current settings (variant, split modes,
 * chunk split), decided by the dispatch's own functions.  Host arithmetic
 * only: it touches no GPU and dereferences no pointer (a and b are read for
 * their alignment).  A divided product (b2k_gemm_tf32x3_scaled) always takes
 * split mode 0.  B2K_EINVAL for the arguments b2k_gemm_tf32x3 refuses, and
 * for m, n or k of 0 (nothing is launched then). */
typedef struct {
  int32_t split_mode;  /* 0 both operands pre-split, 1 A split in the kernel,
                          2 B split in the kernel (C^T = B^T A^T) */
  int32_t tile_width;  /* the kernel's tile width: output columns, or output
                          rows in mode 2 */
  int32_t chunk_split; /* 1: one CTA per (128 x 128 tile, 256-wide K chunk),
                          then the in-order fold */
  int32_t chunks;      /* 256-wide K chunks of the call */
} b2k_gemm_plan_info;
int b2k_gemm_plan(int32_t sms, const float *a, const float *b, int64_t m, int64_t n, int64_t k, int64_t lda,
                  int64_t ldb, int32_t b_layout, b2k_gemm_plan_info *out);
/* Process-wide choice of where b2k_gemm_tf32x3 (and the no-alloc variant)
 * split operands into TF32 hi/lo halves:
 *   3            direct: A is staged raw by TMA and split inside the
 *                tensor-core kernel into tensor memory, which the MMAs read A
 *                from (128 x 192 tiles, 128 x 128 for n <= 128); B is split
 *                once by a pre-pass.  Needs A 16-byte aligned, not stored
 *                transposed, with a row stride that is a multiple of 4
 *                elements, and K >= 16.
 *   2            transposed: the kernel computes C^T = B^T A^T, so B is staged
 *                raw and split inside the kernel into tensor memory (a [K, N]
 *                B read in 128-column boxes, a [N, K] B by rows) and only A is
 *                split by the pre-pass; the epilogue writes C transposed back
 *                into row-major C.  For short, wide outputs (a row shard of a
 *                large GEMM) it splits the small operand and tiles the output
 *                128 columns by 128 or 192 rows.  Needs B 16-byte aligned with
 *                a row stride that is a multiple of 4 elements, K >= 16 and,
 *                for a [K, N] B, N >= 128.
 *   1 (default)  whichever of 0, 2 and 3 the operands allow and an estimate
 *                of (waves of tiles over the SMs) x (tile time) + (pre-pass
 *                bytes) says is fastest.
 *   0            both operands split by the pre-pass (128 x 256 tiles).
 * Calls whose operands do not meet a mode's conditions take the pre-pass
 * path.  Every path runs the same three TF32 products per 8-wide K step with
 * the same 256-wide chunked FP32 accumulation.  Returns B2K_EINVAL for other
 * values.  No counterpart in the reference. */
int b2k_gemm_set_fused_split(int mode);

/* --- pipelined host-array calls ----------------------------------------------
 * The runner's per-request host flow -- copy every input in, launch, copy
 * every output out (tools/local_runner.py:287-338) -- as one call that
 * overlaps the three.  Arguments are HOST pointers with the meaning of the
 * device entry point of the same name.  Inputs are cut into slabs (rows of
 * the softmax or of A, element ranges, batch*heads); slab i is copied in on
 * a context-owned host-to-device stream, its kernels run on `stream` once it
 * has landed, and its output is copied out on a device-to-host stream while
 * later slabs compute and copy in.  Device staging memory belongs to the
 * context.  Asynchronous like the device entry points: the host outputs are
 * complete once `stream` is synchronised (b2k_stream_sync).  Host buffers
 * should be page-locked (b2k_host_alloc); pageable buffers work with less
 * overlap.  Results equal the device entry points' bit for bit. */
int b2k_row_softmax_f32_host(b2k_ctx *ctx, const float *x, float *y, int64_t rows, int64_t cols, int64_t ld_x,
                             int64_t ld_y, void *stream);
int b2k_pointwise_f32_host(b2k_ctx *ctx, const b2k_pw_program *program, const float *const *inputs, float *out,
                           int64_t n, void *stream);
int b2k_gemm_tf32x3_host(b2k_ctx *ctx, const float *a, const float *b, float *c, int64_t m, int64_t n, int64_t k,
                         int64_t lda, int64_t ldb, int64_t ldc, int32_t b_layout, const float *bias, int32_t relu,
                         void *stream);
/* Host variant of b2k_attention_tf32x3 with the scale divisor by value. */
int b2k_attention_tf32x3_host(b2k_ctx *ctx, const float *q, const float *k, const float *v, float *o, int64_t bh,
                              int64_t s_q, int64_t s_kv, int64_t d, int64_t dv, float scale_div, int32_t k_layout,
                              void *stream);

#ifdef __cplusplus
}
#endif

#endif /* B200K_H */
