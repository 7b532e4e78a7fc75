// Pointwise FP32 programs: 16-byte vectorised streaming kernels.
//
// The reference lowers a pointwise Tile per thread to 2-4 adjacent elements
// with v4 loads/stores behind a runtime alignment predicate
// (compile.py:1425-1600 access_descriptors, 5865-5942 vector groups,
// 8586-8661 Write).  Here one thread owns UNROLL float4 chunks per pass; the
// arithmetic is either a compiled-in binary operation (the common
// `c = a op b` programs, including the n=2^24 add) or a small interpreted
// straight-line program for everything else.  Both are HBM-bound.
#include "common.cuh"

namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 4;  // float4 chunks in flight per thread

struct PwParams {
  b2k_pw_program prog;
  const float *in[B2K_PW_MAX_INPUTS];
  float *out;
  int64_t n;
};

__device__ __forceinline__ float apply(int op, float a, float b, float c, float imm) {
  switch (op) {
    case B2K_OP_CONST: return imm;
    case B2K_OP_COPY: return a;
    case B2K_OP_ADD: return __fadd_rn(a, b);
    case B2K_OP_SUB: return __fsub_rn(a, b);
    case B2K_OP_MUL: return __fmul_rn(a, b);
    case B2K_OP_DIV: return __fdiv_rn(a, b);
    case B2K_OP_MAX: return fmaxf(a, b);
    case B2K_OP_MIN: return fminf(a, b);
    case B2K_OP_NEG: return -a;
    case B2K_OP_RCP: return __frcp_rn(a);
    case B2K_OP_SQRT: return __fsqrt_rn(a);
    case B2K_OP_RSQRT: return __frcp_rn(__fsqrt_rn(a));
    case B2K_OP_EXP: return b2k_exp(a);
    case B2K_OP_RELU: return a > 0.0f ? a : 0.0f;
    case B2K_OP_ABS: return fabsf(a);
    case B2K_OP_FMA: return __fmaf_rn(a, b, c);
    case B2K_OP_GT: return a > b ? 1.0f : 0.0f;
    case B2K_OP_GE: return a >= b ? 1.0f : 0.0f;
    case B2K_OP_LT: return a < b ? 1.0f : 0.0f;
    case B2K_OP_LE: return a <= b ? 1.0f : 0.0f;
    case B2K_OP_WHERE: return a != 0.0f ? b : c;
    case B2K_OP_LOG: {
      float r;
      asm("lg2.approx.f32 %0, %1;" : "=f"(r) : "f"(a));
      return __fmul_rn(r, 0.693147182464599609375f);  // f32(ln 2)
    }
    default: return __int_as_float(0x7fffffff);
  }
}

// Evaluate the program on one element; registers live in local memory
// (indexed by the program), which is acceptable for the rare programs that
// miss the compiled-in fast paths.
__device__ __forceinline__ float run_program(const b2k_pw_program &p, const float *inputs) {
  float reg[B2K_PW_MAX_REGS];
  for (int i = 0; i < p.n_inputs; ++i) reg[i] = inputs[i];
  for (int i = 0; i < p.n_insns; ++i) {
    const b2k_pw_insn &ins = p.insns[i];
    const float a = reg[ins.a], b = reg[ins.b], c = reg[ins.c];
    reg[p.n_inputs + i] = apply(ins.op, a, b, c, ins.imm);
  }
  return reg[p.result];
}

__global__ void __launch_bounds__(kThreads) pw_program_vec4(const __grid_constant__ PwParams p) {
  grid_dependency_wait();
  grid_dependents_launch();
  const int64_t n4 = p.n >> 2;
  const int64_t base = (int64_t)blockIdx.x * kThreads * kUnroll + threadIdx.x;
  float scalars[B2K_PW_MAX_INPUTS];
  for (int i = 0; i < p.prog.n_inputs; ++i) scalars[i] = p.prog.broadcast[i] ? __ldg(p.in[i]) : 0.0f;
#pragma unroll 1
  for (int u = 0; u < kUnroll; ++u) {
    const int64_t chunk = base + (int64_t)u * kThreads;
    if (chunk >= n4) break;
    float4 lanes[B2K_PW_MAX_INPUTS];
    for (int i = 0; i < p.prog.n_inputs; ++i)
      lanes[i] = p.prog.broadcast[i] ? make_float4(scalars[i], scalars[i], scalars[i], scalars[i])
                                     : ld_stream(reinterpret_cast<const float4 *>(p.in[i]) + chunk);
    float4 result;
    float values[B2K_PW_MAX_INPUTS];
    for (int i = 0; i < p.prog.n_inputs; ++i) values[i] = lanes[i].x;
    result.x = run_program(p.prog, values);
    for (int i = 0; i < p.prog.n_inputs; ++i) values[i] = lanes[i].y;
    result.y = run_program(p.prog, values);
    for (int i = 0; i < p.prog.n_inputs; ++i) values[i] = lanes[i].z;
    result.z = run_program(p.prog, values);
    for (int i = 0; i < p.prog.n_inputs; ++i) values[i] = lanes[i].w;
    result.w = run_program(p.prog, values);
    st_stream(reinterpret_cast<float4 *>(p.out) + chunk, result);
  }
}

// Scalar path: unaligned streams and the (n mod 4) tail of the vector path.
__global__ void __launch_bounds__(kThreads) pw_program_scalar(const __grid_constant__ PwParams p,
                                                              int64_t start) {
  grid_dependency_wait();
  grid_dependents_launch();
  const int64_t i = start + (int64_t)blockIdx.x * kThreads + threadIdx.x;
  if (i >= p.n) return;
  float values[B2K_PW_MAX_INPUTS];
  for (int k = 0; k < p.prog.n_inputs; ++k) values[k] = p.prog.broadcast[k] ? __ldg(p.in[k]) : __ldg(p.in[k] + i);
  p.out[i] = run_program(p.prog, values);
}

// Compiled-in binary operation of two streams (either may be a broadcast
// scalar): the fast path for `c[i] = a[i] op b[i]`.
template <int OP, bool BA, bool BB>
__global__ void __launch_bounds__(kThreads) pw_binary_vec4(const float *__restrict__ a,
                                                           const float *__restrict__ b,
                                                           float *__restrict__ out, int64_t n4) {
  grid_dependency_wait();
  grid_dependents_launch();
  const int64_t base = (int64_t)blockIdx.x * kThreads * kUnroll + threadIdx.x;
  const float sa = BA ? __ldg(a) : 0.0f, sb = BB ? __ldg(b) : 0.0f;
  float4 va[kUnroll], vb[kUnroll];
#pragma unroll
  for (int u = 0; u < kUnroll; ++u) {
    const int64_t chunk = base + (int64_t)u * kThreads;
    if (chunk < n4) {
      va[u] = BA ? make_float4(sa, sa, sa, sa) : ld_stream(reinterpret_cast<const float4 *>(a) + chunk);
      vb[u] = BB ? make_float4(sb, sb, sb, sb) : ld_stream(reinterpret_cast<const float4 *>(b) + chunk);
    }
  }
#pragma unroll
  for (int u = 0; u < kUnroll; ++u) {
    const int64_t chunk = base + (int64_t)u * kThreads;
    if (chunk < n4) {
      float4 r;
      r.x = apply(OP, va[u].x, vb[u].x, 0.0f, 0.0f);
      r.y = apply(OP, va[u].y, vb[u].y, 0.0f, 0.0f);
      r.z = apply(OP, va[u].z, vb[u].z, 0.0f, 0.0f);
      r.w = apply(OP, va[u].w, vb[u].w, 0.0f, 0.0f);
      st_stream(reinterpret_cast<float4 *>(out) + chunk, r);
    }
  }
}

template <int OP>
void launch_binary(bool ba, bool bb, const float *a, const float *b, float *out, int64_t n4, int blocks,
                   cudaStream_t s) {
  // programmatic dependent launch: back-to-back launches hide each other's
  // launch latency and tail (each kernel waits for its predecessor first)
  const bool pdl = b2k::pdl_enabled();
  if (ba && bb) b2k::launch_kernel(pdl, pw_binary_vec4<OP, true, true>, dim3(blocks), dim3(kThreads), 0, s, a, b, out, n4);
  else if (ba) b2k::launch_kernel(pdl, pw_binary_vec4<OP, true, false>, dim3(blocks), dim3(kThreads), 0, s, a, b, out, n4);
  else if (bb) b2k::launch_kernel(pdl, pw_binary_vec4<OP, false, true>, dim3(blocks), dim3(kThreads), 0, s, a, b, out, n4);
  else b2k::launch_kernel(pdl, pw_binary_vec4<OP, false, false>, dim3(blocks), dim3(kThreads), 0, s, a, b, out, n4);
}

bool launch_binary_fast(const b2k_pw_program &p, const float *const *in, float *out, int64_t n4, int blocks,
                        cudaStream_t s) {
  if (p.n_insns != 1 || p.result != p.n_inputs) return false;
  const b2k_pw_insn &ins = p.insns[0];
  if (ins.a >= p.n_inputs || ins.b >= p.n_inputs) return false;
  const bool ba = p.broadcast[ins.a] != 0, bb = p.broadcast[ins.b] != 0;
  const float *a = in[ins.a], *b = in[ins.b];
  switch (ins.op) {
    case B2K_OP_ADD: launch_binary<B2K_OP_ADD>(ba, bb, a, b, out, n4, blocks, s); return true;
    case B2K_OP_SUB: launch_binary<B2K_OP_SUB>(ba, bb, a, b, out, n4, blocks, s); return true;
    case B2K_OP_MUL: launch_binary<B2K_OP_MUL>(ba, bb, a, b, out, n4, blocks, s); return true;
    case B2K_OP_DIV: launch_binary<B2K_OP_DIV>(ba, bb, a, b, out, n4, blocks, s); return true;
    case B2K_OP_MAX: launch_binary<B2K_OP_MAX>(ba, bb, a, b, out, n4, blocks, s); return true;
    case B2K_OP_MIN: launch_binary<B2K_OP_MIN>(ba, bb, a, b, out, n4, blocks, s); return true;
    default: return false;
  }
}

int validate_program(b2k_ctx *ctx, const b2k_pw_program *p) {
  if (!p) return b2k::fail(ctx, B2K_EINVAL, "pointwise: null program");
  if (p->n_inputs < 0 || p->n_inputs > B2K_PW_MAX_INPUTS)
    return b2k::fail(ctx, B2K_EINVAL, "pointwise: n_inputs %d outside [0, %d]", p->n_inputs, B2K_PW_MAX_INPUTS);
  if (p->n_insns < 0 || p->n_insns > B2K_PW_MAX_INSNS)
    return b2k::fail(ctx, B2K_EINVAL, "pointwise: n_insns %d outside [0, %d]", p->n_insns, B2K_PW_MAX_INSNS);
  const int regs = p->n_inputs + p->n_insns;
  if (p->result < 0 || p->result >= regs)
    return b2k::fail(ctx, B2K_EINVAL, "pointwise: result register %d undefined", p->result);
  for (int i = 0; i < p->n_insns; ++i) {
    const b2k_pw_insn &ins = p->insns[i];
    const int defined = p->n_inputs + i;  // registers readable by instruction i
    if (ins.op < 0 || ins.op >= B2K_OP_COUNT)
      return b2k::fail(ctx, B2K_EINVAL, "pointwise: instruction %d has opcode %d", i, ins.op);
    if (ins.a < 0 || ins.a >= defined || ins.b < 0 || ins.b >= defined || ins.c < 0 || ins.c >= defined) {
      if (!(ins.op == B2K_OP_CONST && defined == 0))
        return b2k::fail(ctx, B2K_EINVAL, "pointwise: instruction %d reads an undefined register", i);
    }
  }
  return B2K_OK;
}

}  // namespace

extern "C" int b2k_pointwise_f32(b2k_ctx *ctx, const b2k_pw_program *program, const float *const *inputs,
                                 float *out, int64_t n, void *stream) {
  B2K_CHECK_CTX(ctx);
  int status = validate_program(ctx, program);
  if (status != B2K_OK) return status;
  if (n < 0) return b2k::fail(ctx, B2K_EINVAL, "pointwise: negative extent");
  if (n == 0) return B2K_OK;
  if (!out || (program->n_inputs && !inputs)) return b2k::fail(ctx, B2K_EINVAL, "pointwise: null buffer");
  PwParams params;
  params.prog = *program;
  params.out = out;
  params.n = n;
  bool vector_ok = b2k::aligned16(out);
  // Each stream's first element: its base, shifted by the program's offset.
  const float *in[B2K_PW_MAX_INPUTS] = {};
  for (int i = 0; i < B2K_PW_MAX_INPUTS; ++i) params.in[i] = nullptr;
  for (int i = 0; i < program->n_inputs; ++i) {
    if (!inputs[i]) return b2k::fail(ctx, B2K_EINVAL, "pointwise: input %d is null", i);
    if (!program->broadcast[i] && program->offset[i] < 0)
      return b2k::fail(ctx, B2K_EINVAL, "pointwise: input %d has a negative offset", i);
    in[i] = program->broadcast[i] ? inputs[i] : inputs[i] + program->offset[i];
    params.in[i] = in[i];
    if (!program->broadcast[i]) vector_ok = vector_ok && b2k::aligned16(in[i]);
  }
  cudaStream_t s = (cudaStream_t)stream;
  b2k::PhaseTimer timer(ctx, B2K_PHASE_POINTWISE, s);
  int64_t done = 0;
  int launches = 0;
  if (vector_ok && n >= 4) {
    const int64_t n4 = n >> 2;
    const int64_t per_block = (int64_t)kThreads * kUnroll;
    const int64_t blocks = (n4 + per_block - 1) / per_block;
    if (blocks > INT32_MAX) return b2k::fail(ctx, B2K_EINVAL, "pointwise: extent too large");
    if (!launch_binary_fast(*program, in, out, n4, (int)blocks, s))
      b2k::launch_kernel(b2k::pdl_enabled(), pw_program_vec4, dim3((unsigned)blocks), dim3(kThreads), 0, s, params);
    done = n4 << 2;
    ++launches;
  }
  if (done < n) {
    const int64_t rest = n - done;
    const int64_t blocks = (rest + kThreads - 1) / kThreads;
    if (blocks > INT32_MAX) return b2k::fail(ctx, B2K_EINVAL, "pointwise: extent too large");
    b2k::launch_kernel(b2k::pdl_enabled(), pw_program_scalar, dim3((unsigned)blocks), dim3(kThreads), 0, s, params,
                       done);
    ++launches;
  }
  return b2k::check_launch(ctx, "pointwise launch", launches);
}
