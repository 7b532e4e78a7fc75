// b2k_launch: one entry point for every recognised IR kernel, taking the
// runner's positional argument array (the cuLaunchKernel params convention of
// tools/local_runner.py:296-324) and a descriptor that names the kernel and
// maps its operand roles to positional arguments.  Host-side only: it resolves
// the roles, validates them and calls the kind's entry point.
#include "common.cuh"

namespace {

// Resolve `role` to the device address held by its positional argument.
int role_address(b2k_ctx *ctx, const b2k_kernel_desc *d, void *const *args, int32_t nargs, int role, bool required,
                 const void **out) {
  const int32_t idx = d->role[role];
  if (idx == B2K_NO_ARG) {
    if (required) return b2k::fail(ctx, B2K_EINVAL, "launch: kind %d needs role %d", d->kind, role);
    *out = nullptr;
    return B2K_OK;
  }
  if (idx < 0 || idx >= nargs) return b2k::fail(ctx, B2K_EINVAL, "launch: role %d -> argument %d of %d", role, idx, nargs);
  if (!args[idx]) return b2k::fail(ctx, B2K_EINVAL, "launch: argument %d has no value slot", idx);
  *out = reinterpret_cast<const void *>(*static_cast<const uint64_t *>(args[idx]));
  if (required && !*out) return b2k::fail(ctx, B2K_EINVAL, "launch: argument %d is a null buffer", idx);
  return B2K_OK;
}

}  // namespace

extern "C" int b2k_launch(b2k_ctx *ctx, const b2k_kernel_desc *d, void *const *args, int32_t nargs, void *stream) {
  B2K_CHECK_CTX(ctx);
  if (!d) return b2k::fail(ctx, B2K_EINVAL, "launch: null descriptor");
  if (nargs < 0 || (nargs > 0 && !args)) return b2k::fail(ctx, B2K_EINVAL, "launch: bad argument array");
  const void *p[B2K_MAX_ROLES] = {};
  int st = B2K_OK;
  auto need = [&](int role) { if (st == B2K_OK) st = role_address(ctx, d, args, nargs, role, true, &p[role]); };
  auto maybe = [&](int role) { if (st == B2K_OK) st = role_address(ctx, d, args, nargs, role, false, &p[role]); };
  switch (d->kind) {
    case B2K_KIND_POINTWISE: {
      if (!d->program) return b2k::fail(ctx, B2K_EINVAL, "launch: pointwise without a program");
      const int n_in = d->program->n_inputs;
      if (n_in < 1 || n_in > B2K_PW_MAX_INPUTS) return b2k::fail(ctx, B2K_EINVAL, "launch: %d pointwise inputs", n_in);
      for (int i = 0; i < n_in; ++i) need(i);
      need(B2K_ROLE_PW_OUT);
      if (st != B2K_OK) return st;
      const float *in[B2K_PW_MAX_INPUTS] = {};
      for (int i = 0; i < n_in; ++i) in[i] = static_cast<const float *>(p[i]);
      return b2k_pointwise_f32(ctx, d->program, in, (float *)p[B2K_ROLE_PW_OUT], d->dims[0], stream);
    }
    case B2K_KIND_ROW_SOFTMAX:
      need(0), need(1);
      if (st != B2K_OK) return st;
      return b2k_row_softmax_f32(ctx, (const float *)p[0], (float *)p[1], d->dims[0], d->dims[1], d->dims[2],
                                 d->dims[3], stream);
    case B2K_KIND_ROW_OP: {
      need(0), need(1), maybe(2), maybe(3), maybe(4), maybe(5);
      if (st != B2K_OK) return st;
      b2k_row_params rp{d->flags[0], d->values[0], (const float *)p[3], d->values[1], (const float *)p[4],
                        d->values[2], (const float *)p[5], (const float *)p[2]};
      return b2k_row_op_f32(ctx, &rp, (const float *)p[0], (float *)p[1], d->dims[0], d->dims[1], d->dims[2],
                            d->dims[3], stream);
    }
    case B2K_KIND_GEMM_3XTF32:
      need(0), need(1), need(2), maybe(3), maybe(4);
      if (st != B2K_OK) return st;
      if (p[4])  // the product divided by a one-element buffer
        return b2k_gemm_tf32x3_scaled(ctx, (const float *)p[0], (const float *)p[1], (float *)p[2], d->dims[0],
                                      d->dims[1], d->dims[2], d->dims[3], d->dims[4], d->dims[5], d->flags[0],
                                      (const float *)p[3], d->flags[1], (const float *)p[4], 1.0f, stream);
      return b2k_gemm_tf32x3(ctx, (const float *)p[0], (const float *)p[1], (float *)p[2], d->dims[0], d->dims[1],
                             d->dims[2], d->dims[3], d->dims[4], d->dims[5], d->flags[0], (const float *)p[3],
                             d->flags[1], stream);
    case B2K_KIND_GEMM_BATCHED: {
      need(0), need(1), need(2), maybe(3);
      if (st != B2K_OK) return st;
      const int64_t bt = d->dims[0], m = d->dims[1], n = d->dims[2], k = d->dims[3];
      const bool nk = d->flags[0] == B2K_B_NK;
      return b2k_gemm_tf32x3_batched(ctx, (const float *)p[0], (const float *)p[1], (float *)p[2], bt, m, n, k, k,
                                     nk ? k : n, n, m * k, n * k, m * n, d->flags[0], (const float *)p[3],
                                     d->flags[1], stream);
    }
    case B2K_KIND_AXIS_REDUCE:
      need(0), need(1), maybe(3);
      if (st != B2K_OK) return st;
      return b2k_axis_reduce_f32(ctx, d->flags[0], (const float *)p[0], (float *)p[1], d->dims[0], d->dims[1],
                                 d->dims[2], d->values[0], (const float *)p[3], stream);
    case B2K_KIND_ATTENTION_3XTF32:
      need(0), need(1), need(2), need(3), maybe(4);
      if (st != B2K_OK) return st;
      return b2k_attention_tf32x3(ctx, (const float *)p[0], (const float *)p[1], (const float *)p[2], (float *)p[3],
                                  d->dims[0], d->dims[1], d->dims[2], d->dims[3], d->dims[4], d->values[0],
                                  (const float *)p[4], d->flags[0], stream);
    default:
      return b2k::fail(ctx, B2K_EINVAL, "launch: unknown kernel kind %d", d->kind);
  }
}
