// Context management and memory helpers of the C ABI (include/b200k.h).
#include <new>

#include "common.cuh"

namespace b2k {

// Grow one of the context's arenas to at least `bytes` (2 MiB granules).
// An arena is reused by every call on this context's stream order; wait for
// in-flight users before releasing the old one.
static int grow_arena(b2k_ctx *ctx, void **arena, size_t *arena_bytes, size_t bytes, cudaStream_t stream,
                      const char *name) {
  if (bytes <= *arena_bytes) return B2K_OK;
  if (ctx->fixed_scratch) return fail(ctx, B2K_ESCRATCH, "%s: this entry point allocates nothing", name);
  cudaError_t err = cudaStreamSynchronize(stream);
  if (err != cudaSuccess) return fail(ctx, B2K_ECUDA, "%s: stream sync: %s", name, cudaGetErrorName(err));
  if (*arena) {
    err = cudaFree(*arena);
    *arena = nullptr;
    *arena_bytes = 0;
    if (err != cudaSuccess) return fail(ctx, B2K_ECUDA, "%s: cudaFree: %s", name, cudaGetErrorName(err));
  }
  const size_t rounded = (bytes + (size_t(1) << 21) - 1) & ~((size_t(1) << 21) - 1);
  err = cudaMalloc(arena, rounded);
  if (err != cudaSuccess) {
    *arena = nullptr;
    return fail(ctx, B2K_ECUDA, "%s: cudaMalloc: %s", name, cudaGetErrorName(err));
  }
  *arena_bytes = rounded;
  return B2K_OK;
}

int reserve_workspace(b2k_ctx *ctx, size_t bytes, cudaStream_t stream) {
  return grow_arena(ctx, &ctx->workspace, &ctx->workspace_bytes, bytes, stream, "workspace");
}

int reserve_partials(b2k_ctx *ctx, size_t bytes, cudaStream_t stream) {
  return grow_arena(ctx, &ctx->partials, &ctx->partials_bytes, bytes, stream, "partials");
}

static cudaEvent_t take_event(b2k_ctx *ctx) {
  if (!ctx->event_pool.empty()) {
    cudaEvent_t e = ctx->event_pool.back();
    ctx->event_pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
  return e;
}

static bool g_pdl = true;
bool pdl_enabled() { return g_pdl; }

PhaseTimer::PhaseTimer(b2k_ctx *ctx, int phase, cudaStream_t stream) : ctx_(ctx), phase_(phase), stream_(stream) {
  if (!ctx_->timing || !((ctx_->timing_mask >> phase) & 1u)) return;
  start_ = take_event(ctx_);
  if (start_) cudaEventRecord(start_, stream_);
}

PhaseTimer::~PhaseTimer() {
  if (!start_) return;
  cudaEvent_t stop = take_event(ctx_);
  if (!stop) {
    ctx_->event_pool.push_back(start_);
    return;
  }
  cudaEventRecord(stop, stream_);
  ctx_->phase_events[phase_].emplace_back(start_, stop);
}

}  // namespace b2k

extern "C" {

int b2k_timing_enable(b2k_ctx *ctx, int on) {
  if (!ctx) return B2K_EINVAL;
  ctx->timing = on != 0;
  return B2K_OK;
}

int b2k_timing_select(b2k_ctx *ctx, uint32_t phase_mask) {
  if (!ctx) return B2K_EINVAL;
  ctx->timing_mask = phase_mask;
  return B2K_OK;
}

int b2k_set_pdl(int on) {
  b2k::g_pdl = on != 0;
  return B2K_OK;
}

int b2k_timing_read(b2k_ctx *ctx, int phase, double *total_ms, int64_t *launches) {
  if (!ctx || phase < 0 || phase >= B2K_PHASE_COUNT || !total_ms || !launches) return B2K_EINVAL;
  double sum = 0.0;
  for (auto &pair : ctx->phase_events[phase]) {
    cudaError_t err = cudaEventSynchronize(pair.second);
    if (err != cudaSuccess) return b2k::cuda_fail(ctx, err, "timing: event sync");
    float ms = 0.0f;
    err = cudaEventElapsedTime(&ms, pair.first, pair.second);
    if (err != cudaSuccess) return b2k::cuda_fail(ctx, err, "timing: elapsed");
    sum += ms;
  }
  *total_ms = sum;
  *launches = (int64_t)ctx->phase_events[phase].size();
  return B2K_OK;
}

int b2k_kernel_launches(b2k_ctx *ctx, int64_t *count) {
  if (!ctx || !count) return B2K_EINVAL;
  *count = ctx->kernel_launches;
  return B2K_OK;
}

int b2k_timing_reset(b2k_ctx *ctx) {
  if (!ctx) return B2K_EINVAL;
  for (auto &list : ctx->phase_events) {
    for (auto &pair : list) {
      cudaEventSynchronize(pair.second);
      ctx->event_pool.push_back(pair.first);
      ctx->event_pool.push_back(pair.second);
    }
    list.clear();
  }
  return B2K_OK;
}

int b2k_version(void) { return 100; }

int b2k_init(int device_ordinal, b2k_ctx **out) {
  if (!out) return B2K_EINVAL;
  *out = nullptr;
  int count = 0;
  cudaError_t err = cudaGetDeviceCount(&count);
  if (err != cudaSuccess) return B2K_ECUDA;
  if (device_ordinal < 0 || device_ordinal >= count) return B2K_EINVAL;
  b2k_ctx *ctx = new (std::nothrow) b2k_ctx;
  if (!ctx) return B2K_ECUDA;
  ctx->device = device_ordinal;
  if ((err = cudaSetDevice(device_ordinal)) != cudaSuccess ||
      (err = cudaDeviceGetAttribute(&ctx->sm_count, cudaDevAttrMultiProcessorCount, device_ordinal)) !=
          cudaSuccess ||
      (err = cudaDeviceGetAttribute(&ctx->max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin,
                                    device_ordinal)) != cudaSuccess) {
    delete ctx;
    return B2K_ECUDA;
  }
  int major = 0, minor = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device_ordinal);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device_ordinal);
  if (major != 10 || minor != 0) {
    // The fatbin holds sm_100a code only; any other device cannot run it.
    delete ctx;
    return B2K_EUNSUPPORTED;
  }
  err = cudaMalloc(&ctx->error_flag, sizeof(unsigned int) * 4);
  if (err == cudaSuccess) err = cudaMemset(ctx->error_flag, 0, sizeof(unsigned int) * 4);
  if (err != cudaSuccess) {
    delete ctx;
    return B2K_ECUDA;
  }
  *out = ctx;
  return B2K_OK;
}

int b2k_destroy(b2k_ctx *ctx) {
  if (!ctx) return B2K_EINVAL;
  cudaSetDevice(ctx->device);
  b2k_timing_reset(ctx);
  for (cudaEvent_t e : ctx->event_pool) cudaEventDestroy(e);
  if (ctx->copy_in) cudaStreamSynchronize(ctx->copy_in);
  if (ctx->copy_out) cudaStreamSynchronize(ctx->copy_out);
  for (cudaEvent_t e : ctx->sync_events) cudaEventDestroy(e);
  for (cudaStream_t st : ctx->compute)
    if (st) cudaStreamSynchronize(st);
  for (cudaStream_t st : ctx->compute)
    if (st) cudaStreamDestroy(st);
  if (ctx->copy_in) cudaStreamDestroy(ctx->copy_in);
  if (ctx->copy_out) cudaStreamDestroy(ctx->copy_out);
  if (ctx->staging) cudaFree(ctx->staging);
  if (ctx->workspace) cudaFree(ctx->workspace);
  if (ctx->partials) cudaFree(ctx->partials);
  if (ctx->error_flag) cudaFree(ctx->error_flag);
  delete ctx;
  return B2K_OK;
}

const char *b2k_last_error(const b2k_ctx *ctx) { return ctx ? ctx->error.c_str() : "null context"; }

int b2k_sm_count(const b2k_ctx *ctx) { return ctx ? ctx->sm_count : 0; }

int b2k_malloc(b2k_ctx *ctx, void **ptr, size_t bytes) {
  B2K_CHECK_CTX(ctx);
  if (!ptr) return b2k::fail(ctx, B2K_EINVAL, "b2k_malloc: null output pointer");
  cudaError_t err = cudaMalloc(ptr, bytes ? bytes : 1);
  if (err != cudaSuccess) return b2k::cuda_fail(ctx, err, "cudaMalloc");
  return B2K_OK;
}

int b2k_free(b2k_ctx *ctx, void *ptr) {
  B2K_CHECK_CTX(ctx);
  cudaError_t err = cudaFree(ptr);
  if (err != cudaSuccess) return b2k::cuda_fail(ctx, err, "cudaFree");
  return B2K_OK;
}

int b2k_host_alloc(b2k_ctx *ctx, void **ptr, size_t bytes) {
  B2K_CHECK_CTX(ctx);
  if (!ptr) return b2k::fail(ctx, B2K_EINVAL, "b2k_host_alloc: null output pointer");
  cudaError_t err = cudaMallocHost(ptr, bytes ? bytes : 1);
  if (err != cudaSuccess) return b2k::cuda_fail(ctx, err, "cudaMallocHost");
  return B2K_OK;
}

int b2k_host_free(b2k_ctx *ctx, void *ptr) {
  B2K_CHECK_CTX(ctx);
  cudaError_t err = cudaFreeHost(ptr);
  if (err != cudaSuccess) return b2k::cuda_fail(ctx, err, "cudaFreeHost");
  return B2K_OK;
}

int b2k_memcpy_htod(b2k_ctx *ctx, void *dst, const void *src, size_t bytes, void *stream) {
  B2K_CHECK_CTX(ctx);
  cudaError_t err = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, (cudaStream_t)stream);
  if (err != cudaSuccess) return b2k::cuda_fail(ctx, err, "cudaMemcpyAsync(HtoD)");
  return B2K_OK;
}

int b2k_memcpy_dtoh(b2k_ctx *ctx, void *dst, const void *src, size_t bytes, void *stream) {
  B2K_CHECK_CTX(ctx);
  cudaError_t err = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, (cudaStream_t)stream);
  if (err != cudaSuccess) return b2k::cuda_fail(ctx, err, "cudaMemcpyAsync(DtoH)");
  return B2K_OK;
}

int b2k_memset(b2k_ctx *ctx, void *dst, int value, size_t bytes, void *stream) {
  B2K_CHECK_CTX(ctx);
  cudaError_t err = cudaMemsetAsync(dst, value, bytes, (cudaStream_t)stream);
  if (err != cudaSuccess) return b2k::cuda_fail(ctx, err, "cudaMemsetAsync");
  return B2K_OK;
}

int b2k_stream_sync(b2k_ctx *ctx, void *stream) {
  B2K_CHECK_CTX(ctx);
  cudaError_t err = cudaStreamSynchronize((cudaStream_t)stream);
  if (err != cudaSuccess) return b2k::cuda_fail(ctx, err, "cudaStreamSynchronize");
  unsigned int flag = 0;
  err = cudaMemcpy(&flag, ctx->error_flag, sizeof flag, cudaMemcpyDeviceToHost);
  if (err != cudaSuccess) return b2k::cuda_fail(ctx, err, "error flag readback");
  if (flag) {
    cudaMemset(ctx->error_flag, 0, sizeof(unsigned int) * 4);
    return b2k::fail(ctx, B2K_ETIMEOUT, "a kernel's bounded wait expired (code 0x%x)", flag);
  }
  return B2K_OK;
}

}  // extern "C"
