// b2k_gemm_tf32x3_noalloc: the 3xTF32 GEMM for callers that cannot allocate
// device memory.
//
// Some callers may not call cudaMalloc at all: embedders whose device memory
// is owned by another allocator or a pre-sized pool, runtimes that plan every
// buffer up front and treat an allocation after start-up as an error, and
// code running inside a host callback or a library hook where a
// device-synchronising call is not allowed.  b2k_gemm_tf32x3 needs a context
// whose scratch arena grows with cudaMalloc; this entry point instead uses a
// fixed scratch array that is part of the library image itself (a file-scope
// __device__ array), so it needs no context and calls no allocator.
//
// The operand split needs 2 * (m + n) * round_up(k, 32) floats of scratch;
// the array holds B2K_NOALLOC_SCRATCH_BYTES (32 MiB), and larger problems are
// rejected with B2K_ESCRATCH before anything is launched.  Every GPU that
// loads the library keeps this array until the process exits.
#include <mutex>

#include "common.cuh"

// The tensor-core GEMM of gemm.cu: splits A and B into `ws` and launches the
// main kernel on `s`.
int b2k_gemm_tf32x3_impl(b2k_ctx *ctx, const float *a, const float *b, float *c, int64_t m, int64_t n, int64_t k,
                         int64_t lda, int64_t ldb, int64_t ldc, int layout, const float *bias, int relu,
                         float *ws, cudaStream_t s, const float *div_ptr, float div_value);

namespace {

constexpr size_t kScratchFloats = B2K_NOALLOC_SCRATCH_BYTES / sizeof(float);
constexpr int kMaxDevices = 64;

// Shared by every call on a device: the split operands of the current call.
static __device__ __align__(256) float g_scratch[kScratchFloats];
// Device-side status word for the kernels' bounded waits.
static __device__ __align__(256) unsigned int g_status[4];

struct DeviceSymbols {
  bool ready = false;
  float *scratch = nullptr;
  unsigned int *status = nullptr;
  int sm_count = 0;
};

DeviceSymbols g_devices[kMaxDevices];
std::mutex g_mutex;

// Host code cannot pass g_scratch itself to a kernel: on the host that name
// is only a stand-in for the device array.  Look up the device addresses once
// per device, with that device current.  The first call of the entry point on
// a device does this set-up, so that first call should come before any
// stream capture begins.
int device_symbols(int device, DeviceSymbols *out) {
  std::lock_guard<std::mutex> lock(g_mutex);
  DeviceSymbols &entry = g_devices[device];
  if (!entry.ready) {
    void *scratch = nullptr, *status = nullptr;
    if (cudaGetSymbolAddress(&scratch, g_scratch) != cudaSuccess) return B2K_ECUDA;
    if (cudaGetSymbolAddress(&status, g_status) != cudaSuccess) return B2K_ECUDA;
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return B2K_ECUDA;
    entry.scratch = static_cast<float *>(scratch);
    entry.status = static_cast<unsigned int *>(status);
    entry.sm_count = sms;
    entry.ready = true;
  }
  *out = entry;
  return B2K_OK;
}

}  // namespace

extern "C" int b2k_gemm_tf32x3_noalloc(const float *a, const float *b, float *c, int64_t m, int64_t n, int64_t k,
                                       int64_t lda, int64_t ldb, int64_t ldc, int32_t b_layout, const float *bias,
                                       int32_t relu, void *stream) {
  if (m < 0 || n < 0 || k < 0) return B2K_EINVAL;
  if ((b_layout & ~(B2K_B_NK | B2K_A_KM)) != 0) return B2K_EINVAL;
  if (m == 0 || n == 0) return B2K_OK;
  if (!a || !b || !c) return B2K_EINVAL;
  if (lda < ((b_layout & B2K_A_KM) ? m : k) || ldc < n || ldb < ((b_layout & B2K_B_NK) ? k : n)) return B2K_EINVAL;
  if (k == 0) return B2K_EUNSUPPORTED;
  // The extents must fit the kernels' 32-bit TMA coordinates (the limits of
  // b2k_gemm_tf32x3); this also keeps the scratch arithmetic below far from
  // int64 overflow.
  if (m > INT32_MAX - 256 || n > INT32_MAX - 256 || k > INT32_MAX - 64) return B2K_EINVAL;
  const int64_t kp = (k + 31) / 32 * 32;
  // 2 * (m + n) * kp floats, compared without forming the product.
  if (kp > (int64_t)kScratchFloats / (2 * (m + n))) return B2K_ESCRATCH;
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= kMaxDevices) return B2K_ECUDA;
  DeviceSymbols symbols;
  int status = device_symbols(device, &symbols);
  if (status != B2K_OK) return status;
  // A context on the stack, pointing at the static scratch and status word;
  // it owns nothing and is never passed to b2k_destroy.
  b2k_ctx local;
  local.fixed_scratch = true;
  local.device = device;
  local.sm_count = symbols.sm_count;
  local.error_flag = symbols.status;
  return b2k_gemm_tf32x3_impl(&local, a, b, c, m, n, k, lda, ldb, ldc, b_layout, bias, relu,
                              symbols.scratch, (cudaStream_t)stream, nullptr, 1.0f);
}

extern "C" int b2k_gemm_noalloc_status(int32_t device) {
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess) return B2K_ECUDA;
  if (device < 0 || device >= count || device >= kMaxDevices) return B2K_EINVAL;
  int previous = 0;
  if (cudaGetDevice(&previous) != cudaSuccess) return B2K_ECUDA;
  if (cudaSetDevice(device) != cudaSuccess) return B2K_ECUDA;
  DeviceSymbols symbols;
  int status = device_symbols(device, &symbols);
  unsigned int word = 0;
  if (status == B2K_OK && cudaMemcpy(&word, symbols.status, sizeof word, cudaMemcpyDeviceToHost) != cudaSuccess)
    status = B2K_ECUDA;
  if (status == B2K_OK && word != 0) {
    const unsigned int zero = 0;
    status = cudaMemcpy(symbols.status, &zero, sizeof zero, cudaMemcpyHostToDevice) == cudaSuccess ? B2K_ETIMEOUT
                                                                                                  : B2K_ECUDA;
  }
  if (cudaSetDevice(previous) != cudaSuccess && status == B2K_OK) status = B2K_ECUDA;
  return status;
}
