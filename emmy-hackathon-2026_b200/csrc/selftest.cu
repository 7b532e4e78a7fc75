// Failure-detection self test: a kernel whose mbarrier wait can never
// complete (nothing arrives on the barrier), run with a short cycle budget.
// The wait gives up, records its site code in the context's device error
// word and the kernel returns normally, so the host sees B2K_ETIMEOUT from
// b2k_stream_sync and the context stays usable.  This exercises the same
// bounded-wait path every tensor-core kernel relies on, without faulting or
// hanging the GPU.
#include "common.cuh"
#include "sm100.cuh"

namespace {

constexpr unsigned kSiteSelfTest = 0x80000000u;

__global__ void __launch_bounds__(32, 1) wait_forever_bounded(unsigned *err, long long budget) {
  __shared__ __align__(8) uint64_t never_arrived;
  __shared__ int abort_word;
  if (threadIdx.x == 0) {
    abort_word = 0;
    sm100::mbar_init(&never_arrived, 1);
    sm100::fence_barrier_init();
  }
  __syncwarp();
  // Lane 0 waits for phase 0 of a barrier nobody arrives on.
  if (threadIdx.x == 0) sm100::mbar_wait(&never_arrived, 0, err, kSiteSelfTest, &abort_word, budget);
  __syncwarp();
}

}  // namespace

extern "C" int b2k_selftest_wait_timeout(b2k_ctx *ctx, int64_t budget_cycles, void *stream) {
  B2K_CHECK_CTX(ctx);
  if (budget_cycles <= 0 || budget_cycles > (int64_t)sm100::kWaitCycles)
    return b2k::fail(ctx, B2K_EINVAL, "selftest: budget must be in (0, %lld] cycles", sm100::kWaitCycles);
  wait_forever_bounded<<<1, 32, 0, (cudaStream_t)stream>>>(ctx->error_flag, (long long)budget_cycles);
  return b2k::check_launch(ctx, "selftest launch");
}
