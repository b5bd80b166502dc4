// Self-test of the bounded device-side waits.
//
// Every pipelined kernel of this library (attention, GEMM) bounds its mbarrier waits: a wait that
// gives up records a code in the kernel's device status word, raises the CTA's abort flag and lets
// the kernel return, so a stuck pipeline surfaces as a status the host reads instead of a hang.
// fa_watchdog_selftest exercises exactly that path on demand, without faulting anything: one warp
// waits, with the caller's limit, on an mbarrier that nothing ever arrives on. The wait gives up,
// writes FA_STATUS_WATCHDOG_SELFTEST into the attention status word, and the kernel returns
// normally; the context stays usable.
#include "attention.cuh"
#include "fa_common.cuh"
#include "ptx.cuh"

namespace fa {
namespace {

__global__ void __launch_bounds__(32, 1) watchdog_selftest_kernel(int* status, uint64_t timeout_ns, int code) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    abort_flag = 0;
    ptx::mbar_init(ptx::smem_u32(&bar), 1);
    ptx::fence_mbarrier_init();
  }
  __syncwarp();
  if (threadIdx.x == 0) {
    // Phase 0 of `bar` never completes (its one expected arrival never comes): the bounded wait
    // returns false after about timeout_ns and records `code`.
    ptx::mbar_wait(ptx::smem_u32(&bar), 0u, &abort_flag, status, code, timeout_ns);
  }
  __syncwarp();
}

}  // namespace
}  // namespace fa

extern "C" int fa_watchdog_selftest(int64_t timeout_ns, void* stream) {
  FA_REQUIRE(timeout_ns >= 1000 && timeout_ns <= 100000000, FA_ERR_INVALID,
             "timeout_ns must be between 1 us and 100 ms");
  int* status = fa::attn::status_ptr();
  FA_REQUIRE(status, FA_ERR_CUDA, "cannot resolve the attention status word");
  fa::watchdog_selftest_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(status, (uint64_t)timeout_ns,
                                                                     FA_STATUS_WATCHDOG_SELFTEST);
  return fa::check_launch("watchdog_selftest_kernel");
}
