// nbl_selftest_bounded_wait: makes the library's bounded device wait run out, on purpose and harmlessly.
//
// Every wait in the TMA/tensor-core kernels (mbarrier phases of copies and MMAs) goes through mbar_wait_slow
// (nbl_device.cuh), which gives up after a wall-clock limit, sets kErrTimeout in the context's error word and
// returns false, so the kernel can finish instead of hanging the GPU. This entry point runs that same routine in a
// one-thread kernel against an mbarrier that nothing ever arrives on, with a caller-chosen short limit: the wait
// must give up, the kernel must return, and nbl_ctx_check must then report NBL_E_DEVICE. No reference counterpart
// (the reference's error convention is nibble::Error, include/nibble/error.h:8-13); this is the device-side form
// of its failure reporting.
#include <string>

#include "nbl_device.cuh"
#include "nbl_internal.h"

namespace {

__global__ void bounded_wait_selftest_kernel(int* err, uint64_t limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  nbl::mbar_init(&bar, 1);
  nbl::fence_barrier_init();
  // phase 0 never completes: the expected arrival count is 1 and no thread arrives. The wait gives up after
  // limit_ns and sets kErrTimeout in *err; the kernel then simply ends.
  (void)nbl::mbar_wait_slow(&bar, 0, err, limit_ns);
}

}  // namespace

extern "C" NBL_API int nbl_selftest_bounded_wait(nbl_ctx* ctx, int64_t limit_ns) {
  try {
    if (!ctx) nbl::fail(NBL_E_INVALID, "selftest_bounded_wait: ctx is NULL");
    if (limit_ns <= 0 || limit_ns > 1000000000)
      nbl::fail(NBL_E_INVALID, "selftest_bounded_wait: limit_ns must be in (0, 1e9], got " + std::to_string(limit_ns));
    nbl::check_cuda(cudaSetDevice(ctx->device), "cudaSetDevice");
    bounded_wait_selftest_kernel<<<1, 1, 0, ctx->stream>>>(ctx->d_err, static_cast<uint64_t>(limit_ns));
    nbl::check_cuda(cudaGetLastError(), "selftest launch");
    return NBL_OK;
  } catch (const nbl::Failure& e) {
    return nbl::record_error(e.status, e.what());
  } catch (const std::exception& e) {
    return nbl::record_error(NBL_E_INVALID, e.what());
  }
}
