// Probe of the bounded device-side wait that every tcgen05 kernel here relies on.
//
// A kernel that loses a handshake (a producer that never arrives on an mbarrier) must
// give up after its time limit, record the wait site in the context's error word and
// return, so that the context stays usable and the host sees WEDLM_ERR_TIMEOUT from
// wedlm_check_device_error instead of a hung GPU.  This entry point builds exactly that
// situation on purpose and safely: one CTA initialises an mbarrier that no thread
// ever arrives on and no copy is in flight for, and one warp waits on it with the
// same mbar_wait_for helper the GEMM and attention kernels use, with a short limit.
// No counterpart in the reference (its host code has no device waits).
#include "../../include/wedlm_b200_kernels.h"
#include "context.h"
#include "sm100.cuh"

namespace wedlm {
namespace {

using namespace sm100;

// out[0] = 1 if the wait succeeded (it must not), out[1] = microseconds waited.
__global__ void wait_probe_kernel(int* err, uint64_t limit_ns, int* out) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x >= 32) {
    // the "consumer" warp: phase 0 of a fresh barrier with count 1 completes only when
    // one thread arrives, and none does
    const uint64_t t0 = global_ns();
    const bool ok = mbar_wait_for(&bar, 0, err, kErrWaitFull, limit_ns);
    if (threadIdx.x == 32) {
      out[0] = ok ? 1 : 0;
      out[1] = (int)((global_ns() - t0) / 1000);
    }
  }
}

}  // namespace
}  // namespace wedlm

extern "C" int wedlm_kernel_wait_probe(wedlm_ctx* ctx, int64_t limit_ns, int32_t* out,
                                       void* stream) {
  using wedlm::Status;
  if (!ctx) return WEDLM_ERR_INVALID_ARG;
  cudaError_t e = cudaSetDevice(ctx->device);
  if (e != cudaSuccess) return ctx->fail(Status::err(WEDLM_ERR_CUDA, cudaGetErrorString(e)));
  if (!out || limit_ns <= 0 || limit_ns > 2000000000LL)
    return ctx->fail(Status::err(WEDLM_ERR_INVALID_ARG,
                                 "wait probe: out is required and the limit must be in (0, 2 s]"));
  Status s = wedlm::ensure_gemm_scratch(ctx, 0, 0);  // the context's device error word
  if (!s.good()) return ctx->fail(s);
  wedlm::wait_probe_kernel<<<1, 64, 0, (cudaStream_t)stream>>>(ctx->dev_err, (uint64_t)limit_ns,
                                                               out);
  e = cudaGetLastError();
  if (e != cudaSuccess) return ctx->fail(Status::err(WEDLM_ERR_CUDA, cudaGetErrorString(e)));
  return WEDLM_OK;
}
