// Shared helpers for the WeDLM B200 kernels: status handling, bf16 conversion,
// warp reductions, and small PTX wrappers.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include <string>
#include <utility>

#include "../../include/wedlm_b200.h"

namespace wedlm {

// A failed call records its message here and returns a status code.
struct Status {
  int code = WEDLM_OK;
  std::string msg;
  static Status ok() { return Status(); }
  static Status err(int c, std::string m) {
    Status s;
    s.code = c;
    s.msg = std::move(m);
    return s;
  }
  bool good() const { return code == WEDLM_OK; }
};

#define WEDLM_CUDA_TRY(expr)                                                            \
  do {                                                                                  \
    cudaError_t e_ = (expr);                                                            \
    if (e_ != cudaSuccess)                                                              \
      return ::wedlm::Status::err(WEDLM_ERR_CUDA, std::string(#expr) + ": " +           \
                                                      cudaGetErrorString(e_));          \
  } while (0)

#define WEDLM_TRY(expr)            \
  do {                             \
    ::wedlm::Status s_ = (expr);   \
    if (!s_.good()) return s_;     \
  } while (0)

#define WEDLM_CHECK_ARG(cond, what)                                                     \
  do {                                                                                  \
    if (!(cond)) return ::wedlm::Status::err(WEDLM_ERR_INVALID_ARG, what);              \
  } while (0)

inline int dtype_size(int dt) { return dt == WEDLM_F32 ? 4 : 2; }

// ---- device helpers ------------------------------------------------------------------

__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

template <typename T> __device__ __forceinline__ float to_f32(T v);
template <> __device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}

template <typename T> __device__ __forceinline__ T from_f32(float v);
template <> __device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

// 2^x on the MUFU unit (PTX ex2.approx.ftz.f32).
// Programmatic dependent launch.  A kernel launched with launch_pdl() may start while
// the previous kernel on the stream is still running; pdl_wait() blocks until that
// kernel has completed and its writes are visible, so every such kernel calls it before
// it reads anything the previous kernels wrote or writes anything they may still read.
// pdl_trigger() lets the next kernel on the stream be scheduled early.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

bool pdl_enabled();  // WEDLM_PDL=0 turns the early launch off (the kernels are unchanged)

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ int warp_min_i(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// 128-bit streaming load that bypasses L1 allocation (read-once data).
__device__ __forceinline__ uint4 ld_stream_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

}  // namespace wedlm
