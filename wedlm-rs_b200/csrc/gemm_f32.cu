// f32 projection GEMM on the CUDA cores, for f32 models (the reference's f32 parity
// configuration, src/config.rs:101-124 honours dtype = float32).  Same epilogues as the
// tcgen05 path, with f32 storage and no intermediate rounding:
//   EPI_STORE_*   out = Y
//   EPI_RESID_*   out = resid + Y
//   EPI_SWIGLU_*  out = silu(Y_gate) * Y_up
// 64 x 64 output tiles, 16-wide K steps through shared memory, 4 x 4 outputs per thread.
#include "gemm.h"

namespace wedlm {

namespace {

constexpr int kT = 64, kK = 16;

__global__ void __launch_bounds__(256)
gemm_f32_kernel(const float* __restrict__ X, long ldx, const float* __restrict__ W,
                const float* __restrict__ W2, long ldw, int M, int N, int K, int epi,
                float* out, long ldo, const float* resid, long ldr) {
  __shared__ float sx[kK][kT + 1];
  __shared__ float sw[kK][kT + 1];
  __shared__ float sw2[kK][kT + 1];
  const bool dual = epi == EPI_SWIGLU_BF16;
  const int tm = blockIdx.y * kT, tn = blockIdx.x * kT;
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  float acc[4][4] = {}, acc2[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += kK) {
    for (int i = threadIdx.x; i < kK * kT; i += 256) {
      const int r = i / kK, c = i % kK;
      const int gm = tm + r, gn = tn + r, gk = k0 + c;
      sx[c][r] = (gm < M && gk < K) ? X[(long)gm * ldx + gk] : 0.f;
      sw[c][r] = (gn < N && gk < K) ? W[(long)gn * ldw + gk] : 0.f;
      if (dual) sw2[c][r] = (gn < N && gk < K) ? W2[(long)gn * ldw + gk] : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int c = 0; c < kK; ++c) {
      float a[4], b[4], b2[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        a[i] = sx[c][ty * 4 + i];
        b[i] = sw[c][tx * 4 + i];
        b2[i] = dual ? sw2[c][tx * 4 + i] : 0.f;
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
          if (dual) acc2[i][j] = fmaf(a[i], b2[j], acc2[i][j]);
        }
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int m = tm + ty * 4 + i, n = tn + tx * 4 + j;
      if (m >= M || n >= N) continue;
      float y = acc[i][j];
      if (epi == EPI_RESID_BF16) y = resid[(long)m * ldr + n] + y;
      if (dual) y = (y / (1.f + expf(-y))) * acc2[i][j];
      out[(long)m * ldo + n] = y;
    }
}

}  // namespace

Status run_gemm_f32(const GemmArgs& a, cudaStream_t st) {
  WEDLM_CHECK_ARG(a.M > 0 && a.N > 0 && a.K > 0, "empty GEMM");
  WEDLM_CHECK_ARG(a.epi != EPI_SWIGLU_BF16 || a.W2, "SwiGLU GEMM needs the second weight matrix");
  dim3 grid((a.N + kT - 1) / kT, (a.M + kT - 1) / kT);
  gemm_f32_kernel<<<grid, 256, 0, st>>>(
      (const float*)a.X, a.ldx, (const float*)a.W, (const float*)a.W2, a.ldw, a.M, a.N, a.K, a.epi,
      (float*)a.out, a.ldo, (const float*)a.resid, a.ldr);
  WEDLM_CUDA_TRY(cudaGetLastError());
  return Status::ok();
}

}  // namespace wedlm
