// Epilogue helper shared by the tcgen05 GEMM kernels (gemm_tc.cu, layer_fused.cu).
#pragma once

#include "sm100.cuh"

namespace wedlm {

// Epilogue transpose of one accumulator chunk.  TMEM lane r (weight row rr + r) holds w
// consecutive tokens (w = 32 or 16); through the warp's [32][33] shared buffer each lane
// takes 8 consecutive weight rows, (lane % 4) * 8 .. + 7, of the four tokens
// i * 8 + lane / 4 (i = 0..3), so that four lanes cover one token's 32 rows and the
// global stores are whole 128-byte (f32) or 64-byte (bf16) runs.  Conflict-free: bank
// (token + row) % 32 differs across the warp in both phases.
__device__ __forceinline__ void epi_transpose(uint32_t taddr, int w, float* tb, int lane,
                                              float (&o)[4][8]) {
  float v[32];
  if (w == 32) {
    sm100::tmem_ld32(taddr, v);
  } else {
    float h[16];
    sm100::tmem_ld16(taddr, h);
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = h[j];
#pragma unroll
    for (int j = 16; j < 32; ++j) v[j] = 0.f;
  }
#pragma unroll
  for (int j = 0; j < 32; ++j) tb[j * 33 + lane] = v[j];
  __syncwarp();
  const int r0 = (lane & 3) * 8;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int tl = i * 8 + (lane >> 2);
#pragma unroll
    for (int e = 0; e < 8; ++e) o[i][e] = tb[tl * 33 + r0 + e];
  }
  __syncwarp();
}

}  // namespace wedlm
