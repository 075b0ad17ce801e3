// Projection GEMMs: Y[tok, n] = sum_k X[tok, k] * W[n, k] with fused epilogues.
#pragma once

#include "common.cuh"

namespace wedlm {

enum GemmEpilogue {
  EPI_STORE_BF16 = 0,   // Y -> bf16
  EPI_STORE_F32 = 1,    // Y -> f32
  EPI_RESID_BF16 = 2,   // out = bf16(resid + bf16(Y))            (residual add)
  EPI_SWIGLU_BF16 = 3,  // out = bf16(silu(bf16(Y_gate)) * bf16(Y_up))
};

struct GemmArgs {
  const void* X = nullptr;  // [M, K] (row stride ldx)
  long ldx = 0;
  const void* W = nullptr;  // [N, K] (row stride ldw)
  const void* W2 = nullptr; // second [N, K] matrix (SwiGLU up projection)
  long ldw = 0;
  int M = 0, N = 0, K = 0;
  int epi = EPI_STORE_BF16;
  void* out = nullptr;      // [M, N] (row stride ldo)
  long ldo = 0;
  const void* resid = nullptr;  // [M, N] (row stride ldr); may alias out
  long ldr = 0;
};

struct GemmPlan {
  int tok_tile = 0, t_tiles = 0, n_tiles = 0, kb_total = 0, splits = 1, stages = 0;
  int grid = 0, nbuf = 1;
  uint32_t stage_bytes = 0, tmem_cols = 0, smem_bytes = 0, acc_cols = 0;
  long ws_floats = 0;  // shared-tile partials (two slots per CTA)
  int counters = 0;    // per-tile arrival counters (zero between launches)
};

// bf16 tcgen05 path (K % 64 == 0).
GemmPlan plan_gemm_tc(int M, int N, int K, bool dual, int num_sms);
Status run_gemm_tc(const GemmArgs& a, const GemmPlan& g, float* ws, unsigned* counters, int* err,
                   cudaStream_t st);
void forget_tensor_maps();

// f32 path (CUDA cores, for f32 models): same epilogues with f32 storage.
Status run_gemm_f32(const GemmArgs& a, cudaStream_t st);

}  // namespace wedlm
