// The fused layer tail of the bf16 decode step (layer_fused.cu): one persistent kernel
// per layer that runs, after the block attention of layer l,
//   O projection -> residual + post-attention RMSNorm -> gate/up projection -> SwiGLU
//   -> down projection -> residual + the next RMSNorm -> QKV projection of layer l + 1
//   -> QK-norm + RoPE + KV append of layer l + 1
// (src/model/layer.rs:58-81, mlp.rs:38-45, attention.rs:90-184 of the next layer).
#pragma once

#include "gemm.h"
#include "layer_ops.h"

namespace wedlm {

struct FusedTailArgs {
  int M = 0;                    // token rows of the window (<= 96)
  int H = 0, I = 0, qdim = 0, qkvdim = 0;
  float eps = 1e-6f;
  const void* attn = nullptr;   // [M, qdim] attention output (the O projection's input)
  void* h = nullptr;            // [M, H] residual stream, updated twice
  void* xn = nullptr;           // [M, H] normed rows (gate/up input, then QKV input)
  void* act = nullptr;          // [M, I] SwiGLU output
  const void* wo = nullptr;     // packed weight tiles
  const void* wgate = nullptr;
  const void* wup = nullptr;
  const void* wdown = nullptr;
  const void* wqkv_next = nullptr;  // NULL: last layer (the tail stops after the final norm)
  const void* wo_next = nullptr;    // next layer's O projection (prefetched into L2), or NULL
  const float* ln2 = nullptr;       // post_attention_layernorm of layer l
  const float* ln_next = nullptr;   // input_layernorm of layer l + 1, or the final norm
  RopeKvArgs rope;              // QK-norm / RoPE / KV append of layer l + 1
  float* slots = nullptr;       // split-K partial slots (one set, reused by every GEMM)
  long slot_floats = 0;
  unsigned* sync = nullptr;     // 16 zeroed grid-wide dependency counters for this launch
  int* err = nullptr;
};

// Whether the fused tail applies to these widths / rows on this GPU, and the partial-slot
// floats it needs (the largest partial set of its GEMMs).
bool fused_tail_supported(int M, int H, int I, int qdim, int qkvdim, int head_dim,
                          int num_sms, long* slot_floats);
Status run_fused_tail(const FusedTailArgs& a, int num_sms, cudaStream_t st);

}  // namespace wedlm
