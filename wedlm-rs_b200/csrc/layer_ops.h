// Host interface of the decoder-layer kernels (layer_ops.cu, attention_tc.cu).
#pragma once

#include "common.cuh"
#include "gemm.h"

namespace wedlm {

// Paged KV cache geometry, shared by the append and attention kernels.
//   K: [layers][num_pages][nkv][page_size][d]
//   V: [layers][num_pages][nkv][d][page_size]   (transposed within a page)
struct KvGeom {
  void* kcache = nullptr;
  void* vcache = nullptr;
  const int* page_table = nullptr;  // [seqs][pages_per_seq]
  int pages_per_seq = 0, num_pages = 0, page_size = 64;
  int layer = 0, num_layers = 1;
};

struct RopeKvArgs : KvGeom {
  const void* qkv = nullptr;  // [rows, ld_qkv]: q heads, then k heads, then v heads
  long ld_qkv = 0;
  int rows = 0, nh = 0, nkv = 0, group = 1, head_dim = 0;
  int qk_norm = 1;
  const float* q_norm = nullptr;
  const float* k_norm = nullptr;
  float eps = 1e-6f;
  const int* positions = nullptr;  // [rows] RoPE position of each row
  const float* cos = nullptr;      // [max_pos, d/2]
  const float* sin = nullptr;
  const int* row_seq = nullptr;    // [rows] cache slot (sequence) of each row
  const int* dst_pos = nullptr;    // [rows] cache position written by each row
  void* q_out = nullptr;           // group-major [nkv][rows * group][d]
  // bf16 models: the QKV projection as split-K partials (summed and rounded here)
  const PartialSet* qkv_partials = nullptr;
  // [rows] or NULL: rows with 0 are skipped (the device loop's padding rows)
  const int* row_active = nullptr;
};

struct AttnArgs : KvGeom {
  const void* q = nullptr;  // group-major [nkv][rows * group][d]
  int rows = 0, nh = 0, nkv = 0, group = 1, head_dim = 0;
  const int* row_seq = nullptr;        // [rows] batch index b of each row
  const int* seq_row0 = nullptr;       // [nseq] first row of sequence b
  const int* seq_rows = nullptr;       // [nseq] rows (window length S_b) of sequence b
  const int* seq_cache_len = nullptr;  // [nseq] committed cache length L_b
  const int* seq_slot = nullptr;       // [nseq] cache slot (page-table row) of sequence b
  const int* rank = nullptr;           // [rows] mask rank, NULL = index within window
  void* out = nullptr;                 // [rows, ld_out] (head h at column h * d)
  long ld_out = 0;
  int nseq = 0, max_kv = 0;            // max_kv = max_b (L_b + S_b)
};

// row_active ([rows] or NULL, also below): rows with 0 are skipped (the device loop's
// padding rows keep whatever they held).
Status run_embed(const void* table, int dtype, const int* ids, int rows, int H, int vocab,
                 void* out, int* err, cudaStream_t st, const int* row_active = nullptr);
Status run_rmsnorm(const void* x, long ldx, const float* w, int rows, int H, float eps, int dtype,
                   void* out, long ldo, cudaStream_t st);
Status run_rope_kv(const RopeKvArgs& a, int dtype, cudaStream_t st);
// bf16: h = bf16(h + bf16(sum of partials)) (skipped when ps is NULL), then
// xn = RMSNorm(h) * w (rounded to bf16): the residual add of layer.rs:72,78 fused with
// the next RMSNorm (attention.rs:35-50).
Status run_resid_norm(void* h, const PartialSet* ps, const float* w, int rows, int H, float eps,
                      void* xn, cudaStream_t st, const int* row_active = nullptr);
// bf16: act = bf16(silu(bf16(gate)) * bf16(up)) from the gate/up partials (mlp.rs:40-43).
Status run_swiglu(const PartialSet& ps, int rows, int I, void* act, cudaStream_t st,
                  const int* row_active = nullptr);
Status run_attention_f32(const AttnArgs& a, cudaStream_t st);

// bf16 block attention on the tensor cores.  The plan (work items, split-KV layout) is
// built once per forward from host copies of the per-sequence window and cache lengths
// and uploaded into the workspace `ws`; run_attention_tc is then called per layer.
struct AttnPlan {
  int n_work = 0, n_comb = 0;  // launch sizes (device-built plans: upper bounds)
  const float* work = nullptr;
  const float* comb = nullptr;
  float* part_o = nullptr;
  float* part_ml = nullptr;
  const int* n_work_dev = nullptr;  // device-built plans: the item counts of the step
  const int* n_comb_dev = nullptr;
};
long attention_ws_floats(const AttnArgs& a);
Status plan_attention_tc(const AttnArgs& a, const int* h_seq_rows, const int* h_cache_len,
                         int num_sms, float* ws, long ws_floats, void* h_staging,
                         size_t staging_bytes, AttnPlan* plan, cudaStream_t st);
// The same plan built on the device from a.seq_rows / a.seq_cache_len (device arrays of
// the step), for at most max_work work items and max_comb combine items: a sequence-
// independent upper bound is max(num_sms, sum over sequences of nkv * ceil(S * group /
// 128)).  counts (device int[2]) receives the item counts; err records a plan that did
// not fit the bounds (nothing runs then).  Workspace: attention_ws_floats_device floats.
long attention_ws_floats_device(int max_work, int max_comb);
Status plan_attention_tc_device(const AttnArgs& a, int num_sms, float* ws, long ws_floats,
                                int max_work, int max_comb, int* counts, int* err,
                                AttnPlan* plan, cudaStream_t st);
Status run_attention_tc(const AttnArgs& a, const AttnPlan& plan, int* err, cudaStream_t st);

}  // namespace wedlm
