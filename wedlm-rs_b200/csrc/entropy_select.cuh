// Host-side interface of the fused entropy-select kernels (entropy_select.cu).
#pragma once

#include "common.cuh"

namespace wedlm {

struct EntropyArgs {
  const void* logits = nullptr;
  int dtype = WEDLM_BF16;
  int rows = 0, V = 0;
  long ld = 0;
  float temperature = 0.f, tau = 0.f, lambda = 0.f;
  int nseq = 0;
  const int* seq_rows = nullptr;  // device [nseq + 1]
  const int* mask_pos = nullptr;  // device [rows]
  const int* caps = nullptr;      // device [nseq]
  // Optional streaming-decode mode (wedlm.rs:517-535): when `running` is set, each
  // sequence's entropy EMA running[b] is updated with the mean entropy of its rows and
  // the cap becomes the dynamic cap derived from caps[b] (the preset cap).
  float* running = nullptr;       // device, indexed by running_idx[b] (or b)
  const int* running_idx = nullptr;
  float* H = nullptr;
  int* argmax = nullptr;
  float* maxprob = nullptr;
  int* selected = nullptr;
  int* n_selected = nullptr;
  // Rows the vocabulary split is planned for (0: rows).  The decode loops plan for their
  // row capacity, so that a row's statistics are merged in the same order whatever the
  // step's row count (the host loop's mask rows, the device loop's padded rows).
  int plan_rows = 0;
};

// Scratch (global memory) the kernels need besides their inputs and outputs.
struct EntropyScratch {
  float* partials = nullptr;   // [partial_capacity] floats
  long partial_capacity = 0;
  float* row_H = nullptr;      // [row_capacity]
  unsigned* row_count = nullptr;  // [row_capacity], zero between launches
  int row_capacity = 0;
  unsigned* seq_count = nullptr;  // [seq_capacity], zero between launches
  int seq_capacity = 0;
};

struct EntropyPlan {
  int splits = 1;
  int split_cols = 0;
};

EntropyPlan plan_entropy(int rows, int V, int dtype, int num_sms);
Status run_entropy_select(const EntropyArgs& A, const EntropyScratch& W, int num_sms,
                          cudaStream_t st);
Status run_entropy_partials(const EntropyArgs& A, const EntropyScratch& W, int vocab_offset,
                            float* out, int num_sms, cudaStream_t st);
// Shard k's partial of row r is at partials + (k * shard_stride + r) * 4 (shard_stride in
// rows; <= 0 means A.rows, i.e. [nshards, rows * 4] packed).
Status run_entropy_combine(const float* partials, int nshards, const EntropyArgs& A,
                           const EntropyScratch& W, cudaStream_t st, long shard_stride = 0);

}  // namespace wedlm
