// Seeded T > 0 token sampling on the device (sample.cu): the multinomial and nucleus
// (top-p) branches of sample_from_probs_at_indices (src/decoding/sampler.rs:160-200,
// 306-351) over softmax(logits / T), with the reference's unseeded thread_rng replaced by
// a counter-based draw of (seed, sequence, step, mask row).
#pragma once

#include "common.cuh"

namespace wedlm {

struct SampleArgs {
  const void* logits = nullptr;  // [rows, ld] of dtype (V valid columns)
  int dtype = WEDLM_BF16;
  int rows = 0, V = 0;
  long ld = 0;
  float temperature = 1.f;  // > 0
  float top_p = 1.f;        // >= 1: multinomial; < 1: nucleus
  unsigned long long seed = 0;
  // Decode mode: the rows are the mask rows of nseq sequences (CSR seq_rows, device);
  // only the rows listed in selected / n_selected (the commit rule's output) are sampled,
  // each with the draw of (seed, seq_key[b], seq_step[b], row index within sequence b).
  int nseq = 0;
  const int* seq_rows = nullptr;
  const int* selected = nullptr;
  const int* n_selected = nullptr;
  const int* seq_key = nullptr;
  const int* seq_step = nullptr;
  // Explicit mode (u != NULL): every row is sampled with the draw u[row] (device).
  const float* u = nullptr;
  int* tokens = nullptr;  // [rows] (device): the sampled token of each sampled row
};

Status run_sample(const SampleArgs& a, cudaStream_t st);

}  // namespace wedlm
