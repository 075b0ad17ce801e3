// Seeded T > 0 token sampling on the device (sample.cu): the multinomial and nucleus
// (top-p) branches of sample_from_probs_at_indices (src/decoding/sampler.rs:160-200,
// 306-351) over softmax(logits / T), with the reference's unseeded thread_rng replaced by
// a counter-based draw of (seed, sequence, step, mask row).
#pragma once

#include <cstdint>

#include "common.cuh"

namespace wedlm {

// SplitMix64 finaliser (Steele, Lea and Flood, OOPSLA 2014).
__host__ __device__ inline uint64_t sample_mix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

// The draw u in [0, 1) of mask row `row` of sequence `seq` at step `step`: SplitMix64
// chained over (seed, seq, step, row), 24 bits (the precision of rand's gen::<f32>()).
// Integer arithmetic and an exact conversion: the host and the device give the same u.
__host__ __device__ inline float sample_draw(uint64_t seed, uint64_t seq, uint64_t step,
                                             uint64_t row) {
  uint64_t h = sample_mix64(seed);
  h = sample_mix64(h ^ seq);
  h = sample_mix64(h ^ step);
  h = sample_mix64(h ^ row);
  return (float)(h >> 40) * 5.9604644775390625e-08f;  // 2^-24
}

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

// ---- sampling over a vocabulary split across ranks ----
//
// Each of `nranks` ranks holds the logits of every rank's mask rows over its own
// vocabulary shard (the shards tile [0, V_total) in rank order).  The rows are
// rank-major: row r = k * rmax + j is mask row j of rank k, valid while j < the rows
// field of rank k's gathered header.  Every rank runs the same phases; between phases
// each rank's payload is all-gathered (`gather`, one collective per phase), and every
// rank derives the same per-row state from the gathered payloads.  The owner of a row
// ends with the token the whole-vocabulary sampler gives for the same logits and draw:
// the maximum, the fixed-point sums and the radix buckets are exact under any split.

// Per-row state, replicated on every rank (device).
struct ShardSampleRow {
  unsigned long long S, TA, TB, acc, acc_a, total, j, i_tie;
  float mx;
  int sel, walk_b;
  unsigned prefix, pmask, n, vstar, n_eq, w;
};

struct ShardGather {
  // Enqueue on `st` an all-gather of `bytes` (a multiple of 16) from send into recv
  // ([nranks, bytes], rank order).
  Status (*fn)(void* user, const void* send, void* recv, size_t bytes, cudaStream_t st) = nullptr;
  void* user = nullptr;
};

struct ShardSampleArgs {
  const void* logits = nullptr;  // [rows, ld]: every rank's rows over this rank's shard
  int dtype = WEDLM_BF16;
  int V = 0;                     // this shard's width
  long ld = 0;
  int vocab_begin = 0;           // first token of this shard
  int V_total = 0;
  int nranks = 1, me = 0, rmax = 0;  // rows = nranks * rmax
  float temperature = 1.f, top_p = 1.f;
  const int* hdr = nullptr;      // gathered headers [nranks][4]; field 1 = valid rows
  const float* u = nullptr;      // [rows] gathered draws
  // this rank's selection (the commit rule's output over its own rows)
  int nseq = 0;
  const int* seq_rows = nullptr;
  const int* selected = nullptr;
  const int* n_selected = nullptr;
  ShardSampleRow* state = nullptr;  // [rows]
  void* xsend = nullptr;            // shard_sample_xbytes() bytes
  void* xrecv = nullptr;            // nranks * shard_sample_xbytes() bytes
  int* tokens = nullptr;            // [rmax] own rows: selected rows get the sampled token
};

// Exchange bytes per rank that run_shard_sample needs for `rows` rows.
size_t shard_sample_xbytes(int rows, int rmax, bool nucleus);
Status run_shard_sample(const ShardSampleArgs& a, const ShardGather& g, cudaStream_t st);

}  // namespace wedlm
