/*
 * wedlm_b200.h -- C ABI of the B200-native WeDLM block-parallel decode step.
 *
 * The reference (arkavo-ai/WeDLM-rs) has no FFI layer; its replaceable seam is the
 * Rust model/sampler API that WeDLMDecoder calls.  Each entry point below names the
 * reference function it replaces.  Conventions:
 *   - every call returns an int status (WEDLM_OK = 0, negative = error class);
 *     wedlm_last_error(ctx) returns the message of the last failure on ctx
 *     (wedlm_last_error(NULL): last failure of wedlm_create on this thread);
 *   - one context per GPU; a context is not thread-safe, callers serialise;
 *   - `stream` is a cudaStream_t (NULL = the legacy default stream); calls taking a
 *     stream are stream-ordered and do not synchronise unless stated;
 *   - token ids and positions are int32 (the reference uses i64; a Rust shim narrows);
 *   - pointers documented "device" must be CUDA device pointers on the context's
 *     GPU, pointers documented "host" are ordinary host memory.
 */
#ifndef WEDLM_B200_H
#define WEDLM_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define WEDLM_API __attribute__((visibility("default")))
#else
#define WEDLM_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef struct wedlm_ctx wedlm_ctx;

enum wedlm_status {
  WEDLM_OK = 0,
  WEDLM_ERR_INVALID_ARG = -1,
  WEDLM_ERR_OOM = -2,
  WEDLM_ERR_CUDA = -3,
  WEDLM_ERR_TIMEOUT = -4,
  WEDLM_ERR_NOT_FOUND = -5,
  WEDLM_ERR_IO = -6,
  WEDLM_ERR_STATE = -7,
  WEDLM_ERR_UNSUPPORTED = -8
};

enum wedlm_dtype { WEDLM_F32 = 0, WEDLM_BF16 = 1, WEDLM_F16 = 2 };

/* Model shape, mirrors WeDLMConfig (src/config.rs:9-78).  `dtype` is the model
 * (storage and GEMM input) dtype: WEDLM_F32 or WEDLM_BF16. */
typedef struct wedlm_config {
  int32_t vocab_size;
  int32_t hidden_size;
  int32_t num_hidden_layers;
  int32_t num_attention_heads;
  int32_t num_key_value_heads;
  int32_t head_dim;
  int32_t intermediate_size;
  int32_t max_position_embeddings;
  double rope_theta;
  double rms_norm_eps;
  int32_t qk_norm;
  int32_t eos_token_id;
  int32_t mask_token_id;
  int32_t dtype;
  int32_t max_block_tokens;   /* largest window a forward may carry (0 -> 128) */
  int32_t vocab_shard_begin;  /* LM-head rows held here: [begin, end); 0,0 = all */
  int32_t vocab_shard_end;
} wedlm_config;

/* SamplingParams (src/decoding/sampler.rs:12-44). */
typedef struct wedlm_sampling_params {
  float temperature;
  float top_p;
  float entropy_threshold;
  float distance_penalty;
  int32_t max_tokens_per_step;
  float margin_threshold;
} wedlm_sampling_params;

/* BlockStats (src/decoding/wedlm.rs:41-58). */
typedef struct wedlm_block_stats {
  int64_t steps;
  int64_t tokens_generated;
  float avg_confidence;
  float avg_entropy;
  float max_entropy;
  int64_t high_entropy_count;
  int64_t block_size_reductions;
  int64_t cache_refreshes;
  int32_t prefix_cached;
} wedlm_block_stats;

/* ---- context ------------------------------------------------------------------ */

/* Replaces WeDLMForCausalLM::new (src/model/causal_lm.rs:23-31) plus the decoder's
 * KV cache (src/decoding/wedlm.rs:67-69): allocates the weights and a preallocated
 * paged KV cache of max_seqs x max_ctx tokens on `device`. */
WEDLM_API int wedlm_create(const wedlm_config* cfg, int device, int max_seqs, int max_ctx,
                 wedlm_ctx** out);
WEDLM_API void wedlm_destroy(wedlm_ctx* ctx);
WEDLM_API const char* wedlm_last_error(const wedlm_ctx* ctx);
WEDLM_API int wedlm_get_config(const wedlm_ctx* ctx, wedlm_config* out);

/* ---- weights ------------------------------------------------------------------ */

/* One tensor by its safetensors name (e.g. "model.layers.0.self_attn.q_proj.weight"),
 * host data of `dtype`, converted to the model dtype.  Replaces VarBuilder::get
 * (src/weights.rs:27-46 via src/model/*.rs constructors). */
WEDLM_API int wedlm_set_weight(wedlm_ctx* ctx, const char* name, const void* host_data, int dtype,
                     const int64_t* shape, int ndim);
/* Every tensor the model needs from a Hugging Face checkpoint directory:
 * model.safetensors, or the shards listed by model.safetensors.index.json
 * ("weight_map"), as load_model_vb / load_sharded_vb / load_safetensors_file
 * (src/weights.rs:27-46, 59-107, 110-131) read them.  BF16 / F16 / F32 / F64 data are
 * converted to the model dtype (tensor_from_view, weights.rs:135-210); tensors the model
 * does not use are skipped.  WEDLM_ERR_NOT_FOUND when neither file exists or a needed
 * tensor is missing, WEDLM_ERR_IO for a malformed file. */
WEDLM_API int wedlm_load_weights(wedlm_ctx* ctx, const char* model_dir);
/* Seeded random init on the device: linear and embedding weights N(0, std^2),
 * norm weights 1.  (No reference counterpart; the reference only loads checkpoints.) */
WEDLM_API int wedlm_init_random(wedlm_ctx* ctx, uint64_t seed, float std);
/* Copy of one tensor back to the host in the model dtype (for checks). */
WEDLM_API int wedlm_get_weight(wedlm_ctx* ctx, const char* name, void* host_out, int64_t nbytes);

/* ---- KV cache ----------------------------------------------------------------- */

/* WeDLMDecoder::clear_cache (src/decoding/wedlm.rs:299-302) for one sequence. */
WEDLM_API int wedlm_reset_sequence(wedlm_ctx* ctx, int seq);
/* Committed length of a sequence's cache (prefix_cache_len, wedlm.rs:69). */
WEDLM_API int wedlm_cache_len(const wedlm_ctx* ctx, int seq, int32_t* out_len);
/* Advance the committed length by n_commit (<= last block's size).  The last
 * block's K/V were appended at the committed length in reordered order, so this is
 * truncate_cache(committed_len + n_commit) (src/decoding/wedlm.rs:308-323,455-465). */
WEDLM_API int wedlm_commit(wedlm_ctx* ctx, int seq, int n_commit);
/* Shrink a sequence's committed length (truncate_cache with new_len < len). */
WEDLM_API int wedlm_truncate(wedlm_ctx* ctx, int seq, int new_len);

/* ---- forward ------------------------------------------------------------------ */

/* WeDLMDecoder::cache_prefix (src/decoding/wedlm.rs:85-96) via
 * WeDLMForCausalLM::forward (causal_lm.rs:46-56): causal forward over `n` host
 * token ids at positions [cache_len, cache_len + n), appending their K/V to the
 * cache and committing them.  No LM head (the reference's prefill logits are unused). */
WEDLM_API int wedlm_prefill(wedlm_ctx* ctx, int seq, const int32_t* ids, int n, void* stream);

/* WeDLMForCausalLM::forward_with_positions (src/model/causal_lm.rs:68-79) for a
 * batch of sequences, each carrying an S-token reordered window (host arrays,
 * row-major [nseq, S]).  Block key j is visible to block query i iff
 * rank[j] <= rank[i]; rank = NULL means rank = reordered index (the reference's
 * create_causal_mask, src/model/attention.rs:255-279).  The window K/V are written
 * at each sequence's committed length (not committed; see wedlm_commit).
 * Logits: for sequence b, rows logit_row_begin[b] .. S-1 of its window are
 * projected (NULL -> all rows) and written, densely packed in sequence order, to
 * `logits_out` (device, dtype `logits_dtype`, row stride = vocab shard width);
 * `n_logit_rows_out` (host, may be NULL) receives the total row count.
 * logits_out may be NULL to skip the LM head. */
WEDLM_API int wedlm_block_forward(wedlm_ctx* ctx, int nseq, const int32_t* seq_ids,
                        const int32_t* tokens, const int32_t* positions, const int32_t* rank,
                        int S, const int32_t* logit_row_begin, void* logits_out,
                        int logits_dtype, int32_t* n_logit_rows_out, void* stream);

/* ---- fused entropy-select --------------------------------------------------------- */

/* Replaces compute_entropies_with_probs (src/decoding/sampler.rs:125-154),
 * select_by_entropy_with_distance (sampler.rs:446-493) and the T = 0 branch of
 * sample_from_probs_at_indices (sampler.rs:160-200) with one pass over the logits.
 *   logits      device [rows, ld] of `dtype` (V valid columns per row)
 *   seq_rows    device [nseq + 1] CSR offsets: rows of sequence b are
 *               seq_rows[b] .. seq_rows[b+1]-1 (the mask rows, in mask-row order)
 *   mask_pos    device [rows] logical window position of each mask row
 *   caps        device [nseq] per-sequence max selections (effective cap)
 * Outputs (device): H[rows] entropy of softmax(logits / T) (T scaling only when
 * T > 0 and T != 1), argmax[rows] (ties -> largest index), maxprob[rows],
 * selected[rows] (for sequence b, entries seq_rows[b] .. seq_rows[b]+n_selected[b]-1
 * hold mask-row indices relative to seq_rows[b], ascending logical position),
 * n_selected[nseq].  Any output pointer except selected/n_selected may be NULL. */
WEDLM_API int wedlm_entropy_select(wedlm_ctx* ctx, const void* logits, int dtype, int rows, int V,
                         int ld, float temperature, float tau, float lambda,
                         int nseq, const int32_t* seq_rows, const int32_t* mask_pos,
                         const int32_t* caps, float* H, int32_t* argmax, float* maxprob,
                         int32_t* selected, int32_t* n_selected, void* stream);

/* wedlm_entropy_select without device allocation (no counterpart in the reference,
 * whose selection runs on host vectors).  Same arguments, results and errors as
 * wedlm_entropy_select; the kernels' scratch lives in a fixed 167,936-byte static
 * device array instead of context buffers that grow by cudaMalloc after a device-wide
 * synchronisation.  Limits per call: rows <= 4096, nseq <= 1024 and rows x vocabulary
 * splits <= 8192 (splits = ceil(4 * SMs / rows) capped at ceil(V / 8192), so on a
 * 148-SM B200 rows x splits < rows + 592 and only the first two limits can bind);
 * larger calls fail with WEDLM_ERR_INVALID_ARG and launch nothing.  rows = 0 zeroes
 * n_selected.  The scratch address is looked up per device on the first call and
 * kept for the life of the process, so make one call on each device before any
 * stream capture, and do not reset the device (cudaDeviceReset) between calls.  The
 * scratch is shared by every caller in the process on that device: calls that overlap
 * in time (two streams, or two threads) race on it and must be serialised by the
 * caller. */
WEDLM_API int wedlm_entropy_select_noalloc(wedlm_ctx* ctx, const void* logits, int dtype,
                                           int rows, int V, int ld, float temperature,
                                           float tau, float lambda, int nseq,
                                           const int32_t* seq_rows, const int32_t* mask_pos,
                                           const int32_t* caps, float* H, int32_t* argmax,
                                           float* maxprob, int32_t* selected,
                                           int32_t* n_selected, void* stream);

/* Vocab-shard half of the entropy pass: per-row partial softmax statistics over
 * this shard's columns, global column index = vocab_offset + local column.
 * partials: device [rows * 4] f32 words per row: scaled max m, sum exp(x - m),
 * sum exp(x - m) * (x - m) in log2 units, argmax column (int32 bits; its value is
 * m).  Combine shards with wedlm_entropy_combine. */
WEDLM_API int wedlm_entropy_partials(wedlm_ctx* ctx, const void* logits, int dtype, int rows, int V,
                           int ld, int vocab_offset, float temperature, float* partials,
                           void* stream);
/* Combine [nshards, rows * 4] partials (device) and apply the commit rule. */
WEDLM_API int wedlm_entropy_combine(wedlm_ctx* ctx, const float* partials, int nshards, int rows,
                          float tau, float lambda, int nseq, const int32_t* seq_rows,
                          const int32_t* mask_pos, const int32_t* caps, float* H,
                          int32_t* argmax, float* maxprob, int32_t* selected,
                          int32_t* n_selected, void* stream);

/* Seed of the T > 0 draws of the decode loops (default 0).  The reference samples with
 * the unseeded thread_rng (src/decoding/sampler.rs:180); here the draw of mask row i of
 * sequence b (its index in the call) at step n (1-based) is SplitMix64 chained over
 * (seed, b, n, i), so a seeded run is reproducible.  With T > 0 the selected rows are
 * sampled from softmax(logits / T), by nucleus when top_p < 1 (sampler.rs:306-351);
 * the entropies and the selection are those of the same scaled distribution. */
WEDLM_API int wedlm_set_sampling_seed(wedlm_ctx* ctx, uint64_t seed);

/* ---- multi-GPU: vocabulary-sharded LM head and entropy pass ------------------------- */

/* The reference runs on one device and has no collective; these replace nothing in it.
 * One process per GPU, one context per process.  wedlm_comm_unique_id writes the 128-byte
 * NCCL unique id (ncclGetUniqueId) to `out`; make it on one rank and pass it to every
 * rank.  wedlm_comm_init (collective over nranks) joins the context to an NCCL
 * communicator; the ranks' configs must hold vocab shards that tile [0, V) in rank order
 * (rank r: [vocab_shard_begin, vocab_shard_end)), otherwise WEDLM_ERR_INVALID_ARG.
 * Every wait on the communicator (init, each decode step) gives up after timeout_ms,
 * aborts the communicator and returns WEDLM_ERR_TIMEOUT.  NCCL is loaded at run time
 * (libnccl.so.2; WEDLM_ERR_UNSUPPORTED when it is absent).
 * With a communicator, the decode loops below (wedlm_decode_begin / step, streaming and
 * streaming-batch generation) run the LM head and the entropy pass vocabulary-sharded:
 * each rank decodes its own sequences, the final-normed mask rows and the per-row
 * softmax partials are all-gathered, and each rank applies the commit rule to its rows.
 * They are then collective: every rank calls wedlm_decode_begin, and every rank calls
 * wedlm_decode_step with the same n_steps until it reports n_live == 0 (n_live counts
 * the sequences of all ranks that were live at the step's start).  Block mode and the
 * autoregressive loop need the whole vocabulary on the context.
 * wedlm_comm_destroy (collective) releases the communicator; wedlm_destroy also does. */
WEDLM_API int wedlm_comm_unique_id(void* out, int nbytes);
WEDLM_API int wedlm_comm_init(wedlm_ctx* ctx, const void* unique_id, int rank, int nranks,
                              int timeout_ms);
WEDLM_API int wedlm_comm_destroy(wedlm_ctx* ctx);

/* ---- decode loops --------------------------------------------------------------- */

/* WeDLMDecoder::generate_streaming (src/decoding/wedlm.rs:336-590) on sequence
 * `seq`: prompt prefill, then the commit-before-predict streaming loop with the
 * entropy-EMA dynamic cap.  T must be 0 (greedy).  out_ids (host) receives up to
 * max_new_tokens generated ids; *n_out their count; stats may be NULL. */
WEDLM_API int wedlm_generate_streaming(wedlm_ctx* ctx, int seq, const int32_t* prompt, int n_prompt,
                             int max_new_tokens, int window_size,
                             const wedlm_sampling_params* params, int32_t* out_ids,
                             int32_t* n_out, wedlm_block_stats* stats, void* stream);

/* Step-wise form of the streaming decode for nseq independent sequences (cache slots
 * seq_ids, prompts host [nseq, n_prompt]), stepped together with one forward per step
 * over all live windows.  wedlm_decode_begin prefills the prompts and sets up the
 * windows; wedlm_decode_step runs up to n_steps iterations of the loop body of
 * WeDLMDecoder::generate_streaming (src/decoding/wedlm.rs:380-573), synchronising
 * `stream` once per step, and reports how many sequences are still generating;
 * wedlm_decode_result copies sequence b's generated ids (host, up to max_new_tokens)
 * and stats; wedlm_decode_end releases the session.  One session per context. */
WEDLM_API int wedlm_decode_begin(wedlm_ctx* ctx, int nseq, const int32_t* seq_ids,
                                 const int32_t* prompts, int n_prompt, int max_new_tokens,
                                 int window_size, const wedlm_sampling_params* params,
                                 void* stream);
WEDLM_API int wedlm_decode_step(wedlm_ctx* ctx, int n_steps, int32_t* n_live);
WEDLM_API int wedlm_decode_result(wedlm_ctx* ctx, int b, int32_t* out_ids, int32_t* n_out,
                                  wedlm_block_stats* stats);
/* Steps run so far and the host<->device bytes they moved (inputs up, results down). */
WEDLM_API int wedlm_decode_io_bytes(const wedlm_ctx* ctx, int64_t* steps, int64_t* h2d_bytes,
                                    int64_t* d2h_bytes);
WEDLM_API int wedlm_decode_end(wedlm_ctx* ctx);

/* Block mode, the decoder's secondary path.
 * wedlm_generate_block: WeDLMDecoder::generate_block (src/decoding/wedlm.rs:106-259) on
 * sequence `seq`, whose cache must hold `prefix` (host, n_prefix ids; it is prefilled
 * again when the committed length differs): a block of block_size masks is re-forwarded
 * against the prefix each step (its K/V are not committed) and filled by the
 * entropy / distance rule with the fixed cap params->max_tokens_per_step, until no mask
 * is left or an EOS is produced.  out_block (host, block_size ids) may keep masks.
 * wedlm_commit_block: commit_block_to_cache (wedlm.rs:268-296), the n ids at sequential
 * positions after the committed length.
 * wedlm_generate_with_stats: generate_with_stats (wedlm.rs:610-705) with the adaptive
 * block size and cache refresh; out_ids (host) receives prompt ++ blocks (at most
 * n_prompt + max_new_tokens ids), *n_out their count.  T must be 0. */
WEDLM_API int wedlm_generate_block(wedlm_ctx* ctx, int seq, const int32_t* prefix, int n_prefix,
                                   int block_size, const wedlm_sampling_params* params,
                                   int32_t* out_block, wedlm_block_stats* stats, void* stream);
WEDLM_API int wedlm_commit_block(wedlm_ctx* ctx, int seq, const int32_t* block, int n,
                                 void* stream);
WEDLM_API int wedlm_generate_with_stats(wedlm_ctx* ctx, int seq, const int32_t* prompt,
                                        int n_prompt, int max_new_tokens, int block_size,
                                        const wedlm_sampling_params* params, int32_t* out_ids,
                                        int32_t* n_out, wedlm_block_stats* stats, void* stream);

/* WeDLMEngine::generate_autoregressive (src/engine.rs:160-217), the comparison baseline
 * of the reference's benchmark: one token per forward, the argmax of the last position's
 * logits (T = 0, last maximum on ties), until max_new_tokens or EOS.  The prompt is cached
 * once and every step forwards only the newest token against the cache (the reference
 * recomputes the whole sequence; the logits agree up to rounding).  out_ids (host)
 * receives the generated ids, *n_out their count. */
WEDLM_API int wedlm_generate_autoregressive(wedlm_ctx* ctx, int seq, const int32_t* prompt,
                                            int n_prompt, int max_new_tokens, int32_t* out_ids,
                                            int32_t* n_out, void* stream);

/* Batched streaming decode: nseq independent sequences stepped together, one
 * forward per step over all live windows (data-parallel batching of
 * generate_streaming).  prompts: host [nseq, n_prompt]; out_ids: host
 * [nseq, max_new_tokens]; n_out: host [nseq]; steps_out may be NULL. */
WEDLM_API int wedlm_generate_streaming_batch(wedlm_ctx* ctx, int nseq, const int32_t* prompts,
                                   int n_prompt, int max_new_tokens, int window_size,
                                   const wedlm_sampling_params* params, int32_t* out_ids,
                                   int32_t* n_out, int64_t* steps_out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* WEDLM_B200_H */
