// The device-resident streaming loop (decode_loop.cu): the per-step bookkeeping of
// WeDLMDecoder::generate_streaming (src/decoding/wedlm.rs:380-573) kept on the device, so
// that a step is a fixed sequence of launches -- bookkeeping, forward, entropy / selection
// (and T > 0 draws), bookkeeping -- with no host round trip, captured once as a CUDA graph
// and replayed per step.
//   prep (before the forward), per sequence: the end test of the loop head (:380-385), the
//     contiguous filled prefix (commit-before-predict, :387-390), the mask list and the
//     filled-first / masks-last reordering with true positions (:397-427); the forward's
//     metadata, the selection inputs (mask rows in sequence order, window-logical mask
//     positions, caps, draw keys) and the attention rows of the step.
//   post (after the selection): commit of the filled prefix (truncate_cache, :455-465),
//     the drain to the output with the EOS rule and the refill with masks (:470-499), the
//     fill of the picked mask slots and the entropy statistics (:553-572), and the number
//     of sequences still generating.
// Every sequence keeps a window of W rows in the forward (rows past its window length, and
// all rows of a finished sequence, are padding rows that nothing reads), so every launch
// has the same shape each step.  The host reads one int per step (the live count).
#pragma once

#include <vector>

#include "common.cuh"
#include "../../include/wedlm_b200.h"

struct wedlm_ctx;

namespace wedlm {

struct DeviceLoop;

struct LoopInit {
  int W = 0;             // window capacity (the session's window size)
  int max_new = 0, n_prompt = 0;
  std::vector<int> slots;            // cache slot of each sequence
  wedlm_sampling_params prm{};
  void* logits = nullptr;            // [B * W, vshard] model dtype (the session's buffer)
  float* running = nullptr;          // [B] entropy EMA (the session's buffer, set to tau)
  cudaStream_t st = nullptr;
};

struct LoopSeqResult {
  std::vector<int> out;
  bool done = false;
  int64_t steps = 0;
  int tokens_generated = 0, high_entropy_count = 0;
  float entropy_sum = 0.f, entropy_max = 0.f;
  int cache_len = 0;
};

// Whether this context runs the device loop for such a session (one GPU, no
// vocabulary shard; WEDLM_DEVICE_LOOP=0 selects the host loop).
bool device_loop_eligible(wedlm_ctx* ctx, int B, int W, int n_prompt, int max_new);
// The prompts are cached and the windows start as all masks (decode_begin's state).
Status loop_create(wedlm_ctx* ctx, const LoopInit& init, DeviceLoop** out);
// Up to n_steps steps, stopping after the step that leaves no live sequence (at most one
// step more is enqueued before the host sees that; it changes nothing).  *live = live
// sequences after the last step; *steps_total = steps since loop_create that had a live
// sequence (-1 when no step ran).
Status loop_run(wedlm_ctx* ctx, DeviceLoop* L, int n_steps, int* live, int64_t* steps_total);
// Download the outputs, statistics and committed cache lengths of every sequence.
Status loop_results(wedlm_ctx* ctx, DeviceLoop* L, std::vector<LoopSeqResult>* res);
// Bytes moved between host and device by the loop so far.
void loop_io_bytes(const DeviceLoop* L, int64_t* h2d, int64_t* d2h);
void loop_free(DeviceLoop* L);

}  // namespace wedlm
