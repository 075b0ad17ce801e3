// Streaming parallel decoding (the host loop of WeDLMDecoder::generate_streaming,
// src/decoding/wedlm.rs:336-590), batched over independent sequences.
//
// Each step, per sequence: count the contiguous filled prefix (commit-before-predict,
// :387-390, mask detected by token id), reorder the window filled-first / masks-last
// with true positions (:397-427, src/decoding/reorder.rs:57-90), run ONE forward over
// every live window, commit the filled prefix (truncate_cache == advance the length,
// :455-465), drain it to the output with the EOS rule and refill the window with masks
// (:470-499), then one fused entropy-select pass over all mask rows applies the
// entropy EMA dynamic cap, the distance-penalised selection and the greedy argmax on
// the device (:511-548), and the selected slots are filled (:553-572).
// Host <-> device per step: one metadata upload, one small result download.
#include <algorithm>
#include <cstring>
#include <vector>

#include "entropy_select.cuh"
#include "model.h"

namespace wedlm {

namespace {

constexpr float kSoftThreshold = 8.0f;  // ENTROPY_SOFT_THRESHOLD, wedlm.rs:29

struct SeqRun {
  int slot = 0;
  std::vector<int> window, wpos;
  int next_pos = 0;
  std::vector<int> out;
  bool done = false;
  wedlm_block_stats st{};
  // per step
  int n_commit = 0, num_filled = 0;
  std::vector<int> mask_logical;
};

// Device buffers of the decode loop (one allocation, carved).
struct DecodeBufs {
  void* logits = nullptr;
  int* seq_rows = nullptr;
  int* mask_pos = nullptr;
  int* caps = nullptr;
  float* running = nullptr;
  float* H = nullptr;
  int* argmax = nullptr;
  int* selected = nullptr;
  int* n_selected = nullptr;
  int* h_in = nullptr;    // pinned: seq_rows | mask_pos | caps
  int* h_out = nullptr;   // pinned: H | argmax | selected | n_selected | err
  uint8_t* block = nullptr;
  int rows = 0, nseq = 0;
  long vshard = 0;
  int esz = 0;
};

Status alloc_bufs(ModelState* m, int rows, int nseq, DecodeBufs* b) {
  b->rows = rows;
  b->nseq = nseq;
  b->vshard = m->vshard;
  b->esz = m->esz;
  const size_t lbytes = ((size_t)rows * m->vshard * m->esz + 255) / 256 * 256;
  const size_t ibytes = (size_t)(nseq + 1 + rows + nseq) * 4;
  const size_t obytes = (size_t)(rows * 3 + nseq + 1) * 4;
  WEDLM_CUDA_TRY(cudaMalloc(&b->block, lbytes + 256 + ibytes + obytes + nseq * 4 + 512));
  uint8_t* p = b->block;
  b->logits = p;
  p += lbytes;
  b->seq_rows = reinterpret_cast<int*>(p);
  b->mask_pos = b->seq_rows + nseq + 1;
  b->caps = b->mask_pos + rows;
  b->running = reinterpret_cast<float*>(b->caps + nseq);
  b->H = b->running + nseq;
  b->argmax = reinterpret_cast<int*>(b->H + rows);
  b->selected = b->argmax + rows;
  b->n_selected = b->selected + rows;
  WEDLM_CUDA_TRY(cudaMallocHost(&b->h_in, ibytes + 64));
  WEDLM_CUDA_TRY(cudaMallocHost(&b->h_out, obytes + 64));
  return Status::ok();
}

void free_bufs(DecodeBufs* b) {
  cudaFree(b->block);
  if (b->h_in) cudaFreeHost(b->h_in);
  if (b->h_out) cudaFreeHost(b->h_out);
  *b = DecodeBufs{};
}

Status generate(wedlm_ctx* ctx, const std::vector<int>& slots, const int32_t* prompts, int n_prompt,
                int max_new, int window_size, const wedlm_sampling_params& prm,
                std::vector<SeqRun>* runs_out, cudaStream_t st) {
  ModelState* m = ctx->model;
  const int B = (int)slots.size();
  WEDLM_CHECK_ARG(B >= 1 && B <= m->max_seqs, "bad number of sequences");
  WEDLM_CHECK_ARG(n_prompt >= 1 && max_new >= 0 && window_size >= 1, "bad lengths");
  WEDLM_CHECK_ARG(window_size <= m->cfg.max_block_tokens,
                  "window larger than the context's max_block_tokens");
  WEDLM_CHECK_ARG(prm.temperature == 0.f,
                  "only temperature 0 (greedy) is supported; the reference samples with an "
                  "unseeded RNG at T > 0");
  WEDLM_CHECK_ARG(n_prompt + max_new + window_size <= m->max_ctx, "prompt + generation exceed max_ctx");
  const int mask = m->cfg.mask_token_id, eos = m->cfg.eos_token_id;

  // 1. cache the prompts (clear_cache + cache_prefix, wedlm.rs:348-349)
  std::vector<SeqRun>& runs = *runs_out;
  runs.assign(B, SeqRun());
  for (int b = 0; b < B; ++b) {
    runs[b].slot = slots[b];
    m->cache_len[slots[b]] = 0;
    m->pending_rows[slots[b]] = 0;
    const int32_t* pr = prompts + (long)b * n_prompt;
    std::vector<int> pos(n_prompt);
    for (int off = 0; off < n_prompt; off += m->max_rows) {
      const int c = std::min(m->max_rows, n_prompt - off);
      pos.resize(c);
      for (int j = 0; j < c; ++j) pos[j] = off + j;
      std::vector<SeqSlice> sl(1);
      sl[0].slot = slots[b];
      sl[0].rows = c;
      sl[0].logit_begin = c;
      WEDLM_TRY(model_forward(ctx, sl, pr + off, pos.data(), nullptr, nullptr, m->dt, nullptr, st));
      m->cache_len[slots[b]] += c;
    }
    runs[b].st.prefix_cached = 1;
    const int init = std::min(window_size, max_new);
    runs[b].window.assign(init, mask);
    runs[b].wpos.resize(init);
    for (int j = 0; j < init; ++j) runs[b].wpos[j] = n_prompt + j;
    runs[b].next_pos = n_prompt + init;
    if (max_new == 0) runs[b].done = true;
  }

  DecodeBufs bufs;
  WEDLM_TRY(alloc_bufs(m, B * window_size, B, &bufs));
  struct Guard {
    DecodeBufs* b;
    ~Guard() { free_bufs(b); }
  } guard{&bufs};
  {
    std::vector<float> r0(B, prm.entropy_threshold);  // running entropy starts at tau
    WEDLM_CUDA_TRY(cudaMemcpyAsync(bufs.running, r0.data(), B * 4, cudaMemcpyHostToDevice, st));
    WEDLM_CUDA_TRY(cudaStreamSynchronize(st));
  }

  std::vector<int> tok, pos;
  std::vector<SeqSlice> slices;
  std::vector<int> live;
  while (true) {
    // ---- build the step (steps A-B) ----
    tok.clear();
    pos.clear();
    slices.clear();
    live.clear();
    for (int b = 0; b < B; ++b) {
      SeqRun& R = runs[b];
      if (R.done) continue;
      if ((int)R.out.size() >= max_new || R.window.empty()) {
        R.done = true;
        continue;
      }
      R.st.steps += 1;
      int nc = 0;
      while (nc < (int)R.window.size() && R.window[nc] != mask) ++nc;
      R.n_commit = nc;
      R.mask_logical.clear();
      for (int i = 0; i < (int)R.window.size(); ++i)
        if (R.window[i] == mask) R.mask_logical.push_back(i);
      R.num_filled = (int)R.window.size() - (int)R.mask_logical.size();
      for (int i = 0; i < (int)R.window.size(); ++i)
        if (R.window[i] != mask) {
          tok.push_back(R.window[i]);
          pos.push_back(R.wpos[i]);
        }
      for (int i : R.mask_logical) {
        tok.push_back(R.window[i]);
        pos.push_back(R.wpos[i]);
      }
      SeqSlice sl;
      sl.slot = R.slot;
      sl.rows = (int)R.window.size();
      sl.logit_begin = R.num_filled;
      slices.push_back(sl);
      live.push_back(b);
    }
    if (live.empty()) break;

    // ---- step C: one forward over every live window ----
    int nl = 0;
    WEDLM_TRY(model_forward(ctx, slices, tok.data(), pos.data(), nullptr, bufs.logits, m->dt, &nl, st));

    // ---- steps D, D': commit, drain, refill ----
    for (int b : live) {
      SeqRun& R = runs[b];
      const int remaining = std::max(max_new - (int)R.out.size(), 0);
      const int nc = std::min(R.n_commit, remaining);
      R.n_commit = nc;
      m->cache_len[R.slot] += nc;  // truncate_cache(committed_len + n_commit)
      m->pending_rows[R.slot] = 0;
      if (nc > 0) {
        std::vector<int> toks(R.window.begin(), R.window.begin() + nc);
        R.window.erase(R.window.begin(), R.window.begin() + nc);
        R.wpos.erase(R.wpos.begin(), R.wpos.begin() + nc);
        int add = nc;
        bool has_eos = false;
        for (int i = 0; i < nc; ++i)
          if (toks[i] == eos) {
            add = i + 1;
            has_eos = true;
            break;
          }
        R.out.insert(R.out.end(), toks.begin(), toks.begin() + add);
        R.st.tokens_generated += add;
        if (add < nc) m->cache_len[R.slot] -= nc - add;  // nothing after EOS is kept
        if (has_eos) {
          R.done = true;
          continue;
        }
        for (int i = 0; i < nc; ++i) {
          if ((int)R.out.size() + (int)R.window.size() >= max_new) break;
          R.window.push_back(mask);
          R.wpos.push_back(R.next_pos++);
        }
      }
    }

    // ---- step E: fused entropy / EMA cap / selection / argmax over the mask rows ----
    const int nb = (int)live.size();
    int* hi = bufs.h_in;
    int rr = 0;
    for (int k = 0; k < nb; ++k) {
      const SeqRun& R = runs[live[k]];
      hi[k] = rr;
      for (int i : R.mask_logical) hi[nb + 1 + rr++] = i;
    }
    hi[nb] = rr;
    // rows of every live sequence are present in the logits in slice order; sequences
    // that ended on EOS this step still own rows (their selection is ignored)
    for (int k = 0; k < nb; ++k) hi[nb + 1 + rr + k] = prm.max_tokens_per_step;
    if (rr == 0) continue;
    WEDLM_CUDA_TRY(cudaMemcpyAsync(bufs.seq_rows, hi, (size_t)(nb + 1) * 4, cudaMemcpyHostToDevice, st));
    WEDLM_CUDA_TRY(cudaMemcpyAsync(bufs.mask_pos, hi + nb + 1, (size_t)rr * 4, cudaMemcpyHostToDevice, st));
    WEDLM_CUDA_TRY(cudaMemcpyAsync(bufs.caps, hi + nb + 1 + rr, (size_t)nb * 4, cudaMemcpyHostToDevice, st));
    // the running-entropy slots follow live order: keep them aligned with sequence ids
    EntropyArgs A;
    A.logits = bufs.logits;
    A.dtype = m->dt;
    A.rows = rr;
    A.V = m->vshard;
    A.ld = m->vshard;
    A.temperature = prm.temperature;
    A.tau = prm.entropy_threshold;
    A.lambda = prm.distance_penalty;
    A.nseq = nb;
    A.seq_rows = bufs.seq_rows;
    A.mask_pos = bufs.mask_pos;
    A.caps = bufs.caps;
    A.running = bufs.running;
    A.H = bufs.H;
    A.argmax = bufs.argmax;
    A.selected = bufs.selected;
    A.n_selected = bufs.n_selected;
    // live sequences are a prefix-stable subset: compact the running slots when needed
    EntropyPlan ep = plan_entropy(rr, m->vshard, m->dt, ctx->num_sms);
    WEDLM_TRY(ensure_entropy_scratch(ctx, rr, nb, (long)rr * ep.splits * 4));
    WEDLM_TRY(run_entropy_select(A, ctx->ent, ctx->num_sms, st));
    int* ho = bufs.h_out;
    WEDLM_CUDA_TRY(cudaMemcpyAsync(ho, bufs.H, (size_t)rr * 4, cudaMemcpyDeviceToHost, st));
    WEDLM_CUDA_TRY(cudaMemcpyAsync(ho + rr, bufs.argmax, (size_t)rr * 4, cudaMemcpyDeviceToHost, st));
    WEDLM_CUDA_TRY(cudaMemcpyAsync(ho + 2 * rr, bufs.selected, (size_t)rr * 4, cudaMemcpyDeviceToHost, st));
    WEDLM_CUDA_TRY(cudaMemcpyAsync(ho + 3 * rr, bufs.n_selected, (size_t)nb * 4, cudaMemcpyDeviceToHost, st));
    WEDLM_CUDA_TRY(cudaMemcpyAsync(ho + 3 * rr + nb, ctx->dev_err, 4, cudaMemcpyDeviceToHost, st));
    WEDLM_CUDA_TRY(cudaStreamSynchronize(st));
    if (ho[3 * rr + nb] != 0) {
      cudaMemsetAsync(ctx->dev_err, 0, 4, st);
      return Status::err(WEDLM_ERR_TIMEOUT, "a device-side wait gave up during the decode step");
    }
    const float* Hh = reinterpret_cast<const float*>(ho);
    for (int k = 0; k < nb; ++k) {
      SeqRun& R = runs[live[k]];
      const int r0 = hi[k];
      if (R.done) continue;
      const int ns = ho[3 * rr + k];
      for (int i = 0; i < ns; ++i) {
        const int sel = ho[2 * rr + r0 + i];
        const int pre = R.mask_logical[sel];
        const int post = std::max(pre - R.n_commit, 0);
        if (post < (int)R.window.size()) {
          R.window[post] = ho[rr + r0 + sel];
          const float e = Hh[r0 + sel];
          R.st.avg_entropy += e;
          if (e > R.st.max_entropy) R.st.max_entropy = e;
          if (e > kSoftThreshold) R.st.high_entropy_count += 1;
        }
      }
    }
    // keep each sequence's running entropy in its own slot: sequences that finished are
    // removed from `live` in order, so shift the running values down accordingly
    bool shift = false;
    for (int k = 0; k < nb; ++k)
      if (runs[live[k]].done || (int)runs[live[k]].out.size() >= max_new) shift = true;
    if (shift) {
      std::vector<float> rv(nb);
      WEDLM_CUDA_TRY(cudaMemcpy(rv.data(), bufs.running, nb * 4, cudaMemcpyDeviceToHost));
      std::vector<float> keep;
      for (int k = 0; k < nb; ++k)
        if (!(runs[live[k]].done || (int)runs[live[k]].out.size() >= max_new)) keep.push_back(rv[k]);
      if (!keep.empty())
        WEDLM_CUDA_TRY(cudaMemcpy(bufs.running, keep.data(), keep.size() * 4, cudaMemcpyHostToDevice));
    }
  }
  for (SeqRun& R : runs) {
    if (R.st.tokens_generated > 0) {
      R.st.avg_entropy /= (float)R.st.tokens_generated;
      R.st.avg_confidence = std::max(1.0f - R.st.avg_entropy / 10.0f, 0.0f);
    }
  }
  return Status::ok();
}

}  // namespace

}  // namespace wedlm

extern "C" {

int wedlm_generate_streaming(wedlm_ctx* ctx, int seq, const int32_t* prompt, int n_prompt,
                             int max_new_tokens, int window_size,
                             const wedlm_sampling_params* params, int32_t* out_ids,
                             int32_t* n_out, wedlm_block_stats* stats, void* stream) {
  if (!ctx) return WEDLM_ERR_INVALID_ARG;
  if (!ctx->model) return ctx->fail(wedlm::Status::err(WEDLM_ERR_STATE, "context has no model"));
  if (!prompt || !params || !out_ids || !n_out)
    return ctx->fail(wedlm::Status::err(WEDLM_ERR_INVALID_ARG, "NULL argument"));
  if (seq < 0 || seq >= ctx->model->max_seqs)
    return ctx->fail(wedlm::Status::err(WEDLM_ERR_INVALID_ARG, "bad seq"));
  cudaSetDevice(ctx->device);
  cudaStream_t st = (cudaStream_t)stream;  // NULL: the legacy default stream
  std::vector<wedlm::SeqRun> runs;
  wedlm::Status s = wedlm::generate(ctx, {seq}, prompt, n_prompt, max_new_tokens, window_size,
                                    *params, &runs, st);
  if (!s.good()) return ctx->fail(s);
  const wedlm::SeqRun& R = runs[0];
  for (size_t i = 0; i < R.out.size(); ++i) out_ids[i] = R.out[i];
  *n_out = (int32_t)R.out.size();
  if (stats) *stats = R.st;
  return WEDLM_OK;
}

int wedlm_generate_streaming_batch(wedlm_ctx* ctx, int nseq, const int32_t* prompts, int n_prompt,
                                   int max_new_tokens, int window_size,
                                   const wedlm_sampling_params* params, int32_t* out_ids,
                                   int32_t* n_out, int64_t* steps_out, void* stream) {
  if (!ctx) return WEDLM_ERR_INVALID_ARG;
  if (!ctx->model) return ctx->fail(wedlm::Status::err(WEDLM_ERR_STATE, "context has no model"));
  if (!prompts || !params || !out_ids || !n_out || nseq < 1 || nseq > ctx->model->max_seqs)
    return ctx->fail(wedlm::Status::err(WEDLM_ERR_INVALID_ARG, "bad batch arguments"));
  cudaSetDevice(ctx->device);
  cudaStream_t st = (cudaStream_t)stream;  // NULL: the legacy default stream
  std::vector<int> slots(nseq);
  for (int b = 0; b < nseq; ++b) slots[b] = b;
  std::vector<wedlm::SeqRun> runs;
  wedlm::Status s = wedlm::generate(ctx, slots, prompts, n_prompt, max_new_tokens, window_size,
                                    *params, &runs, st);
  if (!s.good()) return ctx->fail(s);
  for (int b = 0; b < nseq; ++b) {
    const wedlm::SeqRun& R = runs[b];
    for (size_t i = 0; i < R.out.size(); ++i) out_ids[(long)b * max_new_tokens + i] = R.out[i];
    n_out[b] = (int32_t)R.out.size();
    if (steps_out) steps_out[b] = R.st.steps;
  }
  return WEDLM_OK;
}

}  // extern "C"
