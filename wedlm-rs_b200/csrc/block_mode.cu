// Block-mode decoding, the decoder's secondary path: WeDLMDecoder::generate_block,
// commit_block_to_cache and generate_with_stats (src/decoding/wedlm.rs:106-296,
// 610-714).  A block of masks is re-forwarded against the fixed prefix cache each step
// (its K/V are written past the committed length and never committed), the fused
// entropy-select picks the slots to fill with the fixed cap, and the finished block is
// forwarded once more at sequential positions to enter the cache.  generate_with_stats
// adapts the block size to the block's entropies and refreshes the cache.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <vector>

#include "entropy_select.cuh"
#include "model.h"
#include "sample.cuh"

namespace wedlm {
namespace {

constexpr float kSoftEntropy = 8.0f;    // ENTROPY_SOFT_THRESHOLD, wedlm.rs:29
constexpr float kHardEntropy = 12.0f;   // ENTROPY_HARD_THRESHOLD, wedlm.rs:32
constexpr int kMaxCachedLength = 16384; // MAX_CACHED_LENGTH, wedlm.rs:35
constexpr int kCacheCheckInterval = 32; // CACHE_CHECK_INTERVAL, wedlm.rs:38

// Device / pinned buffers of one block-mode call.
struct BlockBuffers {
  void* logits = nullptr;  // [cap, vshard] model dtype
  int* d_io = nullptr;     // in: seq_rows[2], mask_pos[cap], caps[1] | out: H, argmax, selected [cap], n[1]
  int* h_io = nullptr;
  int cap = 0;
  ~BlockBuffers() {
    cudaFree(logits);
    cudaFree(d_io);
    if (h_io) cudaFreeHost(h_io);
  }
  Status alloc(const ModelState* m, int block) {
    cap = block;
    WEDLM_CUDA_TRY(cudaMalloc(&logits, (size_t)block * m->vshard * m->esz + 256));
    // + [sequence key, step] of the T > 0 draws after the outputs
    const size_t ints = 3 + (size_t)block + 3 * (size_t)block + 1 + 2;
    WEDLM_CUDA_TRY(cudaMalloc(&d_io, ints * 4));
    WEDLM_CUDA_TRY(cudaMallocHost(&h_io, ints * 4));
    return Status::ok();
  }
};

Status prefill_ids(wedlm_ctx* ctx, int slot, const int32_t* ids, int n, cudaStream_t st) {
  ModelState* m = ctx->model;
  m->cache_len[slot] = 0;
  m->pending_rows[slot] = 0;
  std::vector<int> pos;
  for (int off = 0; off < n; off += m->max_rows) {
    const int c = std::min(m->max_rows, n - off);
    pos.resize(c);
    for (int j = 0; j < c; ++j) pos[j] = off + j;
    std::vector<SeqSlice> sl(1);
    sl[0].slot = slot;
    sl[0].rows = c;
    sl[0].logit_begin = c;
    WEDLM_TRY(model_forward(ctx, sl, ids + off, pos.data(), nullptr, nullptr, m->dt, nullptr, st));
    m->cache_len[slot] += c;
  }
  return Status::ok();
}

// generate_block (wedlm.rs:106-259) for the sequence in `slot`, whose cache must hold
// the n_prefix tokens of `prefix` (re-prefilled otherwise, :127-135).
Status generate_block(wedlm_ctx* ctx, int slot, const int32_t* prefix, int n_prefix, int bs,
                      const wedlm_sampling_params& prm, BlockBuffers& B, std::vector<int>* block,
                      wedlm_block_stats* stats, cudaStream_t st) {
  ModelState* m = ctx->model;
  const int mask = m->cfg.mask_token_id, eos = m->cfg.eos_token_id;
  wedlm_block_stats s{};
  s.prefix_cached = 1;
  if (m->cache_len[slot] != n_prefix) WEDLM_TRY(prefill_ids(ctx, slot, prefix, n_prefix, st));
  block->assign(bs, mask);
  std::vector<int> mask_pos(bs);
  for (int i = 0; i < bs; ++i) mask_pos[i] = i;
  std::vector<int> tok, pos, orig;
  while (!mask_pos.empty()) {
    s.steps += 1;
    // filled-first / masks-last reorder with true positions (reorder.rs:57-90)
    tok.clear();
    pos.clear();
    orig.clear();
    std::vector<char> is_mask(bs, 0);
    for (int p : mask_pos) is_mask[p] = 1;
    for (int i = 0; i < bs; ++i)
      if (!is_mask[i]) {
        tok.push_back((*block)[i]);
        pos.push_back(n_prefix + i);
      }
    const int nf = (int)tok.size();
    for (int p : mask_pos) {
      tok.push_back((*block)[p]);
      pos.push_back(n_prefix + p);
      orig.push_back(p);
    }
    const int nm = (int)mask_pos.size();
    std::vector<SeqSlice> sl(1);
    sl[0].slot = slot;
    sl[0].rows = bs;
    sl[0].logit_begin = nf;
    int nl = 0;
    WEDLM_TRY(model_forward(ctx, sl, tok.data(), pos.data(), nullptr, B.logits, m->dt, &nl, st));
    m->pending_rows[slot] = 0;  // the block K/V are not kept (wedlm.rs:166-174)
    // entropy / selection (fixed cap) / greedy argmax over the mask rows
    int* hi = B.h_io;
    hi[0] = 0;
    hi[1] = nm;
    for (int i = 0; i < nm; ++i) hi[2 + i] = orig[i];
    hi[2 + nm] = prm.max_tokens_per_step;
    const int nin = 3 + nm;
    WEDLM_CUDA_TRY(cudaMemcpyAsync(B.d_io, hi, (size_t)nin * 4, cudaMemcpyHostToDevice, st));
    int* dout = B.d_io + 3 + B.cap;
    EntropyArgs A;
    A.logits = B.logits;
    A.dtype = m->dt;
    A.rows = nm;
    A.V = m->vshard;
    A.ld = m->vshard;
    A.temperature = prm.temperature;
    A.tau = prm.entropy_threshold;
    A.lambda = prm.distance_penalty;
    A.nseq = 1;
    A.seq_rows = B.d_io;
    A.mask_pos = B.d_io + 2;
    A.caps = B.d_io + 2 + nm;
    A.H = reinterpret_cast<float*>(dout);
    A.argmax = dout + B.cap;
    A.selected = dout + 2 * B.cap;
    A.n_selected = dout + 3 * B.cap;
    EntropyPlan ep = plan_entropy(nm, m->vshard, m->dt, ctx->num_sms);
    WEDLM_TRY(ensure_entropy_scratch(ctx, nm, 1, (long)nm * ep.splits * 4));
    WEDLM_TRY(run_entropy_select(A, ctx->ent, ctx->num_sms, st));
    if (prm.temperature > 0.f) {
      // T > 0: the selected rows are drawn (sample_from_probs / sample_nucleus) in place
      // of their argmax, keyed by (seed, 0, step, mask row)
      int* hkv = B.h_io + 4 + 4 * B.cap;
      int* dkv = B.d_io + 4 + 4 * B.cap;
      hkv[0] = 0;
      hkv[1] = (int)s.steps;
      WEDLM_CUDA_TRY(cudaMemcpyAsync(dkv, hkv, 2 * sizeof(int), cudaMemcpyHostToDevice, st));
      SampleArgs sa;
      sa.logits = B.logits;
      sa.dtype = m->dt;
      sa.rows = nm;
      sa.V = m->vshard;
      sa.ld = m->vshard;
      sa.temperature = prm.temperature;
      sa.top_p = prm.top_p;
      sa.seed = ctx->sample_seed;
      sa.nseq = 1;
      sa.seq_rows = A.seq_rows;
      sa.selected = A.selected;
      sa.n_selected = A.n_selected;
      sa.seq_key = dkv;
      sa.seq_step = dkv + 1;
      sa.tokens = A.argmax;
      WEDLM_TRY(run_sample(sa, st));
    }
    int* ho = B.h_io + 3 + B.cap;
    WEDLM_CUDA_TRY(cudaMemcpyAsync(ho, dout, (size_t)(3 * B.cap + 1) * 4, cudaMemcpyDeviceToHost, st));
    WEDLM_CUDA_TRY(cudaStreamSynchronize(st));
    WEDLM_TRY(check_device_error(ctx, st));
    const float* H = reinterpret_cast<const float*>(ho);
    const int* am = ho + B.cap;
    const int* sel = ho + 2 * B.cap;
    const int nsel = ho[3 * B.cap];
    if (nsel == 0) break;
    bool hit_eos = false;
    std::vector<char> filled(bs, 0);
    for (int i = 0; i < nsel; ++i) {
      const int r = sel[i];
      const int p = orig[r];
      (*block)[p] = am[r];
      filled[p] = 1;
      const float e = H[r];
      s.avg_entropy += e;
      s.max_entropy = std::max(s.max_entropy, e);
      if (e > kSoftEntropy) s.high_entropy_count += 1;
      if (am[r] == eos) hit_eos = true;
    }
    s.tokens_generated += nsel;
    std::vector<int> rest;
    for (int p : mask_pos)
      if (!filled[p]) rest.push_back(p);
    mask_pos.swap(rest);
    if (hit_eos) break;
  }
  if (s.tokens_generated > 0) {
    s.avg_entropy /= (float)s.tokens_generated;
    s.avg_confidence = std::max(1.0f - s.avg_entropy / 10.0f, 0.0f);
  }
  *stats = s;
  return Status::ok();
}

// commit_block_to_cache (wedlm.rs:268-296): the block at sequential positions.
Status commit_block(wedlm_ctx* ctx, int slot, const int32_t* blk, int n, cudaStream_t st) {
  ModelState* m = ctx->model;
  std::vector<int> pos(n);
  for (int i = 0; i < n; ++i) pos[i] = m->cache_len[slot] + i;
  for (int off = 0; off < n;) {
    const int c = std::min(m->max_rows, n - off);
    std::vector<SeqSlice> sl(1);
    sl[0].slot = slot;
    sl[0].rows = c;
    sl[0].logit_begin = c;
    WEDLM_TRY(model_forward(ctx, sl, blk + off, pos.data() + off, nullptr, nullptr, m->dt, nullptr, st));
    m->cache_len[slot] += c;
    m->pending_rows[slot] = 0;
    off += c;
  }
  return Status::ok();
}

// generate_with_stats (wedlm.rs:610-705): blocks with adaptive size and cache refresh.
Status generate_with_stats(wedlm_ctx* ctx, int slot, const int32_t* prompt, int n_prompt,
                           int max_new, int block_size, const wedlm_sampling_params& prm,
                           std::vector<int>* all_ids, wedlm_block_stats* stats, cudaStream_t st) {
  ModelState* m = ctx->model;
  const int eos = m->cfg.eos_token_id;
  all_ids->assign(prompt, prompt + n_prompt);
  BlockBuffers B;
  WEDLM_TRY(B.alloc(m, block_size));
  WEDLM_TRY(prefill_ids(ctx, slot, prompt, n_prompt, st));  // cache_prefix of the prompt
  int total = 0, since_check = 0, eff = block_size;
  wedlm_block_stats cum{};
  std::vector<int> blk;
  while (total < max_new) {
    const int cur = std::min(max_new - total, eff);
    wedlm_block_stats bs{};
    WEDLM_TRY(generate_block(ctx, slot, all_ids->data(), (int)all_ids->size(), cur, prm, B, &blk,
                             &bs, st));
    cum.steps += bs.steps;
    const int64_t prev = cum.tokens_generated;
    cum.tokens_generated += bs.tokens_generated;
    cum.high_entropy_count += bs.high_entropy_count;
    cum.max_entropy = std::max(cum.max_entropy, bs.max_entropy);
    if (cum.tokens_generated > 0)
      cum.avg_entropy = (float)((cum.avg_entropy * (double)prev +
                                 (double)bs.avg_entropy * (double)bs.tokens_generated) /
                                (double)cum.tokens_generated);
    // adaptive block size (wedlm.rs:640-660)
    if (bs.max_entropy > kHardEntropy) {
      eff = 1;
      cum.block_size_reductions += 1;
    } else if (bs.max_entropy > kSoftEntropy) {
      eff = std::max(eff / 2, 1);
      cum.block_size_reductions += 1;
    } else if (eff < block_size && bs.avg_entropy < kSoftEntropy / 2.0f) {
      eff = std::min(eff * 2, block_size);
    }
    all_ids->insert(all_ids->end(), blk.begin(), blk.end());
    total += cur;
    since_check += 1;
    if (std::find(blk.begin(), blk.end(), eos) != blk.end()) break;
    WEDLM_TRY(commit_block(ctx, slot, blk.data(), (int)blk.size(), st));
    // cache refresh (wedlm.rs:676-700, 710-714)
    if (m->cache_len[slot] > kMaxCachedLength) {
      WEDLM_TRY(prefill_ids(ctx, slot, all_ids->data(), (int)all_ids->size(), st));
      cum.cache_refreshes += 1;
    }
    if (since_check >= kCacheCheckInterval) {
      since_check = 0;
      if (cum.high_entropy_count > kCacheCheckInterval / 2) {
        WEDLM_TRY(prefill_ids(ctx, slot, all_ids->data(), (int)all_ids->size(), st));
        cum.cache_refreshes += 1;
        cum.high_entropy_count = 0;
      }
    }
  }
  cum.avg_confidence = std::max(1.0f - cum.avg_entropy / 10.0f, 0.0f);
  cum.prefix_cached = 1;
  *stats = cum;
  return Status::ok();
}

Status check_block_args(wedlm_ctx* ctx, int seq, int block_size, const wedlm_sampling_params* prm) {
  ModelState* m = ctx->model;
  WEDLM_CHECK_ARG(seq >= 0 && seq < m->max_seqs, "bad sequence slot");
  WEDLM_CHECK_ARG(block_size >= 1 && block_size <= m->cfg.max_block_tokens,
                  "block_size must be 1 .. max_block_tokens");
  WEDLM_CHECK_ARG(prm != nullptr, "params is NULL");
  WEDLM_CHECK_ARG(prm->temperature >= 0.f && std::isfinite(prm->temperature),
                  "temperature must be >= 0");
  WEDLM_CHECK_ARG(prm->temperature == 0.f || prm->top_p > 0.f, "top_p must be > 0");
  return Status::ok();
}

// needs_vocab: the call projects and selects over the whole vocabulary on this context.
int block_guard(wedlm_ctx* ctx, bool needs_vocab = true) {
  if (!ctx) return WEDLM_ERR_INVALID_ARG;
  if (!ctx->model) return ctx->fail(Status::err(WEDLM_ERR_STATE, "context has no model"));
  cudaError_t e = cudaSetDevice(ctx->device);
  if (e != cudaSuccess) return ctx->fail(Status::err(WEDLM_ERR_CUDA, cudaGetErrorString(e)));
  if (ctx->session) return ctx->fail(Status::err(WEDLM_ERR_STATE, "a decode session is active"));
  if (needs_vocab && ctx->model->vshard != ctx->model->V)
    return ctx->fail(Status::err(WEDLM_ERR_STATE,
                                 "this context holds a vocabulary shard; block mode and the "
                                 "autoregressive loop need the whole vocabulary"));
  return WEDLM_OK;
}

}  // namespace
}  // namespace wedlm

using wedlm::Status;

extern "C" int wedlm_generate_block(wedlm_ctx* ctx, int seq, const int32_t* prefix, int n_prefix,
                                    int block_size, const wedlm_sampling_params* params,
                                    int32_t* out_block, wedlm_block_stats* stats, void* stream) {
  if (int rc = wedlm::block_guard(ctx)) return rc;
  Status s = wedlm::check_block_args(ctx, seq, block_size, params);
  if (!s.good()) return ctx->fail(s);
  if (!prefix || n_prefix < 1 || !out_block ||
      n_prefix + block_size > ctx->model->max_ctx)
    return ctx->fail(Status::err(WEDLM_ERR_INVALID_ARG, "bad prefix / block length"));
  wedlm::BlockBuffers B;
  s = B.alloc(ctx->model, block_size);
  std::vector<int> blk;
  wedlm_block_stats bs{};
  if (s.good())
    s = wedlm::generate_block(ctx, seq, prefix, n_prefix, block_size, *params, B, &blk, &bs,
                              (cudaStream_t)stream);
  if (!s.good()) return ctx->fail(s);
  std::copy(blk.begin(), blk.end(), out_block);
  if (stats) *stats = bs;
  return WEDLM_OK;
}

extern "C" int wedlm_commit_block(wedlm_ctx* ctx, int seq, const int32_t* block, int n,
                                  void* stream) {
  if (int rc = wedlm::block_guard(ctx, false)) return rc;
  if (seq < 0 || seq >= ctx->model->max_seqs || !block || n < 1 ||
      ctx->model->cache_len[seq] + n > ctx->model->max_ctx)
    return ctx->fail(Status::err(WEDLM_ERR_INVALID_ARG, "bad sequence / block"));
  Status s = wedlm::commit_block(ctx, seq, block, n, (cudaStream_t)stream);
  return s.good() ? WEDLM_OK : ctx->fail(s);
}

extern "C" int wedlm_generate_with_stats(wedlm_ctx* ctx, int seq, const int32_t* prompt,
                                         int n_prompt, int max_new_tokens, int block_size,
                                         const wedlm_sampling_params* params, int32_t* out_ids,
                                         int32_t* n_out, wedlm_block_stats* stats, void* stream) {
  if (int rc = wedlm::block_guard(ctx)) return rc;
  Status s = wedlm::check_block_args(ctx, seq, block_size, params);
  if (!s.good()) return ctx->fail(s);
  if (!prompt || n_prompt < 1 || max_new_tokens < 0 || !out_ids || !n_out ||
      n_prompt + max_new_tokens + block_size > ctx->model->max_ctx)
    return ctx->fail(Status::err(WEDLM_ERR_INVALID_ARG, "bad prompt / lengths (max_ctx)"));
  std::vector<int> ids;
  wedlm_block_stats st{};
  s = wedlm::generate_with_stats(ctx, seq, prompt, n_prompt, max_new_tokens, block_size, *params,
                                 &ids, &st, (cudaStream_t)stream);
  if (!s.good()) return ctx->fail(s);
  std::copy(ids.begin(), ids.end(), out_ids);
  *n_out = (int32_t)ids.size();
  if (stats) *stats = st;
  return WEDLM_OK;
}


// ---- autoregressive baseline -------------------------------------------------------------
// WeDLMEngine::generate_autoregressive (src/engine.rs:160-217): one token per forward, the
// argmax of the last position's logits (T = 0), until max_new tokens or EOS.  The
// reference re-runs the whole sequence without a cache each token; here the prompt is
// cached once and each step forwards only the newest token against the cache, which gives
// the same logits up to rounding.  The argmax takes the last maximum (ties are not pinned
// by the reference, whose argmax runs in candle).
extern "C" int wedlm_generate_autoregressive(wedlm_ctx* ctx, int seq, const int32_t* prompt,
                                             int n_prompt, int max_new_tokens, int32_t* out_ids,
                                             int32_t* n_out, void* stream) {
  using namespace wedlm;
  if (int rc = block_guard(ctx)) return rc;
  ModelState* m = ctx->model;
  if (seq < 0 || seq >= m->max_seqs || !prompt || n_prompt < 1 || max_new_tokens < 0 || !out_ids ||
      !n_out || n_prompt + max_new_tokens > m->max_ctx)
    return ctx->fail(Status::err(WEDLM_ERR_INVALID_ARG, "bad sequence / prompt / lengths (max_ctx)"));
  cudaStream_t st = (cudaStream_t)stream;
  const int eos = m->cfg.eos_token_id;
  BlockBuffers B;
  Status s = B.alloc(m, 1);
  if (s.good() && n_prompt > 1) s = prefill_ids(ctx, seq, prompt, n_prompt - 1, st);
  if (s.good() && n_prompt == 1) {
    m->cache_len[seq] = 0;
    m->pending_rows[seq] = 0;
  }
  int last = prompt[n_prompt - 1];
  int n = 0;
  while (s.good() && n < max_new_tokens) {
    std::vector<SeqSlice> sl(1);
    sl[0].slot = seq;
    sl[0].rows = 1;
    sl[0].logit_begin = 0;
    const int pos = m->cache_len[seq];
    int nl = 0;
    s = model_forward(ctx, sl, &last, &pos, nullptr, B.logits, m->dt, &nl, st);
    if (!s.good()) break;
    m->cache_len[seq] += 1;  // the token's K/V enter the cache
    m->pending_rows[seq] = 0;
    // argmax of the one row through the fused pass (its selection part is unused)
    int* hi = B.h_io;
    hi[0] = 0;
    hi[1] = 1;
    hi[2] = 0;
    hi[3] = 1;
    s = Status::ok();
    cudaError_t e = cudaMemcpyAsync(B.d_io, hi, 4 * sizeof(int), cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) {
      s = Status::err(WEDLM_ERR_CUDA, cudaGetErrorString(e));
      break;
    }
    int* dout = B.d_io + 3 + B.cap;
    EntropyArgs A;
    A.logits = B.logits;
    A.dtype = m->dt;
    A.rows = 1;
    A.V = m->vshard;
    A.ld = m->vshard;
    A.nseq = 1;
    A.seq_rows = B.d_io;
    A.mask_pos = B.d_io + 2;
    A.caps = B.d_io + 3;
    A.argmax = dout + B.cap;
    A.selected = dout + 2 * B.cap;
    A.n_selected = dout + 3 * B.cap;
    EntropyPlan ep = plan_entropy(1, m->vshard, m->dt, ctx->num_sms);
    s = ensure_entropy_scratch(ctx, 1, 1, (long)ep.splits * 4);
    if (s.good()) s = run_entropy_select(A, ctx->ent, ctx->num_sms, st);
    if (!s.good()) break;
    int next = 0;
    e = cudaMemcpyAsync(&next, A.argmax, sizeof(int), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) {
      s = Status::err(WEDLM_ERR_CUDA, cudaGetErrorString(e));
      break;
    }
    out_ids[n++] = next;
    last = next;
    if (next == eos) break;
  }
  if (s.good()) s = check_device_error(ctx, st);
  if (!s.good()) return ctx->fail(s);
  *n_out = n;
  return WEDLM_OK;
}
