// Streaming parallel decoding (the host loop of WeDLMDecoder::generate_streaming,
// src/decoding/wedlm.rs:336-590), batched over independent sequences and exposed as a
// step-wise session (begin / step / result / end) so callers can drive and time it.
//
// Each step, per live sequence: count the contiguous filled prefix (commit-before-
// predict, :387-390, mask detected by token id), reorder the window filled-first /
// masks-last with true positions (:397-427, src/decoding/reorder.rs:57-90); then ONE
// forward over every live window; commit the filled prefix (truncate_cache == advance
// the committed length, :455-465), drain it to the output with the EOS rule and refill
// the window with masks (:470-499); one fused entropy-select pass over all mask rows
// applies the entropy-EMA dynamic cap, the distance-penalised selection and the greedy
// argmax on the device (:511-548); the selected slots are filled (:553-572).
// Host <-> device per step: the forward's metadata upload, one upload of the
// selection inputs, one download of the results.
//
// With a communicator (comm.cu) the LM head and the entropy pass are vocabulary-sharded:
// every rank runs the backbone over its own sequences' windows, the final-normed mask
// rows of all ranks are all-gathered, each rank projects every rank's rows onto its own
// LM-head rows and reduces them to per-row partials (max, sum of exponentials, entropy
// sum, argmax), the partials are all-gathered, and each rank combines the shards for its
// own rows and applies the commit rule.  Both gathers run on NCCL over NVLink; the ranks
// step in lock step until no rank has a live sequence.  At T > 0 the owners' draws travel
// with the hidden rows, and the picked rows are sampled over the split vocabulary in
// phases with a small all-gather after each (sample.cu, run_shard_sample), giving the
// tokens a whole-vocabulary context gives.
#include <algorithm>
#include <cstring>
#include <vector>

#include <cmath>

#include "comm.h"
#include "decode_loop.h"
#include "entropy_select.cuh"
#include "model.h"
#include "sample.cuh"

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
  int n_commit = 0, num_filled = 0;
  std::vector<int> mask_logical;
};

}  // namespace

struct DecodeSession {
  std::vector<SeqRun> runs;
  wedlm_sampling_params prm{};
  int max_new = 0, window = 0;
  cudaStream_t st = nullptr;
  // device block: logits | in: seq_rows, mask_pos, caps, running_idx | running |
  //               out: H, argmax, selected, n_selected
  uint8_t* block = nullptr;
  void* logits = nullptr;
  int* d_in = nullptr;
  float* running = nullptr;
  int* d_out = nullptr;
  int* h_in = nullptr;
  int* h_out = nullptr;
  int rows_cap = 0, nseq_cap = 0;
  std::vector<int> tok, pos, live;
  std::vector<SeqSlice> slices;
  int64_t h2d_bytes = 0, d2h_bytes = 0, steps = 0;

  // Vocabulary-sharded step: rows per rank in the gathered buffers (the largest window
  // capacity of any rank), the header gather (per rank: live sequences, mask rows) and
  // the buffers of the hidden-row and partials gathers.
  bool sharded = false;
  int rmax = 0;
  int* shdr = nullptr;  // device: send [4] | recv [4 * nranks]
  uint8_t* sblock = nullptr;
  void* hsend = nullptr;    // [rmax, H] model dtype
  void* hrecv = nullptr;    // [nranks * rmax, H]
  void* slogits = nullptr;  // [nranks * rmax, vshard]
  float* psend = nullptr;   // [nranks * rmax, 4]
  float* precv = nullptr;   // [nranks, nranks * rmax, 4]
  // T > 0 over the sharded vocabulary: the owners' draws of their mask rows (gathered
  // with the hidden rows), the replicated per-row sampling state and the phase exchange.
  uint8_t* xblock = nullptr;
  float* usend = nullptr;             // [rmax]
  float* urecv = nullptr;             // [nranks * rmax]
  ShardSampleRow* sstate = nullptr;   // [nranks * rmax]
  void* xsend = nullptr;              // shard_sample_xbytes
  void* xrecv = nullptr;              // nranks * shard_sample_xbytes
  // The device-resident loop (decode_loop.cu) when it runs this session; `runs` then
  // mirrors its state only after sync_loop.
  DeviceLoop* loop = nullptr;
  bool loop_stale = false;

  ~DecodeSession() {
    if (loop) loop_free(loop);
    cudaFree(block);
    cudaFree(shdr);
    cudaFree(sblock);
    cudaFree(xblock);
    if (h_in) cudaFreeHost(h_in);
    if (h_out) cudaFreeHost(h_out);
  }
};

// Copy the device loop's outputs, statistics and committed cache lengths into the
// session's host state (and the model's cache lengths).
Status sync_loop(wedlm_ctx* ctx, DecodeSession* S) {
  if (!S->loop || !S->loop_stale) return Status::ok();
  std::vector<LoopSeqResult> res;
  WEDLM_TRY(loop_results(ctx, S->loop, &res));
  ModelState* m = ctx->model;
  for (size_t b = 0; b < res.size() && b < S->runs.size(); ++b) {
    SeqRun& R = S->runs[b];
    const LoopSeqResult& r = res[b];
    R.out = r.out;
    R.done = r.done;
    R.st.steps = r.steps;
    R.st.tokens_generated = r.tokens_generated;
    R.st.avg_entropy = r.entropy_sum;
    R.st.max_entropy = r.entropy_max;
    R.st.high_entropy_count = r.high_entropy_count;
    m->cache_len[R.slot] = r.cache_len;
    m->pending_rows[R.slot] = 0;
  }
  S->loop_stale = false;
  return Status::ok();
}

void session_free(wedlm_ctx* ctx) {
  if (ctx->session) sync_loop(ctx, ctx->session);  // the cache lengths of its slots
  delete ctx->session;
  ctx->session = nullptr;
}

namespace {

// The sampling mode as the ranks compare it: T and, for T > 0, top_p (bit patterns).
void sampling_key(const wedlm_sampling_params& p, int* out) {
  std::memcpy(&out[0], &p.temperature, 4);
  const float tp = p.temperature > 0.f ? p.top_p : 0.f;
  std::memcpy(&out[1], &tp, 4);
}

// Sharded session set-up (collective: every rank of the communicator calls it): agree on
// the rows per rank of the gathered buffers and on the sampling mode (every rank must run
// the same collectives each step), and allocate the buffers.
Status sharded_begin(wedlm_ctx* ctx, DecodeSession* S, cudaStream_t st) {
  ModelState* m = ctx->model;
  Comm* c = ctx->comm;
  const int n = comm_size(c);
  WEDLM_CUDA_TRY(cudaMalloc(&S->shdr, sizeof(int) * 4 * (n + 1)));
  WEDLM_CUDA_TRY(cudaMemsetAsync(S->shdr, 0, sizeof(int) * 4 * (n + 1), st));
  S->h_in[0] = S->rows_cap;
  sampling_key(S->prm, S->h_in + 1);
  S->h_in[3] = 0;
  WEDLM_CUDA_TRY(cudaMemcpyAsync(S->shdr, S->h_in, sizeof(int) * 4, cudaMemcpyHostToDevice, st));
  GatherPiece g;
  g.send = S->shdr;
  g.recv = S->shdr + 4;
  g.count = 4;
  g.dtype = kCommInt32;
  WEDLM_TRY(comm_all_gather(c, &g, 1, st));
  WEDLM_CUDA_TRY(cudaMemcpyAsync(S->h_out, S->shdr + 4, sizeof(int) * 4 * n,
                                 cudaMemcpyDeviceToHost, st));
  WEDLM_TRY(comm_sync(c, st));
  int rmax = 0;
  for (int r = 0; r < n; ++r) {
    rmax = std::max(rmax, S->h_out[4 * r]);
    // every rank sees the same table, so every rank refuses together
    if (S->h_out[4 * r + 1] != S->h_out[1] || S->h_out[4 * r + 2] != S->h_out[2])
      return Status::err(WEDLM_ERR_INVALID_ARG,
                         "the ranks of a sharded decode must use the same temperature and top_p");
  }
  S->rmax = rmax;
  const size_t H = m->H, es = m->esz, rows = (size_t)n * rmax;
  auto up = [](size_t b) { return (b + 255) / 256 * 256; };
  const size_t b_hs = up((size_t)rmax * H * es), b_hr = up(rows * H * es),
               b_lg = up(rows * m->vshard * es), b_ps = up(rows * 4 * 4),
               b_pr = up((size_t)n * rows * 4 * 4);
  WEDLM_CUDA_TRY(cudaMalloc(&S->sblock, b_hs + b_hr + b_lg + b_ps + b_pr));
  S->hsend = S->sblock;
  S->hrecv = S->sblock + b_hs;
  S->slogits = S->sblock + b_hs + b_hr;
  S->psend = reinterpret_cast<float*>(S->sblock + b_hs + b_hr + b_lg);
  S->precv = reinterpret_cast<float*>(S->sblock + b_hs + b_hr + b_lg + b_ps);
  // rows past a rank's mask rows are projected too: keep them finite
  WEDLM_CUDA_TRY(cudaMemsetAsync(S->hsend, 0, b_hs + b_hr, st));
  if (S->prm.temperature > 0.f) {
    const size_t b_us = up((size_t)rmax * 4), b_ur = up(rows * 4),
                 b_st = up(rows * sizeof(ShardSampleRow)),
                 b_x = up(shard_sample_xbytes((int)rows, rmax, S->prm.top_p < 1.f));
    WEDLM_CUDA_TRY(cudaMalloc(&S->xblock, b_us + b_ur + b_st + b_x * (n + 1)));
    S->usend = reinterpret_cast<float*>(S->xblock);
    S->urecv = reinterpret_cast<float*>(S->xblock + b_us);
    S->sstate = reinterpret_cast<ShardSampleRow*>(S->xblock + b_us + b_ur);
    S->xsend = S->xblock + b_us + b_ur + b_st;
    S->xrecv = S->xblock + b_us + b_ur + b_st + b_x;
    WEDLM_CUDA_TRY(cudaMemsetAsync(S->xblock, 0, b_us + b_ur + b_st + b_x * (n + 1), st));
  }
  S->sharded = true;
  return Status::ok();
}

Status session_begin(wedlm_ctx* ctx, const std::vector<int>& slots, const int32_t* prompts,
                     int n_prompt, int max_new, int window, const wedlm_sampling_params& prm,
                     cudaStream_t st) {
  ModelState* m = ctx->model;
  const int B = (int)slots.size();
  WEDLM_CHECK_ARG(B >= 1 && B <= m->max_seqs, "bad number of sequences");
  for (int b = 0; b < B; ++b) {
    WEDLM_CHECK_ARG(slots[b] >= 0 && slots[b] < m->max_seqs, "bad sequence slot");
    for (int c = 0; c < b; ++c) WEDLM_CHECK_ARG(slots[c] != slots[b], "a sequence appears twice");
  }
  WEDLM_CHECK_ARG(n_prompt >= 1 && max_new >= 0 && window >= 1, "bad lengths");
  WEDLM_CHECK_ARG(window <= m->cfg.max_block_tokens, "window larger than max_block_tokens");
  WEDLM_CHECK_ARG(prm.temperature >= 0.f && std::isfinite(prm.temperature),
                  "temperature must be >= 0");
  WEDLM_CHECK_ARG(prm.temperature == 0.f || prm.top_p > 0.f, "top_p must be > 0");
  WEDLM_CHECK_ARG(n_prompt + max_new + window <= m->max_ctx, "prompt + generation exceed max_ctx");
  if (!ctx->comm && m->vshard != m->V)
    return Status::err(WEDLM_ERR_STATE,
                       "this context holds a vocabulary shard: decoding needs the whole "
                       "vocabulary or a communicator (wedlm_comm_init)");
  session_free(ctx);
  DecodeSession* S = new DecodeSession();
  ctx->session = S;
  S->prm = prm;
  S->max_new = max_new;
  S->window = window;
  S->st = st;
  const int mask = m->cfg.mask_token_id;

  // 1. cache the prompts (clear_cache + cache_prefix, wedlm.rs:348-349; no LM head)
  S->runs.assign(B, SeqRun());
  for (int b = 0; b < B; ++b) {
    SeqRun& R = S->runs[b];
    R.slot = slots[b];
    m->cache_len[R.slot] = 0;
    m->pending_rows[R.slot] = 0;
    const int32_t* pr = prompts + (long)b * n_prompt;
    std::vector<int> pos;
    for (int off = 0; off < n_prompt; off += m->max_rows) {
      const int c = std::min(m->max_rows, n_prompt - off);
      pos.resize(c);
      for (int j = 0; j < c; ++j) pos[j] = off + j;
      std::vector<SeqSlice> sl(1);
      sl[0].slot = R.slot;
      sl[0].rows = c;
      sl[0].logit_begin = c;
      WEDLM_TRY(model_forward(ctx, sl, pr + off, pos.data(), nullptr, nullptr, m->dt, nullptr, st));
      m->cache_len[R.slot] += c;
    }
    R.st.prefix_cached = 1;
    const int init = std::min(window, max_new);
    R.window.assign(init, mask);
    R.wpos.resize(init);
    for (int j = 0; j < init; ++j) R.wpos[j] = n_prompt + j;
    R.next_pos = n_prompt + init;
    if (max_new == 0) R.done = true;
  }

  // 2. device / pinned buffers of the loop
  S->rows_cap = B * window;
  S->nseq_cap = B;
  const size_t lbytes = ((size_t)S->rows_cap * m->vshard * m->esz + 255) / 256 * 256;
  // + the sharded step's header and draws
  const size_t in_ints = (size_t)4 * B + 1 + S->rows_cap + 4 + S->rows_cap;
  const size_t out_ints = (size_t)3 * S->rows_cap + B;
  const int nranks = ctx->comm ? comm_size(ctx->comm) : 1;
  WEDLM_CUDA_TRY(cudaMalloc(&S->block, lbytes + (in_ints + B + out_ints) * 4 + 1024));
  S->logits = S->block;
  S->d_in = reinterpret_cast<int*>(S->block + lbytes);
  S->running = reinterpret_cast<float*>(S->d_in + in_ints);
  S->d_out = reinterpret_cast<int*>(S->running + B);
  WEDLM_CUDA_TRY(cudaMallocHost(&S->h_in, in_ints * 4 + 64));
  WEDLM_CUDA_TRY(cudaMallocHost(&S->h_out, (out_ints + 1 + 4 * nranks) * 4 + 64));
  std::vector<float> r0(B, prm.entropy_threshold);  // running entropy starts at tau (:370)
  WEDLM_CUDA_TRY(cudaMemcpyAsync(S->running, r0.data(), B * 4, cudaMemcpyHostToDevice, st));
  if (ctx->comm) WEDLM_TRY(sharded_begin(ctx, S, st));
  WEDLM_CUDA_TRY(cudaStreamSynchronize(st));
  if (device_loop_eligible(ctx, B, window, n_prompt, max_new)) {
    LoopInit li;
    li.W = window;
    li.max_new = max_new;
    li.n_prompt = n_prompt;
    li.slots = slots;
    li.prm = prm;
    li.logits = S->logits;
    li.running = S->running;
    li.st = st ? st : m->stream;  // a graph cannot be captured on the legacy stream
    WEDLM_TRY(loop_create(ctx, li, &S->loop));
  }
  return Status::ok();
}

// Vocabulary-sharded selection of one step (collective).  On entry the forward has
// written this rank's final-normed mask rows to S->hsend and the host staging holds the
// selection inputs (nin ints).  Gathers the hidden rows and headers, projects every
// rank's rows onto this rank's LM-head rows, reduces them to per-row partials, gathers
// the partials, combines this rank's rows and applies the commit rule; downloads the
// results, the device error word and the headers, and waits (bounded).  *global_live =
// live sequences of all ranks at the start of the step.
Status sharded_select(wedlm_ctx* ctx, DecodeSession* S, EntropyArgs& A, int nin,
                      long* global_live) {
  ModelState* m = ctx->model;
  Comm* c = ctx->comm;
  cudaStream_t st = S->st;
  const int n = comm_size(c), me = comm_rank(c);
  const int rows = n * S->rmax;
  // scratch first: growing it synchronises the device
  const EntropyPlan ep = plan_entropy(rows, m->vshard, m->dt, ctx->num_sms);
  WEDLM_TRY(ensure_entropy_scratch(ctx, rows, std::max(A.nseq, 1), (long)rows * ep.splits * 4));
  int* hdr = S->h_in + nin;
  hdr[0] = A.nseq;
  hdr[1] = A.rows;
  hdr[2] = hdr[3] = 0;
  const bool sample = S->prm.temperature > 0.f;
  if (sample && A.rows > 0) {
    // the owner's draw of each of its mask rows: (seed, session index, step, mask row),
    // the key the whole-vocabulary sampler uses
    const int nb = A.nseq;
    const int* h_rows = S->h_in;
    const int* h_ridx = S->h_in + nb + 1 + A.rows + nb;
    const int* h_step = h_ridx + nb;
    float* hu = reinterpret_cast<float*>(hdr + 4);
    for (int k = 0; k < nb; ++k)
      for (int i = h_rows[k]; i < h_rows[k + 1]; ++i)
        hu[i] = sample_draw(ctx->sample_seed, (uint64_t)h_ridx[k], (uint64_t)h_step[k],
                            (uint64_t)(i - h_rows[k]));
  }
  WEDLM_CUDA_TRY(cudaMemcpyAsync(S->d_in, S->h_in, (size_t)(nin + 4) * 4, cudaMemcpyHostToDevice, st));
  S->h2d_bytes += (nin + 4) * 4;
  if (sample && A.rows > 0) {
    WEDLM_CUDA_TRY(cudaMemcpyAsync(S->usend, hdr + 4, (size_t)A.rows * 4, cudaMemcpyHostToDevice, st));
    S->h2d_bytes += A.rows * 4;
  }

  GatherPiece g[3];
  g[0].send = S->hsend;
  g[0].recv = S->hrecv;
  g[0].count = (size_t)S->rmax * m->H;
  g[0].dtype = m->dt;
  g[1].send = S->d_in + nin;
  g[1].recv = S->shdr + 4;
  g[1].count = 4;
  g[1].dtype = kCommInt32;
  g[2].send = S->usend;
  g[2].recv = S->urecv;
  g[2].count = (size_t)S->rmax;
  g[2].dtype = WEDLM_F32;
  int pc = prof_begin(ctx, st);
  Status sg = comm_all_gather(c, g, sample ? 3 : 2, st);
  prof_end(ctx, st, pc, WedlmProfiler::kComm,
           (double)n * (g[0].count * m->esz + 16 + (sample ? S->rmax * 4 : 0)), 0, 0);
  WEDLM_TRY(sg);

  WEDLM_TRY(model_lm_head(ctx, S->hrecv, m->H, rows, S->slogits, m->dt, st));

  EntropyArgs P;
  P.logits = S->slogits;
  P.dtype = m->dt;
  P.rows = rows;
  P.V = m->vshard;
  P.ld = m->vshard;
  P.temperature = A.temperature;
  int ph = prof_begin(ctx, st);
  WEDLM_TRY(run_entropy_partials(P, ctx->ent, comm_shard_begin(c, me), S->psend, ctx->num_sms, st));
  prof_end(ctx, st, ph, WedlmProfiler::kEntropy, (double)rows * m->vshard * m->esz, 0, 1);

  GatherPiece gp;
  gp.send = S->psend;
  gp.recv = S->precv;
  gp.count = (size_t)rows * 4;
  gp.dtype = WEDLM_F32;
  pc = prof_begin(ctx, st);
  sg = comm_all_gather(c, &gp, 1, st);
  prof_end(ctx, st, pc, WedlmProfiler::kComm, (double)n * gp.count * 4, 0, 0);
  WEDLM_TRY(sg);

  if (A.rows > 0) {
    ph = prof_begin(ctx, st);
    WEDLM_TRY(run_entropy_combine(S->precv + (size_t)me * S->rmax * 4, n, A, ctx->ent, st, rows));
    prof_end(ctx, st, ph, WedlmProfiler::kEntropy, (double)n * A.rows * 16, 0, 1);
  }
  if (sample) {
    // T > 0: the picked rows of every rank are drawn over the split vocabulary (every
    // rank runs the same phases); the owners' argmax of those rows is replaced
    ShardSampleArgs sa;
    sa.logits = S->slogits;
    sa.dtype = m->dt;
    sa.V = m->vshard;
    sa.ld = m->vshard;
    sa.vocab_begin = comm_shard_begin(c, me);
    sa.V_total = m->V;
    sa.nranks = n;
    sa.me = me;
    sa.rmax = S->rmax;
    sa.temperature = S->prm.temperature;
    sa.top_p = S->prm.top_p;
    sa.hdr = S->shdr + 4;
    sa.u = S->urecv;
    sa.nseq = A.nseq;
    sa.seq_rows = A.seq_rows;
    sa.selected = A.selected;
    sa.n_selected = A.n_selected;
    sa.state = S->sstate;
    sa.xsend = S->xsend;
    sa.xrecv = S->xrecv;
    sa.tokens = A.argmax;
    // profiled as alternating groups: each phase kernel (entropy class), then its gather
    struct GatherCtx {
      wedlm_ctx* ctx;
      Comm* c;
      int n, open;
    } gc{ctx, c, n, prof_begin(ctx, st)};
    ShardGather sgf;
    sgf.user = &gc;
    sgf.fn = [](void* user, const void* send, void* recv, size_t bytes, cudaStream_t s) {
      GatherCtx* G = static_cast<GatherCtx*>(user);
      prof_end(G->ctx, s, G->open, WedlmProfiler::kEntropy, 0, 0, 1);
      GatherPiece p;
      p.send = send;
      p.recv = recv;
      p.count = bytes / 4;
      p.dtype = kCommInt32;
      const int pg = prof_begin(G->ctx, s);
      Status r = comm_all_gather(G->c, &p, 1, s);
      prof_end(G->ctx, s, pg, WedlmProfiler::kComm, (double)G->n * bytes, 0, 0);
      G->open = prof_begin(G->ctx, s);
      return r;
    };
    Status ss = run_shard_sample(sa, sgf, st);
    prof_end(ctx, st, gc.open, WedlmProfiler::kEntropy, 0, 0, 1);
    WEDLM_TRY(ss);
  }
  const size_t nout = (size_t)3 * S->rows_cap + A.nseq;
  int* ho = S->h_out;
  WEDLM_CUDA_TRY(cudaMemcpyAsync(ho, S->d_out, nout * 4, cudaMemcpyDeviceToHost, st));
  WEDLM_CUDA_TRY(cudaMemcpyAsync(ho + nout, ctx->dev_err, 4, cudaMemcpyDeviceToHost, st));
  WEDLM_CUDA_TRY(cudaMemcpyAsync(ho + nout + 1, S->shdr + 4, sizeof(int) * 4 * n,
                                 cudaMemcpyDeviceToHost, st));
  S->d2h_bytes += (int64_t)(nout + 1 + 4 * n) * 4;
  WEDLM_TRY(comm_sync(c, st));
  long live = 0;
  for (int r = 0; r < n; ++r) live += ho[nout + 1 + 4 * r];
  *global_live = live;
  return Status::ok();
}

// One iteration of the streaming loop for every live sequence.  *live_after = number of
// sequences still generating after the step.
Status session_step(wedlm_ctx* ctx, int* live_after) {
  ModelState* m = ctx->model;
  DecodeSession* S = ctx->session;
  const int mask = m->cfg.mask_token_id, eos = m->cfg.eos_token_id;
  const int max_new = S->max_new;
  cudaStream_t st = S->st;
  S->tok.clear();
  S->pos.clear();
  S->slices.clear();
  S->live.clear();
  for (int b = 0; b < (int)S->runs.size(); ++b) {
    SeqRun& R = S->runs[b];
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
        S->tok.push_back(R.window[i]);
        S->pos.push_back(R.wpos[i]);
      }
    for (int i : R.mask_logical) {
      S->tok.push_back(R.window[i]);
      S->pos.push_back(R.wpos[i]);
    }
    SeqSlice sl;
    sl.slot = R.slot;
    sl.rows = (int)R.window.size();
    sl.logit_begin = R.num_filled;
    S->slices.push_back(sl);
    S->live.push_back(b);
  }
  if (S->live.empty() && !S->sharded) {
    *live_after = 0;
    return Status::ok();
  }
  if (!S->live.empty()) S->steps += 1;
  const int R_rows = (int)S->tok.size();
  S->h2d_bytes += (int64_t)(7 * R_rows + 4 * (int)S->live.size()) * 4;

  // ---- step C: one forward over every live window ----
  // (sharded: the LM head runs after the gather; the forward stops at the final norm)
  int nl = 0;
  if (!S->live.empty())
    WEDLM_TRY(model_forward(ctx, S->slices, S->tok.data(), S->pos.data(), nullptr,
                            S->sharded ? nullptr : S->logits, m->dt, &nl, st,
                            S->sharded ? S->hsend : nullptr));

  // ---- steps D, D': commit, drain, refill ----
  for (int b : S->live) {
    SeqRun& R = S->runs[b];
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
  const int nb = (int)S->live.size();
  int* hi = S->h_in;
  int* h_rows = hi;                // [nb + 1]
  int* h_mpos = hi + nb + 1;       // [rr]
  int rr = 0;
  for (int k = 0; k < nb; ++k) {
    const SeqRun& R = S->runs[S->live[k]];
    h_rows[k] = rr;
    for (int i : R.mask_logical) h_mpos[rr++] = i;
  }
  h_rows[nb] = rr;
  int* h_caps = h_mpos + rr;       // [nb]
  int* h_ridx = h_caps + nb;       // [nb] running-entropy slot (session index) of each sequence
  int* h_step = h_ridx + nb;       // [nb] its step number (key of the T > 0 draws)
  for (int k = 0; k < nb; ++k) {
    h_caps[k] = S->prm.max_tokens_per_step;
    h_ridx[k] = S->live[k];
    h_step[k] = (int)S->runs[S->live[k]].st.steps;
  }
  const int nin = nb + 1 + rr + 3 * nb;
  int* d_rows = S->d_in;
  int* d_mpos = d_rows + nb + 1;
  int* d_caps = d_mpos + rr;
  int* d_ridx = d_caps + nb;
  int* d_step = d_ridx + nb;
  float* dH = reinterpret_cast<float*>(S->d_out);
  int* dA = S->d_out + S->rows_cap;
  int* dS = dA + S->rows_cap;
  int* dN = dS + S->rows_cap;
  EntropyArgs A;
  A.dtype = m->dt;
  A.rows = rr;
  A.temperature = S->prm.temperature;
  A.tau = S->prm.entropy_threshold;
  A.lambda = S->prm.distance_penalty;
  A.nseq = nb;
  A.seq_rows = d_rows;
  A.mask_pos = d_mpos;
  A.caps = d_caps;
  A.running = S->running;
  A.running_idx = d_ridx;
  A.H = dH;
  A.argmax = dA;
  A.selected = dS;
  A.n_selected = dN;
  const size_t nout = (size_t)3 * S->rows_cap + nb;
  int* ho = S->h_out;
  long global_live = 0;
  if (S->sharded) {
    WEDLM_TRY(sharded_select(ctx, S, A, nin, &global_live));
  } else if (rr > 0) {
    WEDLM_CUDA_TRY(cudaMemcpyAsync(S->d_in, hi, (size_t)nin * 4, cudaMemcpyHostToDevice, st));
    S->h2d_bytes += nin * 4;
    A.logits = S->logits;
    A.V = m->vshard;
    A.ld = m->vshard;
    A.plan_rows = S->rows_cap;  // the device loop's split: the same merge order per row
    EntropyPlan ep = plan_entropy(S->rows_cap, m->vshard, m->dt, ctx->num_sms);
    WEDLM_TRY(ensure_entropy_scratch(ctx, rr, nb, (long)rr * ep.splits * 4));
    const int ph = prof_begin(ctx, st);
    WEDLM_TRY(run_entropy_select(A, ctx->ent, ctx->num_sms, st));
    prof_end(ctx, st, ph, WedlmProfiler::kEntropy, (double)rr * m->vshard * m->esz, 0, 1);
    if (S->prm.temperature > 0.f) {
      // T > 0: the selected rows are drawn (sample_from_probs / sample_nucleus) in place
      // of their argmax, keyed by (seed, session index, step, mask row)
      SampleArgs sa;
      sa.logits = S->logits;
      sa.dtype = m->dt;
      sa.rows = rr;
      sa.V = m->vshard;
      sa.ld = m->vshard;
      sa.temperature = S->prm.temperature;
      sa.top_p = S->prm.top_p;
      sa.seed = ctx->sample_seed;
      sa.nseq = nb;
      sa.seq_rows = d_rows;
      sa.selected = dS;
      sa.n_selected = dN;
      sa.seq_key = d_ridx;
      sa.seq_step = d_step;
      sa.tokens = dA;
      const int ps = prof_begin(ctx, st);
      WEDLM_TRY(run_sample(sa, st));
      prof_end(ctx, st, ps, WedlmProfiler::kEntropy, 0, 0, 1);
    }
    WEDLM_CUDA_TRY(cudaMemcpyAsync(ho, S->d_out, nout * 4, cudaMemcpyDeviceToHost, st));
    WEDLM_CUDA_TRY(cudaMemcpyAsync(ho + nout, ctx->dev_err, 4, cudaMemcpyDeviceToHost, st));
    S->d2h_bytes += (int64_t)(nout + 1) * 4;
    WEDLM_CUDA_TRY(cudaStreamSynchronize(st));
  } else {
    WEDLM_CUDA_TRY(cudaStreamSynchronize(st));
  }
  if (S->sharded || rr > 0) {
    prof_collect(ctx);
    if (ho[nout] != 0) {
      cudaMemsetAsync(ctx->dev_err, 0, 4, st);
      return Status::err(WEDLM_ERR_TIMEOUT, "a device-side wait gave up during the decode step");
    }
  }
  if (rr > 0) {
    const float* Hh = reinterpret_cast<const float*>(ho);
    const int* Ah = ho + S->rows_cap;
    const int* Sh = Ah + S->rows_cap;
    const int* Nh = Sh + S->rows_cap;
    for (int k = 0; k < nb; ++k) {
      SeqRun& R = S->runs[S->live[k]];
      if (R.done) continue;
      const int r0 = h_rows[k];
      for (int i = 0; i < Nh[k]; ++i) {
        const int sel = Sh[r0 + i];
        const int post = std::max(R.mask_logical[sel] - R.n_commit, 0);
        if (post < (int)R.window.size()) {
          R.window[post] = Ah[r0 + sel];
          const float e = Hh[r0 + sel];
          R.st.avg_entropy += e;
          if (e > R.st.max_entropy) R.st.max_entropy = e;
          if (e > kSoftThreshold) R.st.high_entropy_count += 1;
        }
      }
    }
  }
  if (S->sharded) {
    // Every rank sees the same gathered header, so every rank stops after the same step.
    *live_after = (int)std::min<long>(global_live, 1L << 30);
    return Status::ok();
  }
  int live = 0;
  for (const SeqRun& R : S->runs)
    if (!R.done && (int)R.out.size() < max_new && !R.window.empty()) ++live;
  *live_after = live;
  return Status::ok();
}

wedlm_block_stats final_stats(const SeqRun& R) {
  wedlm_block_stats s = R.st;
  if (s.tokens_generated > 0) {
    s.avg_entropy /= (float)s.tokens_generated;
    s.avg_confidence = std::max(1.0f - s.avg_entropy / 10.0f, 0.0f);
  }
  return s;
}

int guard(wedlm_ctx* ctx) {
  if (!ctx) return WEDLM_ERR_INVALID_ARG;
  if (!ctx->model) return ctx->fail(Status::err(WEDLM_ERR_STATE, "context has no model"));
  cudaError_t e = cudaSetDevice(ctx->device);
  if (e != cudaSuccess) return ctx->fail(Status::err(WEDLM_ERR_CUDA, cudaGetErrorString(e)));
  return WEDLM_OK;
}

}  // namespace

}  // namespace wedlm

using wedlm::Status;

extern "C" {

int wedlm_decode_begin(wedlm_ctx* ctx, int nseq, const int32_t* seq_ids, const int32_t* prompts,
                       int n_prompt, int max_new_tokens, int window_size,
                       const wedlm_sampling_params* params, void* stream) {
  if (int rc = wedlm::guard(ctx)) return rc;
  if (nseq < 1 || !seq_ids || !prompts || !params)
    return ctx->fail(Status::err(WEDLM_ERR_INVALID_ARG, "bad decode_begin arguments"));
  std::vector<int> slots(seq_ids, seq_ids + nseq);
  Status s = wedlm::session_begin(ctx, slots, prompts, n_prompt, max_new_tokens, window_size,
                                  *params, (cudaStream_t)stream);
  if (!s.good()) {
    wedlm::session_free(ctx);
    return ctx->fail(s);
  }
  return WEDLM_OK;
}

int wedlm_decode_step(wedlm_ctx* ctx, int n_steps, int32_t* n_live) {
  if (int rc = wedlm::guard(ctx)) return rc;
  if (!ctx->session) return ctx->fail(Status::err(WEDLM_ERR_STATE, "no decode session"));
  int live = 1;
  wedlm::DecodeSession* S = ctx->session;
  if (S->loop) {
    int64_t steps = -1;
    S->loop_stale = true;
    Status s = wedlm::loop_run(ctx, S->loop, n_steps, &live, &steps);
    if (!s.good()) return ctx->fail(s);
    if (steps >= 0) S->steps = steps;
  } else {
    for (int i = 0; i < n_steps && live > 0; ++i) {
      Status s = wedlm::session_step(ctx, &live);
      if (!s.good()) return ctx->fail(s);
    }
  }
  if (n_live) *n_live = live;
  return WEDLM_OK;
}

int wedlm_decode_result(wedlm_ctx* ctx, int b, int32_t* out_ids, int32_t* n_out,
                        wedlm_block_stats* stats) {
  if (int rc = wedlm::guard(ctx)) return rc;
  if (!ctx->session) return ctx->fail(Status::err(WEDLM_ERR_STATE, "no decode session"));
  if (b < 0 || b >= (int)ctx->session->runs.size())
    return ctx->fail(Status::err(WEDLM_ERR_INVALID_ARG, "bad sequence index"));
  Status sl = wedlm::sync_loop(ctx, ctx->session);
  if (!sl.good()) return ctx->fail(sl);
  const wedlm::SeqRun& R = ctx->session->runs[b];
  if (out_ids)
    for (size_t i = 0; i < R.out.size(); ++i) out_ids[i] = R.out[i];
  if (n_out) *n_out = (int32_t)R.out.size();
  if (stats) *stats = wedlm::final_stats(R);
  return WEDLM_OK;
}

int wedlm_decode_io_bytes(const wedlm_ctx* ctx, int64_t* steps, int64_t* h2d_bytes,
                          int64_t* d2h_bytes) {
  if (!ctx || !ctx->session) return WEDLM_ERR_STATE;
  const wedlm::DecodeSession* S = ctx->session;
  int64_t lh = 0, ld = 0;
  if (S->loop) wedlm::loop_io_bytes(S->loop, &lh, &ld);
  if (steps) *steps = S->steps;
  if (h2d_bytes) *h2d_bytes = S->h2d_bytes + lh;
  if (d2h_bytes) *d2h_bytes = S->d2h_bytes + ld;
  return WEDLM_OK;
}

int wedlm_decode_end(wedlm_ctx* ctx) {
  if (!ctx) return WEDLM_ERR_INVALID_ARG;
  wedlm::session_free(ctx);
  return WEDLM_OK;
}

int wedlm_generate_streaming(wedlm_ctx* ctx, int seq, const int32_t* prompt, int n_prompt,
                             int max_new_tokens, int window_size,
                             const wedlm_sampling_params* params, int32_t* out_ids,
                             int32_t* n_out, wedlm_block_stats* stats, void* stream) {
  if (int rc = wedlm::guard(ctx)) return rc;
  if (!out_ids || !n_out) return ctx->fail(Status::err(WEDLM_ERR_INVALID_ARG, "NULL argument"));
  int32_t s = seq;
  if (int rc = wedlm_decode_begin(ctx, 1, &s, prompt, n_prompt, max_new_tokens, window_size,
                                  params, stream))
    return rc;
  int32_t live = 1;
  while (live > 0)
    if (int rc = wedlm_decode_step(ctx, 1 << 30, &live)) {
      wedlm::session_free(ctx);
      return rc;
    }
  int rc = wedlm_decode_result(ctx, 0, out_ids, n_out, stats);
  wedlm::session_free(ctx);
  return rc;
}

int wedlm_generate_streaming_batch(wedlm_ctx* ctx, int nseq, const int32_t* prompts, int n_prompt,
                                   int max_new_tokens, int window_size,
                                   const wedlm_sampling_params* params, int32_t* out_ids,
                                   int32_t* n_out, int64_t* steps_out, void* stream) {
  if (int rc = wedlm::guard(ctx)) return rc;
  if (!out_ids || !n_out || nseq < 1)
    return ctx->fail(Status::err(WEDLM_ERR_INVALID_ARG, "bad batch arguments"));
  std::vector<int32_t> slots(nseq);
  for (int b = 0; b < nseq; ++b) slots[b] = b;
  if (int rc = wedlm_decode_begin(ctx, nseq, slots.data(), prompts, n_prompt, max_new_tokens,
                                  window_size, params, stream))
    return rc;
  int32_t live = 1;
  while (live > 0)
    if (int rc = wedlm_decode_step(ctx, 1 << 30, &live)) {
      wedlm::session_free(ctx);
      return rc;
    }
  for (int b = 0; b < nseq; ++b) {
    wedlm_block_stats st;
    wedlm_decode_result(ctx, b, out_ids + (long)b * max_new_tokens, n_out + b, &st);
    if (steps_out) steps_out[b] = st.steps;
  }
  wedlm::session_free(ctx);
  return WEDLM_OK;
}

}  // extern "C"
