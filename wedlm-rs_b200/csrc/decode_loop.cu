// The device-resident streaming loop: bookkeeping kernels around the forward and the
// selection, one CUDA graph per step (decode_loop.h has the overview).
//
// Device state per sequence b (window capacity W):
//   win_tok / win_pos [B][W]  the window in logical order (tokens, true positions)
//   wl, next_pos, done, out_len, cache_len, steps, statistics           [B]
//   out [B][max_new]          the drained tokens
//   live_start, nc, n_mask, n_fill, mlog [B][W]   this step's view (prep -> post)
// The forward's metadata goes to the model's metadata buffer (MetaLayout of B * W rows);
// the selection inputs and outputs live in this loop's buffers.
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "context.h"
#include "decode_loop.h"
#include "entropy_select.cuh"
#include "layer_ops.h"
#include "model.h"
#include "sample.cuh"
#include "sm100.cuh"

namespace wedlm {

namespace {

constexpr float kSoftThreshold = 8.0f;  // ENTROPY_SOFT_THRESHOLD, wedlm.rs:29
constexpr int kLoopThreads = 512;

struct LoopDev {
  int B = 0, W = 0, max_new = 0, mask = 0, eos = 0, cap = 0;
  int* win_tok = nullptr;
  int* win_pos = nullptr;
  int* wl = nullptr;
  int* next_pos = nullptr;
  int* done = nullptr;
  int* live_start = nullptr;
  int* out = nullptr;
  int* out_len = nullptr;
  int* cache_len = nullptr;
  const int* slot = nullptr;
  int* steps = nullptr;
  int* nc = nullptr;
  int* mlog = nullptr;
  int* n_mask = nullptr;
  int* n_fill = nullptr;
  int* tok_gen = nullptr;
  int* high = nullptr;
  float* ent_sum = nullptr;
  float* ent_max = nullptr;
  int* meta = nullptr;
  MetaLayout ml{0, 0};
  int* seq_rows = nullptr;   // [B + 1]
  int* mask_pos = nullptr;   // [B * W]
  int* caps = nullptr;
  int* ridx = nullptr;
  int* step_key = nullptr;
  const float* H = nullptr;        // [B * W] selection outputs
  const int* tokens = nullptr;
  const int* selected = nullptr;
  const int* n_selected = nullptr;
  int* flags = nullptr;            // [2]: live sequences after the step, steps with one
};

// Loop head, commit-before-predict count, mask list and reordering (wedlm.rs:380-427);
// writes the forward's metadata and the selection inputs.  One CTA; warp w handles the
// sequences b = w, w + 32, ...
__global__ void __launch_bounds__(kLoopThreads) loop_prep_kernel(LoopDev a) {
  extern __shared__ int sh_rows[];  // [B + 1]: first mask row of each sequence
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  const unsigned lt = (1u << lane) - 1u;
  const MetaLayout& ml = a.ml;
  for (int b = warp; b < a.B; b += nwarps) {
    const int wlb = a.wl[b];
    int d = a.done[b];
    if (!d && (a.out_len[b] >= a.max_new || wlb == 0)) d = 1;  // (:380-385)
    const int* wt = a.win_tok + (long)b * a.W;
    const int* wp = a.win_pos + (long)b * a.W;
    int nm = 0, first = wlb;
    if (!d) {
      for (int base = 0; base < wlb; base += 32) {
        const int j = base + lane;
        const bool ism = j < wlb && wt[j] == a.mask;
        const unsigned mb = __ballot_sync(0xffffffffu, ism);
        if (first == wlb && mb) first = base + __ffs((int)mb) - 1;
        if (ism) a.mlog[(long)b * a.W + nm + __popc(mb & lt)] = j;
        nm += __popc(mb);
      }
    }
    const int nf = d ? 0 : wlb - nm;
    const int row0 = b * a.W, cl = a.cache_len[b], sl = a.slot[b];
    // forward rows: the filled slots in window order, then the masks, then padding rows
    // (slots past the window, or every slot of a finished sequence, keep their index)
    int fc = 0, mc = 0;
    for (int base = 0; base < a.W; base += 32) {
      const int j = base + lane;
      const bool in = !d && j < wlb;
      const int t = in ? wt[j] : 0;
      const bool ism = in && t == a.mask, isf = in && !ism;
      const unsigned mb = __ballot_sync(0xffffffffu, ism), fb = __ballot_sync(0xffffffffu, isf);
      const int ri = isf ? fc + __popc(fb & lt) : (ism ? nf + mc + __popc(mb & lt) : j);
      fc += __popc(fb);
      mc += __popc(mb);
      if (j < a.W) {
        const int r = row0 + ri;
        a.meta[ml.tok + r] = in ? t : a.mask;
        a.meta[ml.pos + r] = in ? wp[j] : 0;
        a.meta[ml.rank + r] = ri;
        a.meta[ml.rslot + r] = sl;
        a.meta[ml.dst + r] = cl + ri;
        a.meta[ml.rb + r] = b;
        a.meta[ml.act + r] = in ? 1 : 0;
      }
    }
    if (lane == 0) {
      a.done[b] = d;
      a.live_start[b] = !d;
      if (!d) a.steps[b] += 1;
      a.nc[b] = d ? 0 : first;
      a.n_mask[b] = d ? 0 : nm;
      a.n_fill[b] = nf;
      a.meta[ml.s0 + b] = row0;
      a.meta[ml.sr + b] = d ? 0 : wlb;  // the attention's rows of this sequence
      a.meta[ml.sl + b] = cl;
      a.meta[ml.ss + b] = sl;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int b = 0; b < a.B; ++b) {
      sh_rows[b] = acc;
      acc += a.n_mask[b];
    }
    sh_rows[a.B] = acc;
  }
  __syncthreads();
  for (int b = threadIdx.x; b <= a.B; b += blockDim.x) a.seq_rows[b] = sh_rows[b];
  for (int b = warp; b < a.B; b += nwarps) {
    const int r0 = sh_rows[b], nm = a.n_mask[b], nf = a.n_fill[b];
    for (int k = lane; k < nm; k += 32) {
      a.meta[ml.lsrc + r0 + k] = b * a.W + nf + k;  // mask k is reordered row nf + k
      a.mask_pos[r0 + k] = a.mlog[(long)b * a.W + k];
    }
    if (lane == 0) {
      a.caps[b] = a.cap;
      a.ridx[b] = b;
      a.step_key[b] = a.steps[b];
    }
  }
  const int R = a.B * a.W;
  for (int r = sh_rows[a.B] + threadIdx.x; r < R; r += blockDim.x) a.meta[ml.lsrc + r] = 0;
}

// Commit, drain with the EOS rule, refill (wedlm.rs:455-499), fill of the picked slots
// and statistics (:553-572), live count.  One CTA; warp w handles b = w, w + 32, ...
__global__ void __launch_bounds__(kLoopThreads) loop_post_kernel(LoopDev a) {
  __shared__ int s_live, s_any;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  if (threadIdx.x == 0) {
    s_live = 0;
    s_any = 0;
  }
  __syncthreads();
  for (int b = warp; b < a.B; b += nwarps) {
    if (!a.live_start[b]) continue;
    if (lane == 0) s_any = 1;
    int* wt = a.win_tok + (long)b * a.W;
    int* wp = a.win_pos + (long)b * a.W;
    const int ol = a.out_len[b];
    const int nce = min(a.nc[b], max(a.max_new - ol, 0));
    // the committed tokens up to and including the first EOS go to the output
    int add = nce;
    bool eos = false;
    for (int base = 0; base < nce && !eos; base += 32) {
      const int j = base + lane;
      const unsigned eb = __ballot_sync(0xffffffffu, j < nce && wt[j] == a.eos);
      if (eb) {
        add = base + __ffs((int)eb);
        eos = true;
      }
    }
    for (int k = lane; k < add; k += 32) a.out[(long)b * a.max_new + ol + k] = wt[k];
    int wlb = a.wl[b];
    __syncwarp();
    if (lane == 0) {
      a.cache_len[b] += nce;  // truncate_cache(committed + n_commit)
      a.out_len[b] = ol + add;
      a.tok_gen[b] += add;
      if (eos) a.done[b] = 1;
    }
    if (eos) continue;
    // drop the committed slots from the window (in place, 32 slots at a time)
    if (nce > 0) {
      const int keep = wlb - nce;
      for (int base = 0; base < keep; base += 32) {
        const int j = base + lane;
        int t = 0, p = 0;
        if (j < keep) {
          t = wt[j + nce];
          p = wp[j + nce];
        }
        __syncwarp();
        if (j < keep) {
          wt[j] = t;
          wp[j] = p;
        }
        __syncwarp();
      }
      wlb = keep;
    }
    // refill with masks while output + window stay below max_new
    const int nadd = max(0, min(nce, a.max_new - (ol + add) - wlb));
    const int np = a.next_pos[b];
    for (int k = lane; k < nadd; k += 32) {
      wt[wlb + k] = a.mask;
      wp[wlb + k] = np + k;
    }
    wlb += nadd;
    __syncwarp();
    if (lane == 0) {
      a.wl[b] = wlb;
      a.next_pos[b] = np + nadd;
      // the picked mask slots take their tokens (positions shifted by the commit)
      const int r0 = a.seq_rows[b], nm = a.n_mask[b];
      const int ns = min(a.n_selected[b], nm);
      float es = a.ent_sum[b], em = a.ent_max[b];
      int hi = a.high[b];
      for (int i = 0; i < ns; ++i) {
        const int sel = a.selected[r0 + i];
        if (sel < 0 || sel >= nm) continue;
        const int post = max(a.mlog[(long)b * a.W + sel] - nce, 0);
        if (post < wlb) {
          wt[post] = a.tokens[r0 + sel];
          const float e = a.H[r0 + sel];
          es += e;
          if (e > em) em = e;
          if (e > kSoftThreshold) hi += 1;
        }
      }
      a.ent_sum[b] = es;
      a.ent_max[b] = em;
      a.high[b] = hi;
    }
  }
  __syncthreads();
  for (int b = threadIdx.x; b < a.B; b += blockDim.x)
    if (!a.done[b] && a.out_len[b] < a.max_new && a.wl[b] > 0) atomicAdd(&s_live, 1);
  __syncthreads();
  if (threadIdx.x == 0) {
    a.flags[0] = s_live;
    if (s_any) a.flags[1] += 1;
  }
}

}  // namespace

struct DeviceLoop {
  LoopDev d;
  int B = 0, W = 0, max_new = 0;
  wedlm_sampling_params prm{};
  cudaStream_t st = nullptr;
  void* logits = nullptr;
  float* running = nullptr;
  int* ints = nullptr;
  float* floats = nullptr;
  float* attn_ws = nullptr;
  int* h_flags = nullptr;  // pinned [2 slots][2]
  cudaEvent_t ev[2] = {nullptr, nullptr};
  // selection outputs (device)
  float* H = nullptr;
  int* tokens = nullptr;
  int* selected = nullptr;
  int* n_selected = nullptr;
  int* counts = nullptr;  // attention plan counts [2]
  DeviceForward df;
  std::vector<int> len_bound;
  int max_work = 0, max_comb = 0;
  // the step graph
  bool use_graph = true;
  int eager_steps = 0;
  cudaGraphExec_t exec = nullptr;
  int64_t launches_per_step = 0;
  int live = 1;
  int64_t h2d = 0, d2h = 0;

  ~DeviceLoop() {
    if (exec) cudaGraphExecDestroy(exec);
    for (cudaEvent_t e : ev)
      if (e) cudaEventDestroy(e);
    cudaFree(ints);
    cudaFree(floats);
    cudaFree(attn_ws);
    if (h_flags) cudaFreeHost(h_flags);
  }
};

bool device_loop_eligible(wedlm_ctx* ctx, int B, int W, int n_prompt, int max_new) {
  if (const char* e = getenv("WEDLM_DEVICE_LOOP"))
    if (atoi(e) == 0) return false;
  ModelState* m = ctx->model;
  if (ctx->comm || m->vshard != m->V) return false;
  if (B < 1 || B > 4000 || (long)B * W > m->max_rows) return false;
  if ((long)n_prompt + max_new + W > m->cfg.max_position_embeddings) return false;
  return true;
}

namespace {

Status enqueue_step(wedlm_ctx* ctx, DeviceLoop* L) {
  ModelState* m = ctx->model;
  cudaStream_t st = L->st;
  const int B = L->B, R = L->B * L->W;
  int ph = prof_begin(ctx, st);
  loop_prep_kernel<<<1, kLoopThreads, sizeof(int) * (B + 1), st>>>(L->d);
  prof_end(ctx, st, ph, WedlmProfiler::kOther, 0, 0, 1);
  WEDLM_CUDA_TRY(cudaGetLastError());
  WEDLM_TRY(model_forward_device(ctx, L->df, L->logits, m->dt, st));
  EntropyArgs A;
  A.logits = L->logits;
  A.dtype = m->dt;
  A.rows = R;
  A.V = m->vshard;
  A.ld = m->vshard;
  A.temperature = L->prm.temperature;
  A.tau = L->prm.entropy_threshold;
  A.lambda = L->prm.distance_penalty;
  A.nseq = B;
  A.seq_rows = L->d.seq_rows;
  A.mask_pos = L->d.mask_pos;
  A.caps = L->d.caps;
  A.running = L->running;
  A.running_idx = L->d.ridx;
  A.H = L->H;
  A.argmax = L->tokens;
  A.selected = L->selected;
  A.n_selected = L->n_selected;
  A.plan_rows = R;
  ph = prof_begin(ctx, st);
  Status se = run_entropy_select(A, ctx->ent, ctx->num_sms, st);
  prof_end(ctx, st, ph, WedlmProfiler::kEntropy, (double)R * m->vshard * m->esz, 0, 1);
  WEDLM_TRY(se);
  if (L->prm.temperature > 0.f) {
    SampleArgs sa;
    sa.logits = L->logits;
    sa.dtype = m->dt;
    sa.rows = R;
    sa.V = m->vshard;
    sa.ld = m->vshard;
    sa.temperature = L->prm.temperature;
    sa.top_p = L->prm.top_p;
    sa.seed = ctx->sample_seed;
    sa.nseq = B;
    sa.seq_rows = L->d.seq_rows;
    sa.selected = L->selected;
    sa.n_selected = L->n_selected;
    sa.seq_key = L->d.ridx;
    sa.seq_step = L->d.step_key;
    sa.tokens = L->tokens;
    ph = prof_begin(ctx, st);
    Status ss = run_sample(sa, st);
    prof_end(ctx, st, ph, WedlmProfiler::kEntropy, 0, 0, 1);
    WEDLM_TRY(ss);
  }
  ph = prof_begin(ctx, st);
  loop_post_kernel<<<1, kLoopThreads, 0, st>>>(L->d);
  prof_end(ctx, st, ph, WedlmProfiler::kOther, 0, 0, 1);
  WEDLM_CUDA_TRY(cudaGetLastError());
  return Status::ok();
}

// One step: the graph when there is one (captured at the second step, when every scratch
// buffer has grown to the step's shape), else the launches themselves.
Status launch_step(wedlm_ctx* ctx, DeviceLoop* L) {
  cudaStream_t st = L->st;
  const bool graph_ok = L->use_graph && !ctx->prof.on;
  if (graph_ok && !L->exec && L->eager_steps >= 1) {
    const int64_t l0 = ctx->launches;
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal);
    Status s = e == cudaSuccess ? enqueue_step(ctx, L) : Status::err(WEDLM_ERR_CUDA, "capture");
    if (e == cudaSuccess) e = cudaStreamEndCapture(st, &g);
    if (s.good() && e == cudaSuccess && g)
      e = cudaGraphInstantiate(&L->exec, g, 0);
    if (g) cudaGraphDestroy(g);
    L->launches_per_step = ctx->launches - l0;
    ctx->launches = l0;
    if (!s.good() || e != cudaSuccess || !L->exec) {
      // a launch that cannot be captured: run the steps without a graph
      cudaGetLastError();
      if (L->exec) cudaGraphExecDestroy(L->exec);
      L->exec = nullptr;
      L->use_graph = false;
    }
  }
  if (graph_ok && L->exec) {
    WEDLM_CUDA_TRY(cudaGraphLaunch(L->exec, st));
    ctx->launches += L->launches_per_step;
  } else {
    WEDLM_TRY(enqueue_step(ctx, L));
    L->eager_steps += 1;
  }
  return Status::ok();
}

}  // namespace

Status loop_create(wedlm_ctx* ctx, const LoopInit& in, DeviceLoop** out) {
  ModelState* m = ctx->model;
  const int B = (int)in.slots.size(), W = in.W, R = B * W;
  WEDLM_CHECK_ARG(B >= 1 && W >= 1 && in.max_new >= 0, "bad device loop shape");
  DeviceLoop* L = new DeviceLoop();
  *out = L;
  L->B = B;
  L->W = W;
  L->max_new = in.max_new;
  L->prm = in.prm;
  L->st = in.st;
  L->logits = in.logits;
  L->running = in.running;
  if (const char* e = getenv("WEDLM_STEP_GRAPH")) L->use_graph = atoi(e) != 0;

  // int region: [name, count] in this order
  const long mn = std::max(in.max_new, 1);
  const long n_int[] = {(long)B * W, (long)B * W, B, B, B, B, (long)B * mn, B, B, B, B, B,
                        (long)B * W, B, B, B, B, B + 1, (long)R, B, B, B, (long)R, (long)R, B,
                        2, 2};
  long off[sizeof(n_int) / sizeof(n_int[0]) + 1];
  off[0] = 0;
  for (size_t i = 0; i < sizeof(n_int) / sizeof(n_int[0]); ++i)
    off[i + 1] = off[i] + (n_int[i] + 3) / 4 * 4;
  const long total_ints = off[sizeof(n_int) / sizeof(n_int[0])];
  WEDLM_CUDA_TRY(cudaMalloc(&L->ints, total_ints * sizeof(int)));
  int* I = L->ints;
  LoopDev& d = L->d;
  d.B = B;
  d.W = W;
  d.max_new = in.max_new;
  d.mask = m->cfg.mask_token_id;
  d.eos = m->cfg.eos_token_id;
  d.cap = in.prm.max_tokens_per_step;
  d.win_tok = I + off[0];
  d.win_pos = I + off[1];
  d.wl = I + off[2];
  d.next_pos = I + off[3];
  d.done = I + off[4];
  d.live_start = I + off[5];
  d.out = I + off[6];
  d.out_len = I + off[7];
  d.cache_len = I + off[8];
  d.slot = I + off[9];
  d.steps = I + off[10];
  d.nc = I + off[11];
  d.mlog = I + off[12];
  d.n_mask = I + off[13];
  d.n_fill = I + off[14];
  d.tok_gen = I + off[15];
  d.high = I + off[16];
  d.seq_rows = I + off[17];
  d.mask_pos = I + off[18];
  d.caps = I + off[19];
  d.ridx = I + off[20];
  d.step_key = I + off[21];
  L->tokens = I + off[22];
  L->selected = I + off[23];
  L->n_selected = I + off[24];
  d.flags = I + off[25];
  L->counts = I + off[26];
  d.tokens = L->tokens;
  d.selected = L->selected;
  d.n_selected = L->n_selected;
  d.meta = m->d_meta;
  d.ml = MetaLayout(R, B);
  WEDLM_CHECK_ARG((size_t)d.ml.total_dev <= m->meta_ints, "metadata buffer too small");

  WEDLM_CUDA_TRY(cudaMalloc(&L->floats, sizeof(float) * ((long)2 * B + R + 8)));
  d.ent_sum = L->floats;
  d.ent_max = L->floats + B;
  L->H = L->floats + 2 * B;
  d.H = L->H;

  // initial state: every window all masks (decode_begin, wedlm.rs:362-372)
  std::vector<int> h(total_ints, 0);
  const int init = std::min(W, in.max_new);
  for (int b = 0; b < B; ++b) {
    for (int j = 0; j < W; ++j) {
      h[off[0] + (long)b * W + j] = d.mask;
      h[off[1] + (long)b * W + j] = in.n_prompt + j;
    }
    h[off[2] + b] = init;
    h[off[3] + b] = in.n_prompt + init;
    h[off[4] + b] = in.max_new == 0 ? 1 : 0;
    h[off[8] + b] = m->cache_len[in.slots[b]];
    h[off[9] + b] = in.slots[b];
  }
  WEDLM_CUDA_TRY(cudaMemcpyAsync(L->ints, h.data(), total_ints * sizeof(int),
                                 cudaMemcpyHostToDevice, in.st));
  WEDLM_CUDA_TRY(cudaMemsetAsync(L->floats, 0, sizeof(float) * ((long)2 * B + R + 8), in.st));
  L->h2d += total_ints * 4;
  WEDLM_CUDA_TRY(cudaMallocHost(&L->h_flags, sizeof(int) * 4));
  for (cudaEvent_t& e : L->ev) WEDLM_CUDA_TRY(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));

  // forward shape and the device-built attention plan's bounds
  L->len_bound.assign(B, in.n_prompt + in.max_new);
  DeviceForward& df = L->df;
  df.B = B;
  df.W = W;
  df.len_bound = L->len_bound.data();
  if (m->dt == WEDLM_BF16) {
    const long tiles = (long)B * m->nkv * ((W * m->group + 127) / 128);
    // work items <= max(SMs, tiles) (splits = SMs / tiles when that is above 1); combine
    // items: at most one per tile
    L->max_work = (int)std::max<long>(ctx->num_sms, tiles);
    L->max_comb = (int)std::max<long>(1, tiles);
    const long wsf = attention_ws_floats_device(L->max_work, L->max_comb);
    WEDLM_CUDA_TRY(cudaMalloc(&L->attn_ws, wsf * sizeof(float)));
    df.attn_ws = L->attn_ws;
    df.attn_ws_floats = wsf;
    df.max_work = L->max_work;
    df.max_comb = L->max_comb;
    df.counts = L->counts;
  }
  // the rows of finished sequences are never attended: keep them finite from the start
  WEDLM_CUDA_TRY(cudaMemsetAsync(m->attn, 0, (size_t)R * m->qdim * m->esz, in.st));
  const EntropyPlan ep = plan_entropy(R, m->vshard, m->dt, ctx->num_sms);
  WEDLM_TRY(ensure_entropy_scratch(ctx, R, B, (long)R * ep.splits * 4));
  if (!ctx->dev_err) WEDLM_TRY(ensure_gemm_scratch(ctx, 0, 0));
  WEDLM_CUDA_TRY(cudaStreamSynchronize(in.st));
  return Status::ok();
}

Status loop_run(wedlm_ctx* ctx, DeviceLoop* L, int n_steps, int* live, int64_t* steps_total) {
  cudaStream_t st = L->st;
  int launched = 0;
  for (int i = 0; i < n_steps && L->live > 0; ++i) {
    if (i >= 2) {
      // at most two steps in flight: the step two back tells whether to go on
      const int s = (i - 2) & 1;
      WEDLM_CUDA_TRY(cudaEventSynchronize(L->ev[s]));
      if (L->h_flags[2 * s] == 0) break;
    }
    WEDLM_TRY(launch_step(ctx, L));
    const int s = i & 1;
    WEDLM_CUDA_TRY(cudaMemcpyAsync(L->h_flags + 2 * s, L->d.flags, 2 * sizeof(int),
                                   cudaMemcpyDeviceToHost, st));
    WEDLM_CUDA_TRY(cudaEventRecord(L->ev[s], st));
    L->d2h += 8;
    ++launched;
  }
  WEDLM_CUDA_TRY(cudaStreamSynchronize(st));
  prof_collect(ctx);
  int err = 0;
  if (ctx->dev_err) {
    WEDLM_CUDA_TRY(cudaMemcpy(&err, ctx->dev_err, sizeof(int), cudaMemcpyDeviceToHost));
    L->d2h += 4;
  }
  if (launched > 0) L->live = L->h_flags[2 * ((launched - 1) & 1)];
  if (live) *live = L->live;
  if (steps_total) *steps_total = launched > 0 ? L->h_flags[2 * ((launched - 1) & 1) + 1] : -1;
  if (err != 0) {
    cudaMemset(ctx->dev_err, 0, sizeof(int));
    if (err == sm100::kErrAtPlan || err == sm100::kErrLoopRows)
      return Status::err(WEDLM_ERR_STATE, "a device-built plan exceeded its bounds");
    return Status::err(WEDLM_ERR_TIMEOUT, "a device-side wait gave up during the decode step");
  }
  return Status::ok();
}

Status loop_results(wedlm_ctx* ctx, DeviceLoop* L, std::vector<LoopSeqResult>* res) {
  (void)ctx;
  const int B = L->B;
  const long mn = std::max(L->max_new, 1);
  std::vector<int> out((size_t)B * mn), out_len(B), done(B), steps(B), tok(B), high(B), cl(B);
  std::vector<float> es(B), em(B);
  auto get = [&](void* dst, const void* src, size_t bytes) {
    L->d2h += (int64_t)bytes;
    return cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, L->st);
  };
  WEDLM_CUDA_TRY(get(out.data(), L->d.out, out.size() * 4));
  WEDLM_CUDA_TRY(get(out_len.data(), L->d.out_len, B * 4));
  WEDLM_CUDA_TRY(get(done.data(), L->d.done, B * 4));
  WEDLM_CUDA_TRY(get(steps.data(), L->d.steps, B * 4));
  WEDLM_CUDA_TRY(get(tok.data(), L->d.tok_gen, B * 4));
  WEDLM_CUDA_TRY(get(high.data(), L->d.high, B * 4));
  WEDLM_CUDA_TRY(get(cl.data(), L->d.cache_len, B * 4));
  WEDLM_CUDA_TRY(get(es.data(), L->d.ent_sum, B * 4));
  WEDLM_CUDA_TRY(get(em.data(), L->d.ent_max, B * 4));
  WEDLM_CUDA_TRY(cudaStreamSynchronize(L->st));
  res->assign(B, LoopSeqResult());
  for (int b = 0; b < B; ++b) {
    LoopSeqResult& r = (*res)[b];
    const int n = std::min<int>(out_len[b], L->max_new);
    r.out.assign(out.begin() + (long)b * mn, out.begin() + (long)b * mn + n);
    r.done = done[b] != 0;
    r.steps = steps[b];
    r.tokens_generated = tok[b];
    r.high_entropy_count = high[b];
    r.entropy_sum = es[b];
    r.entropy_max = em[b];
    r.cache_len = cl[b];
  }
  return Status::ok();
}

void loop_io_bytes(const DeviceLoop* L, int64_t* h2d, int64_t* d2h) {
  if (h2d) *h2d = L->h2d;
  if (d2h) *d2h = L->d2h;
}

void loop_free(DeviceLoop* L) { delete L; }

}  // namespace wedlm
