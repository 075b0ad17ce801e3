// extern "C" entry points of libwedlm_b200.so (declared in include/wedlm_b200.h).
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <new>

#include "comm.h"
#include "context.h"
#include "model.h"
#include "sample.cuh"
#include "gemm.h"
#include "../../include/wedlm_b200_kernels.h"

using wedlm::Status;

namespace {
thread_local std::string g_create_error;

int set_device(wedlm_ctx* ctx) {
  cudaError_t e = cudaSetDevice(ctx->device);
  if (e != cudaSuccess) return ctx->fail(Status::err(WEDLM_ERR_CUDA, cudaGetErrorString(e)));
  return WEDLM_OK;
}
}  // namespace

namespace wedlm {

bool pdl_enabled() {
  static const bool on = [] {
    const char* e = getenv("WEDLM_PDL");
    return !(e && atoi(e) == 0);
  }();
  return on;
}

Status ensure_entropy_scratch(wedlm_ctx* ctx, int rows, int nseq, long partial_floats) {
  EntropyScratch& W = ctx->ent;
  if (rows <= W.row_capacity && nseq <= W.seq_capacity && partial_floats <= W.partial_capacity)
    return Status::ok();
  WEDLM_CUDA_TRY(cudaDeviceSynchronize());
  int nr = rows > W.row_capacity ? rows : W.row_capacity;
  int ns = nseq > W.seq_capacity ? nseq : W.seq_capacity;
  long np = partial_floats > W.partial_capacity ? partial_floats : W.partial_capacity;
  free_entropy_scratch(ctx);
  WEDLM_CUDA_TRY(cudaMalloc(&W.partials, np * sizeof(float)));
  WEDLM_CUDA_TRY(cudaMalloc(&W.row_H, nr * sizeof(float)));
  WEDLM_CUDA_TRY(cudaMalloc(&W.row_count, nr * sizeof(unsigned)));
  WEDLM_CUDA_TRY(cudaMalloc(&W.seq_count, ns * sizeof(unsigned)));
  WEDLM_CUDA_TRY(cudaMemset(W.row_count, 0, nr * sizeof(unsigned)));
  WEDLM_CUDA_TRY(cudaMemset(W.seq_count, 0, ns * sizeof(unsigned)));
  W.partial_capacity = np;
  W.row_capacity = nr;
  W.seq_capacity = ns;
  return Status::ok();
}

void free_entropy_scratch(wedlm_ctx* ctx) {
  EntropyScratch& W = ctx->ent;
  cudaFree(W.partials);
  cudaFree(W.row_H);
  cudaFree(W.row_count);
  cudaFree(W.seq_count);
  W = EntropyScratch{};
}

Status ensure_gemm_scratch(wedlm_ctx* ctx, long ws_floats, int counters) {
  if (!ctx->dev_err) {
    WEDLM_CUDA_TRY(cudaMalloc(&ctx->dev_err, sizeof(int)));
    WEDLM_CUDA_TRY(cudaMemset(ctx->dev_err, 0, sizeof(int)));
  }
  if (ws_floats <= ctx->gemm_ws_floats && counters <= ctx->gemm_n_counters) return Status::ok();
  WEDLM_CUDA_TRY(cudaDeviceSynchronize());
  long nw = ws_floats > ctx->gemm_ws_floats ? ws_floats : ctx->gemm_ws_floats;
  int nc = counters > ctx->gemm_n_counters ? counters : ctx->gemm_n_counters;
  cudaFree(ctx->gemm_ws);
  cudaFree(ctx->gemm_counters);
  ctx->gemm_ws = nullptr;
  ctx->gemm_counters = nullptr;
  ctx->gemm_ws_floats = 0;
  ctx->gemm_n_counters = 0;
  if (nw > 0) WEDLM_CUDA_TRY(cudaMalloc(&ctx->gemm_ws, nw * sizeof(float)));
  if (nc > 0) {
    WEDLM_CUDA_TRY(cudaMalloc(&ctx->gemm_counters, nc * sizeof(unsigned)));
    WEDLM_CUDA_TRY(cudaMemset(ctx->gemm_counters, 0, nc * sizeof(unsigned)));
  }
  ctx->gemm_ws_floats = nw;
  ctx->gemm_n_counters = nc;
  return Status::ok();
}

void free_gemm_scratch(wedlm_ctx* ctx) {
  cudaFree(ctx->gemm_ws);
  cudaFree(ctx->gemm_counters);
  cudaFree(ctx->dev_err);
  ctx->gemm_ws = nullptr;
  ctx->gemm_counters = nullptr;
  ctx->dev_err = nullptr;
  ctx->gemm_ws_floats = 0;
  ctx->gemm_n_counters = 0;
}

Status check_device_error(wedlm_ctx* ctx, cudaStream_t st) {
  if (!ctx->dev_err) return Status::ok();
  int code = 0;
  WEDLM_CUDA_TRY(cudaMemcpyAsync(&code, ctx->dev_err, sizeof(int), cudaMemcpyDeviceToHost, st));
  WEDLM_CUDA_TRY(cudaStreamSynchronize(st));
  if (code != 0) {
    cudaMemsetAsync(ctx->dev_err, 0, sizeof(int), st);
    return Status::err(WEDLM_ERR_TIMEOUT,
                       "a device-side wait gave up (code " + std::to_string(code) + ")");
  }
  return Status::ok();
}

int prof_begin(wedlm_ctx* ctx, cudaStream_t st) {
  WedlmProfiler& P = ctx->prof;
  if (!P.on) return -1;
  if (P.next + 2 > (int)P.ev.size()) {
    const int n = (int)P.ev.size();
    P.ev.resize(n + 2048);
    for (int i = n; i < (int)P.ev.size(); ++i) cudaEventCreate(&P.ev[i]);
  }
  const int h = P.next;
  P.next += 2;
  cudaEventRecord(P.ev[h], st);
  return h;
}

void prof_end(wedlm_ctx* ctx, cudaStream_t st, int h, int cls, double bytes, double flops,
              int nlaunch) {
  WedlmProfiler& P = ctx->prof;
  ctx->launches += nlaunch;
  if (!P.on || h < 0) return;
  cudaEventRecord(P.ev[h + 1], st);
  P.pending.push_back(WedlmProfiler::Rec{cls, h, h + 1, bytes, flops});
  P.launches[cls] += nlaunch;
}

void prof_collect(wedlm_ctx* ctx) {
  WedlmProfiler& P = ctx->prof;
  for (const auto& r : P.pending) {
    float ms = 0.f;
    if (cudaEventElapsedTime(&ms, P.ev[r.e0], P.ev[r.e1]) == cudaSuccess) {
      P.ms[r.cls] += ms;
      P.bytes[r.cls] += r.bytes;
      P.flops[r.cls] += r.flops;
    }
  }
  P.pending.clear();
  P.next = 0;
}

}  // namespace wedlm

extern "C" {

int wedlm_create(const wedlm_config* cfg, int device, int max_seqs, int max_ctx,
                 wedlm_ctx** out) {
  g_create_error.clear();
  if (!out) {
    g_create_error = "out is NULL";
    return WEDLM_ERR_INVALID_ARG;
  }
  *out = nullptr;
  int ndev = 0;
  cudaError_t e = cudaGetDeviceCount(&ndev);
  if (e != cudaSuccess || device < 0 || device >= ndev) {
    g_create_error = std::string("no such CUDA device: ") +
                     (e != cudaSuccess ? cudaGetErrorString(e) : std::to_string(device));
    return WEDLM_ERR_CUDA;
  }
  cudaSetDevice(device);
  cudaDeviceProp prop;
  cudaGetDeviceProperties(&prop, device);
  if (prop.major != 10) {
    g_create_error = "this library is built for sm_100a (B200); device reports sm_" +
                     std::to_string(prop.major) + std::to_string(prop.minor);
    return WEDLM_ERR_UNSUPPORTED;
  }
  wedlm_ctx* ctx = new (std::nothrow) wedlm_ctx();
  if (!ctx) return WEDLM_ERR_OOM;
  ctx->device = device;
  ctx->num_sms = prop.multiProcessorCount;
  ctx->max_seqs = max_seqs;
  ctx->max_ctx = max_ctx;
  if (cfg) {
    Status s = wedlm::model_create(ctx, *cfg, max_seqs, max_ctx);
    if (!s.good()) {
      g_create_error = s.msg;
      wedlm::model_destroy(ctx);
      delete ctx;
      return s.code;
    }
  }
  *out = ctx;
  return WEDLM_OK;
}

void wedlm_destroy(wedlm_ctx* ctx) {
  if (!ctx) return;
  cudaSetDevice(ctx->device);
  cudaDeviceSynchronize();
  wedlm::session_free(ctx);
  wedlm::comm_free(ctx);
  wedlm::free_attention_kernel_scratch(ctx);
  for (cudaEvent_t e : ctx->prof.ev) cudaEventDestroy(e);
  wedlm::model_destroy(ctx);
  wedlm::free_entropy_scratch(ctx);
  wedlm::free_gemm_scratch(ctx);
  delete ctx;
}

const char* wedlm_last_error(const wedlm_ctx* ctx) {
  return ctx ? ctx->last_error.c_str() : g_create_error.c_str();
}

int wedlm_get_config(const wedlm_ctx* ctx, wedlm_config* out) {
  if (!ctx || !out) return WEDLM_ERR_INVALID_ARG;
  if (!ctx->has_model) return WEDLM_ERR_STATE;
  *out = ctx->cfg;
  return WEDLM_OK;
}

int wedlm_entropy_select(wedlm_ctx* ctx, const void* logits, int dtype, int rows, int V, int ld,
                         float temperature, float tau, float lambda, int nseq,
                         const int32_t* seq_rows, const int32_t* mask_pos, const int32_t* caps,
                         float* H, int32_t* argmax, float* maxprob, int32_t* selected,
                         int32_t* n_selected, void* stream) {
  if (!ctx) return WEDLM_ERR_INVALID_ARG;
  if (int rc = set_device(ctx)) return rc;
  wedlm::EntropyArgs A;
  A.logits = logits;
  A.dtype = dtype;
  A.rows = rows;
  A.V = V;
  A.ld = ld;
  A.temperature = temperature;
  A.tau = tau;
  A.lambda = lambda;
  A.nseq = nseq;
  A.seq_rows = seq_rows;
  A.mask_pos = mask_pos;
  A.caps = caps;
  A.H = H;
  A.argmax = argmax;
  A.maxprob = maxprob;
  A.selected = selected;
  A.n_selected = n_selected;
  if (rows < 0 || V <= 0 || nseq < 1)
    return ctx->fail(Status::err(WEDLM_ERR_INVALID_ARG, "bad rows / V / nseq"));
  wedlm::EntropyPlan p = wedlm::plan_entropy(rows, V, dtype, ctx->num_sms);
  Status s = wedlm::ensure_entropy_scratch(ctx, rows, nseq, (long)rows * p.splits * 4);
  if (!s.good()) return ctx->fail(s);
  s = wedlm::run_entropy_select(A, ctx->ent, ctx->num_sms, (cudaStream_t)stream);
  return s.good() ? WEDLM_OK : ctx->fail(s);
}

int wedlm_entropy_partials(wedlm_ctx* ctx, const void* logits, int dtype, int rows, int V,
                           int ld, int vocab_offset, float temperature, float* partials,
                           void* stream) {
  if (!ctx) return WEDLM_ERR_INVALID_ARG;
  if (int rc = set_device(ctx)) return rc;
  wedlm::EntropyArgs A;
  A.logits = logits;
  A.dtype = dtype;
  A.rows = rows;
  A.V = V;
  A.ld = ld;
  A.temperature = temperature;
  if (rows < 0 || V <= 0)
    return ctx->fail(Status::err(WEDLM_ERR_INVALID_ARG, "bad rows / V"));
  wedlm::EntropyPlan p = wedlm::plan_entropy(rows, V, dtype, ctx->num_sms);
  Status s = wedlm::ensure_entropy_scratch(ctx, rows, 1, (long)rows * p.splits * 4);
  if (!s.good()) return ctx->fail(s);
  s = wedlm::run_entropy_partials(A, ctx->ent, vocab_offset, partials, ctx->num_sms,
                                  (cudaStream_t)stream);
  return s.good() ? WEDLM_OK : ctx->fail(s);
}

int wedlm_entropy_combine(wedlm_ctx* ctx, const float* partials, int nshards, int rows, float tau,
                          float lambda, int nseq, const int32_t* seq_rows, const int32_t* mask_pos,
                          const int32_t* caps, float* H, int32_t* argmax, float* maxprob,
                          int32_t* selected, int32_t* n_selected, void* stream) {
  if (!ctx) return WEDLM_ERR_INVALID_ARG;
  if (int rc = set_device(ctx)) return rc;
  wedlm::EntropyArgs A;
  A.rows = rows;
  A.tau = tau;
  A.lambda = lambda;
  A.nseq = nseq;
  A.seq_rows = seq_rows;
  A.mask_pos = mask_pos;
  A.caps = caps;
  A.H = H;
  A.argmax = argmax;
  A.maxprob = maxprob;
  A.selected = selected;
  A.n_selected = n_selected;
  if (rows < 0 || nseq < 1) return ctx->fail(Status::err(WEDLM_ERR_INVALID_ARG, "bad rows / nseq"));
  Status s = wedlm::ensure_entropy_scratch(ctx, rows, nseq, 4);
  if (!s.good()) return ctx->fail(s);
  s = wedlm::run_entropy_combine(partials, nshards, A, ctx->ent, (cudaStream_t)stream);
  return s.good() ? WEDLM_OK : ctx->fail(s);
}

}  // extern "C"

extern "C" int wedlm_kernel_gemm(wedlm_ctx* ctx, const void* X, int64_t ldx, const void* W,
                                 const void* W2, int64_t ldw, int w_layout, int M, int N, int K,
                                 int dtype, int epilogue, void* out, int64_t ldo,
                                 const void* resid, int64_t ldr, void* stream) {
  if (!ctx) return WEDLM_ERR_INVALID_ARG;
  if (int rc = set_device(ctx)) return rc;
  wedlm::GemmArgs a;
  a.X = X; a.ldx = ldx; a.W = W; a.W2 = W2; a.ldw = ldw;
  a.M = M; a.N = N; a.K = K; a.epi = epilogue;
  a.w_packed = w_layout == 1;
  if (w_layout == 1 && dtype != WEDLM_BF16)
    return ctx->fail(Status::err(WEDLM_ERR_INVALID_ARG, "packed weights are bf16 only"));
  a.out = out; a.ldo = ldo; a.resid = resid; a.ldr = ldr;
  if (M <= 0 || N <= 0 || K <= 0 || !X || !W || !out || epilogue < 0 || epilogue > 3)
    return ctx->fail(Status::err(WEDLM_ERR_INVALID_ARG, "bad GEMM arguments"));
  cudaStream_t st = (cudaStream_t)stream;
  Status s;
  if (dtype == WEDLM_F32) {
    s = wedlm::run_gemm_f32(a, st);
  } else if (dtype == WEDLM_BF16) {
    wedlm::GemmPlan g = wedlm::plan_gemm_tc(M, N, K, epilogue == wedlm::EPI_SWIGLU_BF16, ctx->num_sms);
    s = wedlm::ensure_gemm_scratch(ctx, g.ws_floats, g.counters);
    if (s.good()) s = wedlm::run_gemm_tc(a, g, ctx->gemm_ws, ctx->gemm_counters, ctx->dev_err, st);
  } else {
    s = Status::err(WEDLM_ERR_INVALID_ARG, "dtype must be F32 or BF16");
  }
  return s.good() ? WEDLM_OK : ctx->fail(s);
}

extern "C" int wedlm_check_device_error(wedlm_ctx* ctx, void* stream) {
  if (!ctx) return WEDLM_ERR_INVALID_ARG;
  if (int rc = set_device(ctx)) return rc;
  wedlm::Status s = wedlm::check_device_error(ctx, (cudaStream_t)stream);
  return s.good() ? WEDLM_OK : ctx->fail(s);
}

extern "C" int wedlm_profile_enable(wedlm_ctx* ctx, int on) {
  if (!ctx) return WEDLM_ERR_INVALID_ARG;
  if (int rc = set_device(ctx)) return rc;
  cudaDeviceSynchronize();
  wedlm::prof_collect(ctx);
  WedlmProfiler& P = ctx->prof;
  if (on && !P.on) {
    for (int c = 0; c < WedlmProfiler::kClasses; ++c) {
      P.ms[c] = P.bytes[c] = P.flops[c] = 0;
      P.launches[c] = 0;
    }
  }
  P.on = on != 0;
  return WEDLM_OK;
}

extern "C" int wedlm_profile_read(wedlm_ctx* ctx, int cls, double* ms, double* bytes,
                                  double* flops, int64_t* launches) {
  if (!ctx || cls < 0 || cls >= WedlmProfiler::kClasses) return WEDLM_ERR_INVALID_ARG;
  if (int rc = set_device(ctx)) return rc;
  cudaDeviceSynchronize();
  wedlm::prof_collect(ctx);
  const WedlmProfiler& P = ctx->prof;
  if (ms) *ms = P.ms[cls];
  if (bytes) *bytes = P.bytes[cls];
  if (flops) *flops = P.flops[cls];
  if (launches) *launches = P.launches[cls];
  return WEDLM_OK;
}

extern "C" int wedlm_launch_count(const wedlm_ctx* ctx, int64_t* out) {
  if (!ctx || !out) return WEDLM_ERR_INVALID_ARG;
  *out = ctx->launches;
  return WEDLM_OK;
}

extern "C" int wedlm_kernel_pack_weight(wedlm_ctx* ctx, const void* W, int64_t ld, int N, int K,
                                        void* packed, void* stream) {
  if (!ctx) return WEDLM_ERR_INVALID_ARG;
  if (int rc = set_device(ctx)) return rc;
  if (!W || !packed || N <= 0 || K <= 0 || K % 64 != 0 || (uintptr_t)packed % 16 != 0)
    return ctx->fail(Status::err(WEDLM_ERR_INVALID_ARG, "bad pack arguments"));
  Status s = wedlm::pack_weight(W, ld, 0, N, K, packed, (cudaStream_t)stream);
  return s.good() ? WEDLM_OK : ctx->fail(s);
}

extern "C" int wedlm_set_sampling_seed(wedlm_ctx* ctx, uint64_t seed) {
  if (!ctx) return WEDLM_ERR_INVALID_ARG;
  ctx->sample_seed = seed;
  return WEDLM_OK;
}

extern "C" int wedlm_kernel_sample(wedlm_ctx* ctx, const void* logits, int dtype, int rows, int V,
                                   int ld, float temperature, float top_p, const float* u,
                                   int32_t* tokens, void* stream) {
  if (!ctx) return WEDLM_ERR_INVALID_ARG;
  if (int rc = set_device(ctx)) return rc;
  if (!u) return ctx->fail(Status::err(WEDLM_ERR_INVALID_ARG, "u is NULL"));
  wedlm::SampleArgs a;
  a.logits = logits;
  a.dtype = dtype;
  a.rows = rows;
  a.V = V;
  a.ld = ld;
  a.temperature = temperature;
  a.top_p = top_p;
  a.u = u;
  a.tokens = tokens;
  Status s = wedlm::run_sample(a, (cudaStream_t)stream);
  if (s.good()) ctx->launches += rows > 0 ? 1 : 0;
  return s.good() ? WEDLM_OK : ctx->fail(s);
}
