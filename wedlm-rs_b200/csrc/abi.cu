// extern "C" entry points of libwedlm_b200.so (declared in include/wedlm_b200.h).
#include <cstdio>
#include <cstring>
#include <new>

#include "context.h"
#include "model.h"

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
  wedlm::model_destroy(ctx);
  wedlm::free_entropy_scratch(ctx);
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
