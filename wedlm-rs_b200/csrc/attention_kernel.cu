// Stand-alone block attention: the tensor-core attention of the decode step on caller
// buffers, for parity checks and measurement of that kernel alone.
//
// wedlm_kernel_attention_prepare copies one sequence's queries, cached prefix and window
// keys / values from plain row-major device buffers into the layout the model keeps
// (group-major queries, 64-token K pages, transposed V pages, page table) inside the
// context, and builds the split-KV plan; wedlm_kernel_attention_run launches the
// attention (and the split-KV combine) on it.  The masking is the decode step's: every
// cached key is visible, window key j is visible to window query i iff
// rank[j] <= rank[i].
#include <cstring>
#include <vector>

#include "context.h"
#include "layer_ops.h"
#include "../../include/wedlm_b200_kernels.h"

namespace wedlm {

struct AttnKernelScratch {
  int L = 0, S = 0, nh = 0, nkv = 0, pages = 0;
  size_t cache_cap = 0, q_cap = 0, meta_cap = 0;
  long ws_cap = 0;
  size_t staging_cap = 0;
  void* kcache = nullptr;  // [pages][nkv][64][128] bf16
  void* vcache = nullptr;  // [pages][nkv][128][64] bf16
  void* qg = nullptr;      // [nkv][S][group][128] bf16
  int* meta = nullptr;     // page table | row_seq | seq_row0 | seq_rows | cache_len | slot | rank
  int* h_meta = nullptr;   // pinned staging of meta
  float* ws = nullptr;
  void* h_staging = nullptr;
  AttnArgs args;
  AttnPlan plan;
  bool ready = false;
};

void free_attention_kernel_scratch(wedlm_ctx* ctx) {
  AttnKernelScratch* a = ctx->att;
  if (!a) return;
  cudaFree(a->kcache);
  cudaFree(a->vcache);
  cudaFree(a->qg);
  cudaFree(a->meta);
  cudaFree(a->ws);
  cudaFreeHost(a->h_meta);
  cudaFreeHost(a->h_staging);
  delete a;
  ctx->att = nullptr;
}

namespace {

constexpr int kD = 128, kPage = 64;

// One thread per 8 consecutive elements (16 bytes) of a [tokens][nkv][128] K / V row set:
// K goes to page t / 64, row t % 64 as is; V goes transposed within the page.
__global__ void pack_kv_kernel(const __nv_bfloat16* __restrict__ k,
                               const __nv_bfloat16* __restrict__ v, int tokens, int nkv,
                               __nv_bfloat16* kc, __nv_bfloat16* vc) {
  const long n8 = (long)tokens * nkv * (kD / 8);
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n8;
       i += (long)gridDim.x * blockDim.x) {
    const int c = (int)(i % (kD / 8)) * 8;
    const long tg = i / (kD / 8);
    const int g = (int)(tg % nkv), t = (int)(tg / nkv);
    const int page = t / kPage, row = t % kPage;
    const long src = tg * kD + c;
    *reinterpret_cast<uint4*>(kc + (((long)page * nkv + g) * kPage + row) * kD + c) =
        *reinterpret_cast<const uint4*>(k + src);
    const uint4 vv = *reinterpret_cast<const uint4*>(v + src);
    const __nv_bfloat16* ve = reinterpret_cast<const __nv_bfloat16*>(&vv);
#pragma unroll
    for (int e = 0; e < 8; ++e)
      vc[(((long)page * nkv + g) * kD + c + e) * kPage + row] = ve[e];
  }
}

// queries [S][nh][128] -> group-major [nkv][S][group][128]
__global__ void pack_q_kernel(const __nv_bfloat16* __restrict__ q, int S, int nh, int group,
                              __nv_bfloat16* qg) {
  const long n8 = (long)S * nh * (kD / 8);
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n8;
       i += (long)gridDim.x * blockDim.x) {
    const int c = (int)(i % (kD / 8)) * 8;
    const long sh = i / (kD / 8);
    const int h = (int)(sh % nh), s = (int)(sh / nh);
    const int g = h / group, j = h % group;
    *reinterpret_cast<uint4*>(qg + ((((long)g * S + s) * group + j) * kD) + c) =
        *reinterpret_cast<const uint4*>(q + sh * kD + c);
  }
}

template <typename T>
Status grow(T** p, size_t* cap, size_t bytes, bool zero) {
  if (bytes <= *cap) return Status::ok();
  cudaFree(*p);
  *p = nullptr;
  *cap = 0;
  WEDLM_CUDA_TRY(cudaMalloc(reinterpret_cast<void**>(p), bytes));
  if (zero) WEDLM_CUDA_TRY(cudaMemset(*p, 0, bytes));
  *cap = bytes;
  return Status::ok();
}

}  // namespace
}  // namespace wedlm

using wedlm::Status;

extern "C" int wedlm_kernel_attention_prepare(wedlm_ctx* ctx, const void* q, const void* k,
                                              const void* v, int L, int S, int nh, int nkv,
                                              const int32_t* rank, void* stream) {
  using namespace wedlm;
  if (!ctx) return WEDLM_ERR_INVALID_ARG;
  cudaError_t e = cudaSetDevice(ctx->device);
  if (e != cudaSuccess) return ctx->fail(Status::err(WEDLM_ERR_CUDA, cudaGetErrorString(e)));
  cudaStream_t st = (cudaStream_t)stream;
  if (!q || !k || !v || L < 0 || S < 1 || S > 4096 || nh < 1 || nkv < 1 || nh % nkv != 0 ||
      128 % (nh / nkv) != 0)
    return ctx->fail(Status::err(WEDLM_ERR_INVALID_ARG,
                                 "bad attention shape (need 1 <= S <= 4096, nh % nkv == 0, "
                                 "128 % (nh / nkv) == 0)"));
  if (((uintptr_t)q | (uintptr_t)k | (uintptr_t)v) % 16 != 0)
    return ctx->fail(Status::err(WEDLM_ERR_INVALID_ARG, "q, k and v must be 16-byte aligned"));
  Status s = ensure_gemm_scratch(ctx, 0, 0);  // the device error word
  if (!s.good()) return ctx->fail(s);
  if (!ctx->att) ctx->att = new AttnKernelScratch();
  AttnKernelScratch& a = *ctx->att;
  if (a.ready) {
    // the previous plan's pinned staging may still feed an upload
    e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return ctx->fail(Status::err(WEDLM_ERR_CUDA, cudaGetErrorString(e)));
  }
  a.ready = false;
  const int group = nh / nkv;
  const int tokens = L + S;
  const int pages = 2 * ((tokens + 127) / 128);
  const size_t cache_bytes = (size_t)pages * nkv * kPage * kD * 2;
  size_t kcap = a.cache_cap, vcap = a.cache_cap;
  s = grow(&a.kcache, &kcap, cache_bytes, true);
  if (s.good()) s = grow(&a.vcache, &vcap, cache_bytes, true);
  if (!s.good()) return ctx->fail(s);
  a.cache_cap = kcap < vcap ? kcap : vcap;
  s = grow(&a.qg, &a.q_cap, (size_t)S * nh * kD * 2, false);
  if (!s.good()) return ctx->fail(s);
  const size_t nmeta = (size_t)pages + S + 5 + S;
  if (nmeta * sizeof(int) > a.meta_cap) {
    cudaFreeHost(a.h_meta);
    a.h_meta = nullptr;
    e = cudaHostAlloc(reinterpret_cast<void**>(&a.h_meta), nmeta * sizeof(int), cudaHostAllocDefault);
    if (e != cudaSuccess) return ctx->fail(Status::err(WEDLM_ERR_OOM, cudaGetErrorString(e)));
  }
  s = grow(&a.meta, &a.meta_cap, nmeta * sizeof(int), false);
  if (!s.good()) return ctx->fail(s);
  int* hm = a.h_meta;
  for (int i = 0; i < pages; ++i) hm[i] = i;  // page table of slot 0
  int* h_row_seq = hm + pages;
  for (int i = 0; i < S; ++i) h_row_seq[i] = 0;
  int* h_seq = h_row_seq + S;  // seq_row0, seq_rows, cache_len, slot, (spare)
  h_seq[0] = 0;
  h_seq[1] = S;
  h_seq[2] = L;
  h_seq[3] = 0;
  h_seq[4] = 0;
  int* h_rank = h_seq + 5;
  for (int i = 0; i < S; ++i) h_rank[i] = i;
  e = cudaMemcpyAsync(a.meta, hm, nmeta * sizeof(int), cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess && rank)
    e = cudaMemcpyAsync(a.meta + (pages + S + 5), rank, (size_t)S * sizeof(int),
                        cudaMemcpyDeviceToDevice, st);
  if (e != cudaSuccess) return ctx->fail(Status::err(WEDLM_ERR_CUDA, cudaGetErrorString(e)));
  pack_kv_kernel<<<1184, 256, 0, st>>>((const __nv_bfloat16*)k, (const __nv_bfloat16*)v, tokens,
                                       nkv, (__nv_bfloat16*)a.kcache, (__nv_bfloat16*)a.vcache);
  pack_q_kernel<<<296, 256, 0, st>>>((const __nv_bfloat16*)q, S, nh, group,
                                     (__nv_bfloat16*)a.qg);
  e = cudaGetLastError();
  if (e != cudaSuccess) return ctx->fail(Status::err(WEDLM_ERR_CUDA, cudaGetErrorString(e)));
  ctx->launches += 2;

  AttnArgs& aa = a.args;
  aa = AttnArgs();
  aa.kcache = a.kcache;
  aa.vcache = a.vcache;
  aa.page_table = a.meta;
  aa.pages_per_seq = pages;
  aa.num_pages = pages;
  aa.page_size = kPage;
  aa.layer = 0;
  aa.num_layers = 1;
  aa.q = a.qg;
  aa.rows = S;
  aa.nh = nh;
  aa.nkv = nkv;
  aa.group = group;
  aa.head_dim = kD;
  aa.row_seq = a.meta + pages;
  aa.seq_row0 = a.meta + pages + S;
  aa.seq_rows = aa.seq_row0 + 1;
  aa.seq_cache_len = aa.seq_row0 + 2;
  aa.seq_slot = aa.seq_row0 + 3;
  aa.rank = a.meta + pages + S + 5;
  aa.ld_out = (long)nh * kD;
  aa.nseq = 1;
  aa.max_kv = tokens;
  const long wsf = attention_ws_floats(aa);
  size_t wcap = (size_t)a.ws_cap * sizeof(float);
  s = grow(&a.ws, &wcap, (size_t)wsf * sizeof(float), false);
  if (!s.good()) return ctx->fail(s);
  a.ws_cap = (long)(wcap / sizeof(float));
  // work + combine tables: at most 14 floats per work item
  const long tiles = (long)nkv * (((long)S * group + 127) / 128 + 1);
  const long items = tiles * ((tokens + 127) / 128 + 1);
  const size_t staging = (size_t)items * 14 * sizeof(float) + 64;
  if (staging > a.staging_cap) {
    cudaFreeHost(a.h_staging);
    a.h_staging = nullptr;
    a.staging_cap = 0;
    e = cudaHostAlloc(&a.h_staging, staging, cudaHostAllocDefault);
    if (e != cudaSuccess) return ctx->fail(Status::err(WEDLM_ERR_OOM, cudaGetErrorString(e)));
    a.staging_cap = staging;
  }
  s = plan_attention_tc(aa, &S, &L, ctx->num_sms, a.ws, a.ws_cap, a.h_staging, a.staging_cap,
                        &a.plan, st);
  if (!s.good()) return ctx->fail(s);
  a.L = L;
  a.S = S;
  a.nh = nh;
  a.nkv = nkv;
  a.pages = pages;
  a.ready = true;
  return WEDLM_OK;
}

extern "C" int wedlm_kernel_attention_run(wedlm_ctx* ctx, void* out, void* stream) {
  using namespace wedlm;
  if (!ctx) return WEDLM_ERR_INVALID_ARG;
  if (!ctx->att || !ctx->att->ready)
    return ctx->fail(Status::err(WEDLM_ERR_STATE, "wedlm_kernel_attention_prepare first"));
  if (!out || (uintptr_t)out % 16 != 0)
    return ctx->fail(Status::err(WEDLM_ERR_INVALID_ARG, "out must be 16-byte aligned"));
  cudaError_t e = cudaSetDevice(ctx->device);
  if (e != cudaSuccess) return ctx->fail(Status::err(WEDLM_ERR_CUDA, cudaGetErrorString(e)));
  AttnKernelScratch& a = *ctx->att;
  a.args.out = out;
  Status s = run_attention_tc(a.args, a.plan, ctx->dev_err, (cudaStream_t)stream);
  if (!s.good()) return ctx->fail(s);
  ctx->launches += 1 + (a.plan.n_comb > 0 ? 1 : 0);
  return WEDLM_OK;
}
