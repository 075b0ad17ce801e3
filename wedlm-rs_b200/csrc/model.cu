// Model state and the block forward of the decode step.
//
// Replaces WeDLMForCausalLM (src/model/causal_lm.rs:23-106), WeDLMModel
// (src/model/backbone.rs:61-205), WeDLMDecoderLayer (src/model/layer.rs:58-81) and the
// decoder's KV cache (src/decoding/wedlm.rs:67-69,308-323).  The cache is a
// preallocated paged pool written in place: appending the window K/V replaces
// Tensor::cat (src/model/attention.rs:174-181), and truncate_cache becomes a length
// update.  Per layer (bf16 models):
//   RMSNorm -> QKV GEMM (tcgen05) -> QK-norm + RoPE + KV append -> block attention
//   (tcgen05) -> O GEMM + residual -> RMSNorm -> gate/up GEMM + SwiGLU -> down GEMM +
//   residual; then final RMSNorm and the LM head on the logit rows only.
// f32 models (the reference's f32 parity configuration) run the same sequence on the
// CUDA cores.
#include <cmath>
#include <cstring>
#include <string>

#include "layer_fused.h"
#include "model.h"

namespace wedlm {

namespace {

constexpr int kPage = 64;

// ---- seeded random init ------------------------------------------------------------
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// N(0, std^2) from a counter-based hash (Box-Muller on two 32-bit uniforms).
template <typename T>
__global__ void init_normal_kernel(T* dst, long n, uint64_t seed, uint64_t tensor_id,
                                   long index_offset, float std) {
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const uint64_t h = mix64(seed ^ mix64((tensor_id << 44) + (uint64_t)(i + index_offset) + 1));
    const float u1 = ((float)(uint32_t)(h >> 40) + 1.f) * (1.f / 16777216.f);  // (0, 1]
    const float u2 = (float)(uint32_t)(h & 0xFFFFFF) * (1.f / 16777216.f);     // [0, 1)
    const float z = sqrtf(-2.f * logf(u1)) * cospif(2.f * u2);
    dst[i] = from_f32<T>(z * std);
  }
}

__global__ void fill_f32_kernel(float* dst, long n, float v) {
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
    dst[i] = v;
}

// gather rows src[idx[i]] -> dst[i]
template <typename T>
__global__ void gather_rows_kernel(const T* src, long lds, const int* idx, T* dst, long ldd, int H) {
  pdl_trigger();
  pdl_wait();
  const int r = blockIdx.x;
  const T* s = src + (long)idx[r] * lds;
  T* dd = dst + (long)r * ldd;
  for (int i = threadIdx.x; i < H; i += blockDim.x) dd[i] = s[i];
}

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

float round_bf16_host(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  u = (u + 0x7FFFu + ((u >> 16) & 1u)) & 0xFFFF0000u;
  float r;
  memcpy(&r, &u, 4);
  return r;
}

uint16_t f32_to_bf16_bits(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x7FFFFFu)) return (uint16_t)((u >> 16) | 0x40);
  return (uint16_t)((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}
float bf16_bits_to_f32(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}
float f16_bits_to_f32(uint16_t h) {
  const uint32_t s = (uint32_t)(h & 0x8000) << 16;
  int e = (h >> 10) & 0x1F;
  uint32_t m = h & 0x3FF;
  uint32_t u;
  if (e == 0) {
    if (m == 0) {
      u = s;
    } else {
      e = 1;
      while (!(m & 0x400)) {
        m <<= 1;
        --e;
      }
      m &= 0x3FF;
      u = s | ((uint32_t)(e + 112) << 23) | (m << 13);
    }
  } else if (e == 31) {
    u = s | 0x7F800000u | (m << 13);
  } else {
    u = s | ((uint32_t)(e + 112) << 23) | (m << 13);
  }
  float f;
  memcpy(&f, &u, 4);
  return f;
}

// Where a named tensor lives on the device.
struct WeightRef {
  void* base = nullptr;  // device address of the first stored row (row-major), or of
                         // the packed matrix holding the tensor (packed)
  long rows = 0;         // rows in the checkpoint tensor
  long cols = 0;
  long store_row0 = 0;   // first checkpoint row that is stored (vocab shard)
  long store_rows = 0;   // rows stored on this device
  bool is_norm = false;  // stored as f32
  bool packed = false;   // stored as packed bf16 GEMM tiles
  long pack_row0 = 0;    // row of the packed matrix that holds the first stored row
  int tensor_id = 0;
};

bool parse_layer(const std::string& name, int* layer, std::string* rest) {
  const std::string pfx = "model.layers.";
  if (name.compare(0, pfx.size(), pfx) != 0) return false;
  size_t p = pfx.size(), q = name.find('.', p);
  if (q == std::string::npos) return false;
  try {
    *layer = std::stoi(name.substr(p, q - p));
  } catch (...) {
    return false;
  }
  *rest = name.substr(q + 1);
  return true;
}

Status resolve(ModelState* m, const std::string& name, WeightRef* w) {
  const long H = m->H, I = m->I, d = m->d;
  const int es = m->esz;
  auto mat = [&](void* base, long rows, long cols, int id) {
    w->base = base;
    w->rows = rows;
    w->cols = cols;
    w->store_row0 = 0;
    w->store_rows = rows;
    w->is_norm = false;
    w->packed = false;
    w->pack_row0 = 0;
    w->tensor_id = id;
  };
  // GEMM weights of bf16 models are stored packed; `row0` = row inside the packed matrix
  auto pmat = [&](void* pbase, long row0, long rows, long cols, int id) {
    if (m->dt != WEDLM_BF16) {
      mat(reinterpret_cast<uint8_t*>(pbase) + (size_t)row0 * cols * es, rows, cols, id);
      return;
    }
    mat(pbase, rows, cols, id);
    w->packed = true;
    w->pack_row0 = row0;
  };
  auto norm = [&](float* base, long n, int id) {
    w->base = base;
    w->rows = 1;
    w->cols = n;
    w->store_row0 = 0;
    w->store_rows = 1;
    w->is_norm = true;
    w->tensor_id = id;
  };
  if (name == "model.embed_tokens.weight") {
    mat(m->embed, m->V, H, 1);
    return Status::ok();
  }
  if (name == "lm_head.weight") {
    pmat(m->lm_head, 0, m->V, H, 2);
    w->store_row0 = m->vlo;
    w->store_rows = m->vshard;
    return Status::ok();
  }
  if (name == "model.norm.weight") {
    norm(m->final_norm, H, 3);
    return Status::ok();
  }
  int l;
  std::string rest;
  if (!parse_layer(name, &l, &rest) || l < 0 || l >= m->nlayers)
    return Status::err(WEDLM_ERR_NOT_FOUND, "unknown tensor " + name);
  LayerWeights& L = m->layers[l];
  const int id0 = 16 + l * 16;
  if (rest == "self_attn.q_proj.weight") pmat(L.wqkv, 0, m->qdim, H, id0 + 0);
  else if (rest == "self_attn.k_proj.weight") pmat(L.wqkv, m->qdim, m->kvdim, H, id0 + 1);
  else if (rest == "self_attn.v_proj.weight") pmat(L.wqkv, m->qdim + m->kvdim, m->kvdim, H, id0 + 2);
  else if (rest == "self_attn.o_proj.weight") pmat(L.wo, 0, H, m->qdim, id0 + 3);
  else if (rest == "mlp.gate_proj.weight") pmat(L.wgate, 0, I, H, id0 + 4);
  else if (rest == "mlp.up_proj.weight") pmat(L.wup, 0, I, H, id0 + 5);
  else if (rest == "mlp.down_proj.weight") pmat(L.wdown, 0, H, I, id0 + 6);
  else if (rest == "input_layernorm.weight") norm(L.ln1, H, id0 + 7);
  else if (rest == "post_attention_layernorm.weight") norm(L.ln2, H, id0 + 8);
  else if (rest == "self_attn.q_norm.weight" && m->cfg.qk_norm) norm(L.qn, d, id0 + 9);
  else if (rest == "self_attn.k_norm.weight" && m->cfg.qk_norm) norm(L.kn, d, id0 + 10);
  else return Status::err(WEDLM_ERR_NOT_FOUND, "unknown tensor " + name);
  return Status::ok();
}

std::vector<std::string> all_weight_names(const ModelState* m) {
  std::vector<std::string> v = {"model.embed_tokens.weight", "lm_head.weight", "model.norm.weight"};
  for (int l = 0; l < m->nlayers; ++l) {
    const std::string p = "model.layers." + std::to_string(l) + ".";
    for (const char* s : {"self_attn.q_proj.weight", "self_attn.k_proj.weight", "self_attn.v_proj.weight",
                          "self_attn.o_proj.weight", "mlp.gate_proj.weight", "mlp.up_proj.weight",
                          "mlp.down_proj.weight", "input_layernorm.weight",
                          "post_attention_layernorm.weight"})
      v.push_back(p + s);
    if (m->cfg.qk_norm) {
      v.push_back(p + "self_attn.q_norm.weight");
      v.push_back(p + "self_attn.k_norm.weight");
    }
  }
  return v;
}

}  // namespace

std::vector<std::string> model_weight_names(const ModelState* m) { return all_weight_names(m); }

// ---- create / destroy -------------------------------------------------------------------
Status model_create(wedlm_ctx* ctx, const wedlm_config& c, int max_seqs, int max_ctx) {
  WEDLM_CHECK_ARG(c.vocab_size > 0 && c.hidden_size > 0 && c.num_hidden_layers > 0, "bad shape");
  WEDLM_CHECK_ARG(c.num_attention_heads > 0 && c.num_key_value_heads > 0 &&
                      c.num_attention_heads % c.num_key_value_heads == 0,
                  "heads must be a multiple of kv heads");
  WEDLM_CHECK_ARG(c.head_dim >= 32 && c.head_dim <= 256 && c.head_dim % 32 == 0,
                  "head_dim must be a multiple of 32 in [32, 256]");
  WEDLM_CHECK_ARG(c.intermediate_size > 0 && c.max_position_embeddings > 0, "bad shape");
  WEDLM_CHECK_ARG(c.dtype == WEDLM_F32 || c.dtype == WEDLM_BF16, "dtype must be F32 or BF16");
  WEDLM_CHECK_ARG(max_seqs >= 1 && max_ctx >= 1, "max_seqs and max_ctx must be >= 1");
  WEDLM_CHECK_ARG(c.mask_token_id >= 0 && c.mask_token_id < c.vocab_size,
                  "mask_token_id must be a token of the vocabulary");
  ModelState* m = new ModelState();
  ctx->model = m;
  m->cfg = c;
  if (m->cfg.max_block_tokens <= 0) m->cfg.max_block_tokens = 128;
  m->dt = c.dtype;
  m->esz = dtype_size(c.dtype);
  m->H = c.hidden_size;
  m->I = c.intermediate_size;
  m->V = c.vocab_size;
  m->nh = c.num_attention_heads;
  m->nkv = c.num_key_value_heads;
  m->d = c.head_dim;
  m->group = m->nh / m->nkv;
  m->nlayers = c.num_hidden_layers;
  m->qdim = m->nh * m->d;
  m->kvdim = m->nkv * m->d;
  m->qkvdim = m->qdim + 2 * m->kvdim;
  m->eps = (float)c.rms_norm_eps;
  m->vlo = c.vocab_shard_begin;
  m->vhi = c.vocab_shard_end;
  if (m->vlo == 0 && m->vhi == 0) m->vhi = m->V;
  WEDLM_CHECK_ARG(m->vlo >= 0 && m->vlo < m->vhi && m->vhi <= m->V, "bad vocab shard");
  m->vshard = m->vhi - m->vlo;
  if (m->dt == WEDLM_BF16) {
    WEDLM_CHECK_ARG(m->H % 64 == 0 && m->I % 64 == 0 && m->qdim % 64 == 0,
                    "bf16 models need hidden, intermediate and q dims divisible by 64");
  }
  const int es = m->esz;
  const long H = m->H, I = m->I;

  // weights: one arena, every tensor 256-byte aligned
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t o = off;
    off = align_up(off + bytes, 256);
    return o;
  };
  // GEMM weights of bf16 models are packed (rows padded to whole 128-row tiles)
  auto wsize = [&](long N, long K) -> size_t {
    return (size_t)(m->dt == WEDLM_BF16 ? packed_weight_elems(N, K) : N * K) * es;
  };
  const size_t o_embed = take((size_t)m->V * H * es);
  const size_t o_lm = take(wsize(m->vshard, H));
  const size_t o_fn = take((size_t)H * 4);
  struct LO {
    size_t qkv, o, g, u, dn, l1, l2, qn, kn;
  };
  std::vector<LO> lo(m->nlayers);
  for (int l = 0; l < m->nlayers; ++l) {
    lo[l].qkv = take(wsize(m->qkvdim, H));
    lo[l].o = take(wsize(H, m->qdim));
    lo[l].g = take(wsize(I, H));
    lo[l].u = take(wsize(I, H));
    lo[l].dn = take(wsize(H, I));
    lo[l].l1 = take((size_t)H * 4);
    lo[l].l2 = take((size_t)H * 4);
    lo[l].qn = take((size_t)m->d * 4);
    lo[l].kn = take((size_t)m->d * 4);
  }
  m->arena_bytes = off;
  cudaError_t e = cudaMalloc(&m->arena, m->arena_bytes);
  if (e != cudaSuccess)
    return Status::err(WEDLM_ERR_OOM, "weights: cudaMalloc of " + std::to_string(m->arena_bytes) +
                                          " bytes failed: " + cudaGetErrorString(e));
  WEDLM_CUDA_TRY(cudaMemset(m->arena, 0, m->arena_bytes));
  m->embed = m->arena + o_embed;
  m->lm_head = m->arena + o_lm;
  m->final_norm = reinterpret_cast<float*>(m->arena + o_fn);
  m->layers.resize(m->nlayers);
  for (int l = 0; l < m->nlayers; ++l) {
    LayerWeights& L = m->layers[l];
    L.wqkv = m->arena + lo[l].qkv;
    L.wo = m->arena + lo[l].o;
    L.wgate = m->arena + lo[l].g;
    L.wup = m->arena + lo[l].u;
    L.wdown = m->arena + lo[l].dn;
    L.ln1 = reinterpret_cast<float*>(m->arena + lo[l].l1);
    L.ln2 = reinterpret_cast<float*>(m->arena + lo[l].l2);
    L.qn = reinterpret_cast<float*>(m->arena + lo[l].qn);
    L.kn = reinterpret_cast<float*>(m->arena + lo[l].kn);
  }

  // RoPE tables (rope.rs:37-97): inv_freq in f64 -> f32, freqs = pos * inv_freq in f32,
  // cos/sin in f32 then cast to the model dtype
  {
    const int half = m->d / 2, P = c.max_position_embeddings;
    std::vector<float> inv(half), cs((size_t)P * half), sn((size_t)P * half);
    for (int i = 0; i < half; ++i)
      inv[i] = (float)(1.0 / std::pow(c.rope_theta, (double)(2 * i) / (double)m->d));
    for (int p = 0; p < P; ++p)
      for (int i = 0; i < half; ++i) {
        const float f = (float)p * inv[i];
        float cv = std::cos(f), sv = std::sin(f);
        if (m->dt == WEDLM_BF16) {
          cv = round_bf16_host(cv);
          sv = round_bf16_host(sv);
        }
        cs[(size_t)p * half + i] = cv;
        sn[(size_t)p * half + i] = sv;
      }
    WEDLM_CUDA_TRY(cudaMalloc(&m->cos, cs.size() * 4));
    WEDLM_CUDA_TRY(cudaMalloc(&m->sin, sn.size() * 4));
    WEDLM_CUDA_TRY(cudaMemcpy(m->cos, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice));
    WEDLM_CUDA_TRY(cudaMemcpy(m->sin, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice));
  }

  // paged KV cache (zeroed: masked keys of a partial page must be finite)
  m->max_seqs = max_seqs;
  m->max_ctx = max_ctx;
  m->pages_per_seq = (int)(((max_ctx + 2 * kPage - 1) / (2 * kPage)) * 2);  // even: 128-key chunks
  m->num_pages = m->pages_per_seq * max_seqs;
  const size_t kv_elems = (size_t)m->nlayers * m->num_pages * m->nkv * kPage * m->d;
  e = cudaMalloc(&m->kcache, kv_elems * es);
  if (e == cudaSuccess) e = cudaMalloc(&m->vcache, kv_elems * es);
  if (e != cudaSuccess) return Status::err(WEDLM_ERR_OOM, "KV cache: cudaMalloc failed");
  WEDLM_CUDA_TRY(cudaMemset(m->kcache, 0, kv_elems * es));
  WEDLM_CUDA_TRY(cudaMemset(m->vcache, 0, kv_elems * es));
  {
    std::vector<int> pt((size_t)m->num_pages);
    for (int i = 0; i < m->num_pages; ++i) pt[i] = i;  // slot s owns pages [s*P, (s+1)*P)
    WEDLM_CUDA_TRY(cudaMalloc(&m->page_table, pt.size() * 4));
    WEDLM_CUDA_TRY(cudaMemcpy(m->page_table, pt.data(), pt.size() * 4, cudaMemcpyHostToDevice));
  }
  m->cache_len.assign(max_seqs, 0);
  m->pending_rows.assign(max_seqs, 0);

  // activations
  m->max_rows = max_seqs * m->cfg.max_block_tokens;
  if (m->max_rows < 256) m->max_rows = 256;
  const long R = m->max_rows;
  WEDLM_CUDA_TRY(cudaMalloc(&m->h, R * H * es));
  WEDLM_CUDA_TRY(cudaMalloc(&m->xn, R * H * es));
  WEDLM_CUDA_TRY(cudaMalloc(&m->xl, R * H * es));
  WEDLM_CUDA_TRY(cudaMalloc(&m->qkv, R * m->qkvdim * es));
  WEDLM_CUDA_TRY(cudaMalloc(&m->q, R * m->qdim * es));
  WEDLM_CUDA_TRY(cudaMalloc(&m->attn, R * m->qdim * es));
  WEDLM_CUDA_TRY(cudaMalloc(&m->act, R * I * es));
  m->meta_ints = (size_t)R * 8 + (size_t)max_seqs * 8 + 64;
  WEDLM_CUDA_TRY(cudaMalloc(&m->d_meta, m->meta_ints * 4));
  WEDLM_CUDA_TRY(cudaMallocHost(&m->h_meta, m->meta_ints * 4));
  if (m->dt == WEDLM_BF16 && m->d == 128) {
    const long tiles = (long)m->nkv * ((R * m->group + 127) / 128 + max_seqs);
    const long items = 2 * tiles + 2 * ctx->num_sms + 64;
    m->attn_ws_floats = items * (8 + 6) + items * 128L * 130 + 1024;
    WEDLM_CUDA_TRY(cudaMalloc(&m->attn_ws, m->attn_ws_floats * 4));
    m->attn_staging_bytes = (size_t)items * 64;
    WEDLM_CUDA_TRY(cudaMallocHost(&m->h_attn_staging, m->attn_staging_bytes));
  }
  WEDLM_CUDA_TRY(cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking));
  // norms default to one
  Status s = Status::ok();
  for (auto& L : m->layers) {
    fill_f32_kernel<<<16, 256>>>(L.ln1, H, 1.f);
    fill_f32_kernel<<<16, 256>>>(L.ln2, H, 1.f);
    fill_f32_kernel<<<1, 256>>>(L.qn, m->d, 1.f);
    fill_f32_kernel<<<1, 256>>>(L.kn, m->d, 1.f);
  }
  fill_f32_kernel<<<16, 256>>>(m->final_norm, H, 1.f);
  WEDLM_CUDA_TRY(cudaGetLastError());
  WEDLM_CUDA_TRY(cudaDeviceSynchronize());
  ctx->has_model = true;
  ctx->cfg = m->cfg;
  return s;
}

void model_destroy(wedlm_ctx* ctx) {
  ModelState* m = ctx->model;
  if (!m) return;
  cudaFree(m->arena);
  cudaFree(m->cos);
  cudaFree(m->sin);
  cudaFree(m->kcache);
  cudaFree(m->vcache);
  cudaFree(m->page_table);
  cudaFree(m->h);
  cudaFree(m->xn);
  cudaFree(m->xl);
  cudaFree(m->qkv);
  cudaFree(m->q);
  cudaFree(m->attn);
  cudaFree(m->act);
  cudaFree(m->slots);
  cudaFree(m->sync);
  cudaFree(m->d_meta);
  if (m->h_meta) cudaFreeHost(m->h_meta);
  cudaFree(m->attn_ws);
  if (m->h_attn_staging) cudaFreeHost(m->h_attn_staging);
  if (m->stream) cudaStreamDestroy(m->stream);
  delete m;
  ctx->model = nullptr;
  ctx->has_model = false;
  forget_tensor_maps();
}

// ---- forward --------------------------------------------------------------------------
namespace {

// The forward after its metadata is on the device (d, layout ml): embedding, the layers,
// the final norm, the logit-row gather and the LM head.  h_rows / h_len: host copies of
// the window rows and cache lengths (device mode: the window capacity and upper bounds of
// the lengths, used for the profiler's byte counts; the attention plan is then built on
// the device from the step's own lengths).
Status forward_body(wedlm_ctx* ctx, int B, int R, int RL, const int* d, const MetaLayout& ml,
                    const int* h_rows_p, const int* h_len_p, const DeviceForward* dev,
                    void* logits, int logits_dtype, cudaStream_t st, void* hidden_out) {
  ModelState* m = ctx->model;
  const int o_tok = ml.tok, o_pos = ml.pos, o_rank = ml.rank, o_rslot = ml.rslot, o_dst = ml.dst,
            o_rb = ml.rb, o_lsrc = ml.lsrc, o_s0 = ml.s0, o_sr = ml.sr, o_sl = ml.sl, o_ss = ml.ss;
  (void)o_ss;
  std::vector<int> h_rows(h_rows_p, h_rows_p + B), h_len(h_len_p, h_len_p + B);
  // device loop: its padding rows skip the row-wise kernels
  const int* act = dev ? d + ml.act : nullptr;

  const long H = m->H;
  const int es = m->esz;
  if (!ctx->dev_err) WEDLM_TRY(ensure_gemm_scratch(ctx, 0, 0));
  int* err = ctx->dev_err;

  {
    const int ph = prof_begin(ctx, st);
    Status se = run_embed(m->embed, m->dt, d + o_tok, R, m->H, m->V, m->h, err, st, act);
    prof_end(ctx, st, ph, WedlmProfiler::kOther, 2.0 * R * m->H * es, 0, 1);
    WEDLM_TRY(se);
  }

  // attention geometry shared by the layers
  AttnArgs aa;
  aa.kcache = m->kcache;
  aa.vcache = m->vcache;
  aa.page_table = m->page_table;
  aa.pages_per_seq = m->pages_per_seq;
  aa.num_pages = m->num_pages;
  aa.page_size = kPage;
  aa.num_layers = m->nlayers;
  aa.q = m->q;
  aa.rows = R;
  aa.nh = m->nh;
  aa.nkv = m->nkv;
  aa.group = m->group;
  aa.head_dim = m->d;
  aa.row_seq = d + o_rb;
  aa.seq_row0 = d + o_s0;
  aa.seq_rows = d + o_sr;
  aa.seq_cache_len = d + o_sl;
  aa.seq_slot = d + o_ss;
  aa.rank = d + o_rank;
  aa.out = m->attn;
  aa.ld_out = m->qdim;
  aa.nseq = B;
  int maxkv = 0;
  for (int b = 0; b < B; ++b) maxkv = std::max(maxkv, h_len[b] + h_rows[b]);
  aa.max_kv = maxkv;
  const bool tc = m->dt == WEDLM_BF16;
  AttnPlan plan;
  if (tc && dev) {
    const int ph = prof_begin(ctx, st);
    Status sp = plan_attention_tc_device(aa, ctx->num_sms, dev->attn_ws, dev->attn_ws_floats,
                                         dev->max_work, dev->max_comb, dev->counts, err, &plan, st);
    prof_end(ctx, st, ph, WedlmProfiler::kOther, 0, 0, 1);
    WEDLM_TRY(sp);
  } else if (tc) {
    WEDLM_CHECK_ARG(m->attn_ws != nullptr, "tensor-core attention needs head_dim 128");
    WEDLM_TRY(plan_attention_tc(aa, h_rows.data(), h_len.data(), ctx->num_sms, m->attn_ws,
                                m->attn_ws_floats, m->h_attn_staging, m->attn_staging_bytes, &plan,
                                st));
  }

  RopeKvArgs rk;
  rk.kcache = m->kcache;
  rk.vcache = m->vcache;
  rk.page_table = m->page_table;
  rk.pages_per_seq = m->pages_per_seq;
  rk.num_pages = m->num_pages;
  rk.page_size = kPage;
  rk.num_layers = m->nlayers;
  rk.qkv = m->qkv;
  rk.ld_qkv = m->qkvdim;
  rk.rows = R;
  rk.nh = m->nh;
  rk.nkv = m->nkv;
  rk.group = m->group;
  rk.head_dim = m->d;
  rk.qk_norm = m->cfg.qk_norm;
  rk.eps = m->eps;
  rk.positions = d + o_pos;
  rk.cos = m->cos;
  rk.sin = m->sin;
  rk.row_seq = d + o_rslot;
  rk.dst_pos = d + o_dst;
  rk.q_out = m->q;
  rk.row_active = act;

  // One projection.  f32 models: CUDA-core GEMM with its epilogue.  bf16 models:
  // tcgen05 GEMM on the packed weights; `ps` != NULL selects slot mode (split-K partials
  // for the consumer kernel), otherwise the direct epilogue `epi` writes `out`.
  auto gemm = [&](const void* X, long ldx, const void* W, const void* W2, int N, int K, int epi,
                  void* out, long ldo, const void* resid, long ldr, int M, PartialSet* ps) -> Status {
    GemmArgs g;
    g.X = X;
    g.ldx = ldx;
    g.W = W;
    g.W2 = W2;
    g.ldw = K;
    g.M = M;
    g.N = N;
    g.K = K;
    g.epi = epi;
    g.out = out;
    g.ldo = ldo;
    g.resid = resid;
    g.ldr = ldr;
    const double nw = W2 ? 2.0 : 1.0;
    const double bytes = nw * N * K * es + (double)M * K * es +
                         (double)M * N * (epi == EPI_STORE_F32 ? 4 : es) * (epi == EPI_RESID_BF16 ? 2 : 1);
    const double flops = 2.0 * nw * M * N * K;
    if (!tc) {
      const int ph = prof_begin(ctx, st);
      Status s = run_gemm_f32(g, st);
      prof_end(ctx, st, ph, WedlmProfiler::kGemm, bytes, flops, 1);
      return s;
    }
    g.w_packed = true;
    const bool dual = W2 != nullptr;
    GemmPlan gp = plan_gemm_tc(M, N, K, dual, ctx->num_sms);
    if (ps) {
      if (gp.slot_floats > m->slot_floats) {
        WEDLM_CUDA_TRY(cudaStreamSynchronize(st));
        cudaFree(m->slots);
        m->slots = nullptr;
        m->slot_floats = 0;
        WEDLM_CUDA_TRY(cudaMalloc(&m->slots, gp.slot_floats * sizeof(float)));
        m->slot_floats = gp.slot_floats;
      }
      g.slots = m->slots;
      *ps = partial_set(gp, m->slots, dual);
      if (!ctx->dev_err) WEDLM_TRY(ensure_gemm_scratch(ctx, 0, 0));
    } else {
      WEDLM_TRY(ensure_gemm_scratch(ctx, gp.ws_floats, gp.counters));
    }
    const int ph = prof_begin(ctx, st);
    Status s = run_gemm_tc(g, gp, ctx->gemm_ws, ctx->gemm_counters, ctx->dev_err, st);
    prof_end(ctx, st, ph, WedlmProfiler::kGemm, bytes, flops, (!ps && gp.grid > 1) ? 2 : 1);
    return s;
  };
  // algorithmic bytes / flops of the other kernels of one layer
  double attn_bytes = 2.0 * R * m->qdim * es, attn_flops = 0;
  for (int b = 0; b < B; ++b) {
    attn_bytes += 2.0 * (h_len[b] + h_rows[b]) * m->kvdim * es;
    attn_flops += 4.0 * m->nh * m->d * h_rows[b] * (h_len[b] + (h_rows[b] + 1) / 2.0);
  }
  const double norm_bytes = 2.0 * R * m->H * es;
  const double rope_bytes = (double)R * m->qkvdim * es * 2;
  auto other = [&](Status s, int ph, double bytes) {
    prof_end(ctx, st, ph, WedlmProfiler::kOther, bytes, 0, 1);
    return s;
  };
  auto attention = [&](int l) -> Status {
    aa.layer = l;
    const int ph = prof_begin(ctx, st);
    Status s = tc ? run_attention_tc(aa, plan, err, st) : run_attention_f32(aa, st);
    prof_end(ctx, st, ph, WedlmProfiler::kAttention, attn_bytes, attn_flops,
             tc ? 1 + (plan.n_comb > 0) : 1);
    return s;
  };

  // bf16 windows of up to 96 rows: after each attention, one persistent kernel runs the
  // rest of the layer and the next layer's QKV projection and RoPE (layer_fused.cu)
  long fused_slots = 0;
  const bool fused = tc && fused_tail_supported(R, m->H, m->I, m->qdim, m->qkvdim, m->d,
                                                ctx->num_sms, &fused_slots);
  if (fused) {
    if (fused_slots > m->slot_floats) {
      WEDLM_CUDA_TRY(cudaStreamSynchronize(st));
      cudaFree(m->slots);
      m->slots = nullptr;
      m->slot_floats = 0;
      WEDLM_CUDA_TRY(cudaMalloc(&m->slots, fused_slots * sizeof(float)));
      m->slot_floats = fused_slots;
    }
    if (!m->sync) {
      m->sync_count = m->nlayers * 16;
      WEDLM_CUDA_TRY(cudaMalloc(&m->sync, m->sync_count * sizeof(unsigned)));
    }
    WEDLM_CUDA_TRY(cudaMemsetAsync(m->sync, 0, m->sync_count * sizeof(unsigned), st));
  }
  const double fused_bytes =
      (double)es * ((double)m->H * m->qdim + 2.0 * m->I * m->H + (double)m->H * m->I +
                    (double)m->qkvdim * m->H + (double)R * (m->qdim + 2.0 * m->H + m->I));
  const double fused_flops =
      2.0 * R * ((double)m->H * m->qdim + 3.0 * m->I * m->H + (double)m->qkvdim * m->H);

  if (tc && fused) {
    // embed -> norm -> QKV of layer 0 -> RoPE; then per layer: attention, fused tail
    PartialSet ps;
    int ph = prof_begin(ctx, st);
    WEDLM_TRY(other(run_resid_norm(m->h, nullptr, m->layers[0].ln1, R, m->H, m->eps, m->xn, st,
                                   act),
                    ph, norm_bytes));
    WEDLM_TRY(gemm(m->xn, H, m->layers[0].wqkv, nullptr, m->qkvdim, m->H, EPI_STORE_BF16, nullptr,
                   0, nullptr, 0, R, &ps));
    rk.layer = 0;
    rk.q_norm = m->layers[0].qn;
    rk.k_norm = m->layers[0].kn;
    rk.qkv_partials = &ps;
    ph = prof_begin(ctx, st);
    WEDLM_TRY(other(run_rope_kv(rk, m->dt, st), ph, rope_bytes));
    for (int l = 0; l < m->nlayers; ++l) {
      const LayerWeights& L = m->layers[l];
      const bool last = l + 1 == m->nlayers;
      WEDLM_TRY(attention(l));
      FusedTailArgs ta;
      ta.M = R;
      ta.H = m->H;
      ta.I = m->I;
      ta.qdim = m->qdim;
      ta.qkvdim = m->qkvdim;
      ta.eps = m->eps;
      ta.attn = m->attn;
      ta.h = m->h;
      ta.xn = m->xn;
      ta.act = m->act;
      ta.wo = L.wo;
      ta.wgate = L.wgate;
      ta.wup = L.wup;
      ta.wdown = L.wdown;
      ta.wqkv_next = last ? nullptr : m->layers[l + 1].wqkv;
      ta.wo_next = last ? nullptr : m->layers[l + 1].wo;
      ta.ln2 = L.ln2;
      ta.ln_next = last ? m->final_norm : m->layers[l + 1].ln1;
      ta.rope = rk;
      ta.rope.layer = last ? l : l + 1;
      ta.rope.q_norm = last ? L.qn : m->layers[l + 1].qn;
      ta.rope.k_norm = last ? L.kn : m->layers[l + 1].kn;
      ta.rope.qkv_partials = nullptr;
      ta.slots = m->slots;
      ta.slot_floats = m->slot_floats;
      ta.sync = m->sync + (size_t)l * 16;
      ta.err = err;
      const double b = last ? fused_bytes - (double)es * m->qkvdim * m->H : fused_bytes;
      const double f = last ? fused_flops - 2.0 * R * m->qkvdim * m->H : fused_flops;
      ph = prof_begin(ctx, st);
      Status sf = run_fused_tail(ta, ctx->num_sms, st);
      prof_end(ctx, st, ph, WedlmProfiler::kGemm, b, f, 1);
      WEDLM_TRY(sf);
    }
  } else if (tc) {
    // bf16: split-K partials are summed by the consuming kernel (RoPE / residual + norm /
    // SwiGLU); the residual add and the following RMSNorm are one kernel.
    PartialSet ps;
    int ph = prof_begin(ctx, st);
    WEDLM_TRY(other(run_resid_norm(m->h, nullptr, m->layers[0].ln1, R, m->H, m->eps, m->xn, st,
                                   act),
                    ph, norm_bytes));
    for (int l = 0; l < m->nlayers; ++l) {
      const LayerWeights& L = m->layers[l];
      WEDLM_TRY(gemm(m->xn, H, L.wqkv, nullptr, m->qkvdim, m->H, EPI_STORE_BF16, nullptr, 0,
                     nullptr, 0, R, &ps));
      rk.layer = l;
      rk.q_norm = L.qn;
      rk.k_norm = L.kn;
      rk.qkv_partials = &ps;
      ph = prof_begin(ctx, st);
      WEDLM_TRY(other(run_rope_kv(rk, m->dt, st), ph, rope_bytes));
      WEDLM_TRY(attention(l));
      WEDLM_TRY(gemm(m->attn, m->qdim, L.wo, nullptr, m->H, m->qdim, EPI_STORE_BF16, nullptr, 0,
                     nullptr, 0, R, &ps));
      ph = prof_begin(ctx, st);
      WEDLM_TRY(other(run_resid_norm(m->h, &ps, L.ln2, R, m->H, m->eps, m->xn, st, act), ph,
                      2 * norm_bytes));
      WEDLM_TRY(gemm(m->xn, H, L.wgate, L.wup, m->I, m->H, EPI_SWIGLU_BF16, nullptr, 0, nullptr, 0,
                     R, &ps));
      ph = prof_begin(ctx, st);
      WEDLM_TRY(other(run_swiglu(ps, R, m->I, m->act, st, act), ph, (double)R * m->I * es));
      WEDLM_TRY(gemm(m->act, m->I, L.wdown, nullptr, m->H, m->I, EPI_STORE_BF16, nullptr, 0,
                     nullptr, 0, R, &ps));
      // residual add + the next RMSNorm: next layer's input norm, or the final norm
      const float* wn = (l + 1 < m->nlayers) ? m->layers[l + 1].ln1 : m->final_norm;
      ph = prof_begin(ctx, st);
      WEDLM_TRY(other(run_resid_norm(m->h, &ps, wn, R, m->H, m->eps, m->xn, st, act), ph,
                      2 * norm_bytes));
    }
  } else {
    for (int l = 0; l < m->nlayers; ++l) {
      const LayerWeights& L = m->layers[l];
      int ph = prof_begin(ctx, st);
      WEDLM_TRY(other(run_rmsnorm(m->h, H, L.ln1, R, m->H, m->eps, m->dt, m->xn, H, st), ph, norm_bytes));
      WEDLM_TRY(gemm(m->xn, H, L.wqkv, nullptr, m->qkvdim, m->H, EPI_STORE_BF16, m->qkv, m->qkvdim,
                     nullptr, 0, R, nullptr));
      rk.layer = l;
      rk.q_norm = L.qn;
      rk.k_norm = L.kn;
      rk.qkv_partials = nullptr;
      ph = prof_begin(ctx, st);
      WEDLM_TRY(other(run_rope_kv(rk, m->dt, st), ph, rope_bytes));
      WEDLM_TRY(attention(l));
      WEDLM_TRY(gemm(m->attn, m->qdim, L.wo, nullptr, m->H, m->qdim, EPI_RESID_BF16, m->h, H, m->h,
                     H, R, nullptr));
      ph = prof_begin(ctx, st);
      WEDLM_TRY(other(run_rmsnorm(m->h, H, L.ln2, R, m->H, m->eps, m->dt, m->xn, H, st), ph, norm_bytes));
      WEDLM_TRY(gemm(m->xn, H, L.wgate, L.wup, m->I, m->H, EPI_SWIGLU_BF16, m->act, m->I, nullptr, 0,
                     R, nullptr));
      WEDLM_TRY(gemm(m->act, m->I, L.wdown, nullptr, m->H, m->I, EPI_RESID_BF16, m->h, H, m->h, H, R,
                     nullptr));
    }
  }
  if ((!logits && !hidden_out) || RL == 0) return Status::ok();

  if (!tc) {
    const int ph = prof_begin(ctx, st);
    Status sn = run_rmsnorm(m->h, H, m->final_norm, R, m->H, m->eps, m->dt, m->xn, H, st);
    prof_end(ctx, st, ph, WedlmProfiler::kOther, norm_bytes, 0, 1);
    WEDLM_TRY(sn);
  }
  const void* xl = m->xn;
  // (device mode: the mask rows in selection order, then padding rows, always gathered)
  if (RL != R || hidden_out || dev) {
    void* dst = hidden_out ? hidden_out : m->xl;
    ctx->launches += 1;
    if (m->dt == WEDLM_BF16)
      WEDLM_CUDA_TRY(launch_pdl(gather_rows_kernel<__nv_bfloat16>, dim3(RL), dim3(256), 0, st,
                                (const __nv_bfloat16*)m->xn, (long)H, (const int*)(d + o_lsrc),
                                (__nv_bfloat16*)dst, (long)H, m->H));
    else
      WEDLM_CUDA_TRY(launch_pdl(gather_rows_kernel<float>, dim3(RL), dim3(256), 0, st,
                                (const float*)m->xn, (long)H, (const int*)(d + o_lsrc),
                                (float*)dst, (long)H, m->H));
    xl = dst;
  }
  if (hidden_out) return Status::ok();
  (void)es;
  return model_lm_head(ctx, xl, H, RL, logits, logits_dtype, st);
}

}  // namespace

Status model_forward(wedlm_ctx* ctx, const std::vector<SeqSlice>& seqs, const int* tokens,
                     const int* positions, const int* rank, void* logits, int logits_dtype,
                     int* n_logit_rows, cudaStream_t st, void* hidden_out) {
  ModelState* m = ctx->model;
  const int B = (int)seqs.size();
  WEDLM_CHECK_ARG(B >= 1 && B <= m->max_seqs, "bad number of sequences");
  int R = 0, RL = 0;
  for (const SeqSlice& s : seqs) {
    WEDLM_CHECK_ARG(s.slot >= 0 && s.slot < m->max_seqs, "bad cache slot");
    WEDLM_CHECK_ARG(s.rows >= 0 && s.logit_begin >= 0 && s.logit_begin <= s.rows, "bad window");
    WEDLM_CHECK_ARG(m->cache_len[s.slot] + s.rows <= m->max_ctx,
                    "window does not fit the KV cache (max_ctx)");
    R += s.rows;
    RL += s.rows - s.logit_begin;
  }
  WEDLM_CHECK_ARG(R <= m->max_rows, "more window rows than the context was created for");
  if (n_logit_rows) *n_logit_rows = RL;
  for (int i = 0; i < R; ++i) {
    WEDLM_CHECK_ARG(tokens[i] >= 0 && tokens[i] < m->V, "token id out of range");
    WEDLM_CHECK_ARG(positions[i] >= 0 && positions[i] < m->cfg.max_position_embeddings,
                    "position out of range of the RoPE table");
  }
  WEDLM_CHECK_ARG(logits_dtype == m->dt || logits_dtype == WEDLM_F32 || !logits,
                  "logits dtype must be the model dtype or F32");
  if (R == 0) return Status::ok();

  // ---- metadata (one upload) ----
  int* hm = m->h_meta;
  const MetaLayout ml(R, B);
  const int o_tok = ml.tok, o_pos = ml.pos, o_rank = ml.rank, o_rslot = ml.rslot, o_dst = ml.dst,
            o_rb = ml.rb, o_lsrc = ml.lsrc, o_s0 = ml.s0, o_sr = ml.sr, o_sl = ml.sl, o_ss = ml.ss;
  const int total = ml.total;
  WEDLM_CHECK_ARG((size_t)total <= m->meta_ints, "metadata buffer too small");
  // the pinned staging buffer is reused by the next forward: wait for its last upload
  WEDLM_CUDA_TRY(cudaStreamSynchronize(st));
  int r = 0, rl = 0;
  std::vector<int> h_rows(B), h_len(B);
  for (int b = 0; b < B; ++b) {
    const SeqSlice& s = seqs[b];
    hm[o_s0 + b] = r;
    hm[o_sr + b] = s.rows;
    hm[o_sl + b] = m->cache_len[s.slot];
    hm[o_ss + b] = s.slot;
    h_rows[b] = s.rows;
    h_len[b] = m->cache_len[s.slot];
    for (int j = 0; j < s.rows; ++j, ++r) {
      hm[o_tok + r] = tokens[r];
      hm[o_pos + r] = positions[r];
      hm[o_rank + r] = rank ? rank[r] : j;
      hm[o_rslot + r] = s.slot;
      hm[o_dst + r] = m->cache_len[s.slot] + j;
      hm[o_rb + r] = b;
      if (j >= s.logit_begin) hm[o_lsrc + rl++] = r;
    }
  }
  WEDLM_CUDA_TRY(cudaMemcpyAsync(m->d_meta, hm, (size_t)total * 4, cudaMemcpyHostToDevice, st));
  WEDLM_TRY(forward_body(ctx, B, R, RL, m->d_meta, ml, h_rows.data(), h_len.data(), nullptr, logits,
                         logits_dtype, st, hidden_out));
  for (int b = 0; b < B; ++b) m->pending_rows[seqs[b].slot] = seqs[b].rows;
  return Status::ok();
}

Status model_forward_device(wedlm_ctx* ctx, const DeviceForward& df, void* logits,
                            int logits_dtype, cudaStream_t st) {
  ModelState* m = ctx->model;
  const int B = df.B, R = df.B * df.W;
  WEDLM_CHECK_ARG(B >= 1 && B <= m->max_seqs && df.W >= 1, "bad device forward shape");
  WEDLM_CHECK_ARG(R <= m->max_rows, "more window rows than the context was created for");
  WEDLM_CHECK_ARG((size_t)MetaLayout(R, B).total_dev <= m->meta_ints, "metadata buffer too small");
  WEDLM_CHECK_ARG(logits_dtype == m->dt || logits_dtype == WEDLM_F32,
                  "logits dtype must be the model dtype or F32");
  std::vector<int> h_rows(B, df.W);
  std::vector<int> h_len(df.len_bound, df.len_bound + B);
  return forward_body(ctx, B, R, R, m->d_meta, MetaLayout(R, B), h_rows.data(), h_len.data(), &df,
                      logits, logits_dtype, st, nullptr);
}

Status model_lm_head(wedlm_ctx* ctx, const void* x, long ldx, int M, void* logits,
                     int logits_dtype, cudaStream_t st) {
  ModelState* m = ctx->model;
  WEDLM_CHECK_ARG(logits_dtype == m->dt || logits_dtype == WEDLM_F32,
                  "logits dtype must be the model dtype or F32");
  WEDLM_CHECK_ARG(M >= 0 && x && logits, "bad LM-head rows");
  if (M == 0) return Status::ok();
  const bool tc = m->dt == WEDLM_BF16;
  const int es = m->esz;
  GemmArgs g;
  g.X = x;
  g.ldx = ldx;
  g.W = m->lm_head;
  g.ldw = m->H;
  g.M = M;
  g.N = m->vshard;
  g.K = m->H;
  g.epi = (logits_dtype == WEDLM_F32 && tc) ? EPI_STORE_F32 : EPI_STORE_BF16;
  g.out = logits;
  g.ldo = m->vshard;
  const double bytes = (double)m->vshard * m->H * es + (double)M * m->H * es +
                       (double)M * m->vshard * (g.epi == EPI_STORE_F32 ? 4 : es);
  const double flops = 2.0 * M * m->vshard * m->H;
  if (!tc) {
    const int ph = prof_begin(ctx, st);
    Status s = run_gemm_f32(g, st);
    prof_end(ctx, st, ph, WedlmProfiler::kGemm, bytes, flops, 1);
    return s;
  }
  g.w_packed = true;
  GemmPlan gp = plan_gemm_tc(M, m->vshard, m->H, false, ctx->num_sms);
  WEDLM_TRY(ensure_gemm_scratch(ctx, gp.ws_floats, gp.counters));
  const int ph = prof_begin(ctx, st);
  Status s = run_gemm_tc(g, gp, ctx->gemm_ws, ctx->gemm_counters, ctx->dev_err, st);
  prof_end(ctx, st, ph, WedlmProfiler::kGemm, bytes, flops, gp.grid > 1 ? 2 : 1);
  return s;
}

}  // namespace wedlm

// ---- C ABI ------------------------------------------------------------------------------
using wedlm::Status;
using ModelState = wedlm::ModelState;

namespace {

int model_guard(wedlm_ctx* ctx) {
  if (!ctx) return WEDLM_ERR_INVALID_ARG;
  if (!ctx->model) return ctx->fail(Status::err(WEDLM_ERR_STATE, "context has no model"));
  cudaError_t e = cudaSetDevice(ctx->device);
  if (e != cudaSuccess) return ctx->fail(Status::err(WEDLM_ERR_CUDA, cudaGetErrorString(e)));
  return WEDLM_OK;
}

// NULL means the legacy default stream, as documented in the header.
cudaStream_t pick_stream(wedlm_ctx*, void* stream) { return (cudaStream_t)stream; }

}  // namespace

extern "C" {

int wedlm_set_weight(wedlm_ctx* ctx, const char* name, const void* host_data, int dtype,
                     const int64_t* shape, int ndim) {
  if (int rc = model_guard(ctx)) return rc;
  ModelState* m = ctx->model;
  if (!name || !host_data || !shape || ndim < 1 || ndim > 2)
    return ctx->fail(Status::err(WEDLM_ERR_INVALID_ARG, "bad weight arguments"));
  wedlm::WeightRef w;
  Status s = wedlm::resolve(m, name, &w);
  if (!s.good()) return ctx->fail(s);
  const long rows = ndim == 2 ? shape[0] : 1, cols = shape[ndim - 1];
  if ((w.is_norm && (ndim != 1 || cols != w.cols)) || (!w.is_norm && (rows != w.rows || cols != w.cols)))
    return ctx->fail(Status::err(WEDLM_ERR_INVALID_ARG, std::string("shape mismatch for ") + name));
  if (dtype != WEDLM_F32 && dtype != WEDLM_BF16 && dtype != WEDLM_F16)
    return ctx->fail(Status::err(WEDLM_ERR_INVALID_ARG, "bad dtype"));
  const long n = w.store_rows * w.cols;
  const long src0 = w.store_row0 * w.cols;
  auto get = [&](long i) -> float {
    if (dtype == WEDLM_F32) return reinterpret_cast<const float*>(host_data)[i];
    const uint16_t b = reinterpret_cast<const uint16_t*>(host_data)[i];
    return dtype == WEDLM_BF16 ? wedlm::bf16_bits_to_f32(b) : wedlm::f16_bits_to_f32(b);
  };
  const int es = (w.is_norm || m->dt == WEDLM_F32) ? 4 : 2;
  std::vector<uint8_t> buf((size_t)n * es);
  if (es == 4) {
    float* f = reinterpret_cast<float*>(buf.data());
    for (long i = 0; i < n; ++i) f[i] = get(src0 + i);
  } else if (dtype == WEDLM_BF16) {
    memcpy(buf.data(), reinterpret_cast<const uint16_t*>(host_data) + src0, (size_t)n * 2);
  } else {
    uint16_t* b = reinterpret_cast<uint16_t*>(buf.data());
    for (long i = 0; i < n; ++i) b[i] = wedlm::f32_to_bf16_bits(get(src0 + i));
  }
  if (w.packed) {
    // stage the row-major block on the device, then scatter it into the packed tiles
    void* tmp = nullptr;
    cudaError_t e = cudaMalloc(&tmp, buf.size());
    if (e == cudaSuccess) e = cudaMemcpy(tmp, buf.data(), buf.size(), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
      cudaFree(tmp);
      return ctx->fail(Status::err(WEDLM_ERR_CUDA, cudaGetErrorString(e)));
    }
    Status ps = wedlm::pack_weight(tmp, w.cols, w.pack_row0, w.store_rows, w.cols, w.base, 0);
    e = cudaDeviceSynchronize();
    cudaFree(tmp);
    if (!ps.good()) return ctx->fail(ps);
    if (e != cudaSuccess) return ctx->fail(Status::err(WEDLM_ERR_CUDA, cudaGetErrorString(e)));
    return WEDLM_OK;
  }
  cudaError_t e = cudaMemcpy(w.base, buf.data(), buf.size(), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return ctx->fail(Status::err(WEDLM_ERR_CUDA, cudaGetErrorString(e)));
  return WEDLM_OK;
}

int wedlm_get_weight(wedlm_ctx* ctx, const char* name, void* host_out, int64_t nbytes) {
  if (int rc = model_guard(ctx)) return rc;
  ModelState* m = ctx->model;
  wedlm::WeightRef w;
  Status s = wedlm::resolve(m, name ? name : "", &w);
  if (!s.good()) return ctx->fail(s);
  const int es = (w.is_norm || m->dt == WEDLM_F32) ? 4 : 2;
  const int64_t need = (int64_t)w.store_rows * w.cols * es;
  if (!host_out || nbytes != need)
    return ctx->fail(Status::err(WEDLM_ERR_INVALID_ARG,
                                 "host buffer must be " + std::to_string(need) + " bytes"));
  if (w.packed) {
    void* tmp = nullptr;
    cudaError_t e = cudaMalloc(&tmp, need);
    if (e != cudaSuccess) return ctx->fail(Status::err(WEDLM_ERR_OOM, cudaGetErrorString(e)));
    Status us = wedlm::unpack_weight(w.base, w.pack_row0, w.store_rows, w.cols, tmp, 0);
    e = cudaDeviceSynchronize();
    if (us.good() && e == cudaSuccess) e = cudaMemcpy(host_out, tmp, need, cudaMemcpyDeviceToHost);
    cudaFree(tmp);
    if (!us.good()) return ctx->fail(us);
    if (e != cudaSuccess) return ctx->fail(Status::err(WEDLM_ERR_CUDA, cudaGetErrorString(e)));
    return WEDLM_OK;
  }
  cudaError_t e = cudaMemcpy(host_out, w.base, need, cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return ctx->fail(Status::err(WEDLM_ERR_CUDA, cudaGetErrorString(e)));
  return WEDLM_OK;
}

int wedlm_init_random(wedlm_ctx* ctx, uint64_t seed, float stdv) {
  if (int rc = model_guard(ctx)) return rc;
  ModelState* m = ctx->model;
  for (const std::string& name : wedlm::all_weight_names(m)) {
    wedlm::WeightRef w;
    Status s = wedlm::resolve(m, name, &w);
    if (!s.good()) return ctx->fail(s);
    const long n = w.store_rows * w.cols;
    if (w.is_norm) {
      wedlm::fill_f32_kernel<<<64, 256>>>(reinterpret_cast<float*>(w.base), n, 1.f);
    } else if (w.packed) {
      Status is = wedlm::init_normal_packed(w.base, w.pack_row0, w.store_rows, w.cols, seed,
                                            (uint64_t)w.tensor_id, w.store_row0 * w.cols, stdv, 0);
      if (!is.good()) return ctx->fail(is);
    } else if (m->dt == WEDLM_BF16) {
      wedlm::init_normal_kernel<__nv_bfloat16><<<1184, 256>>>(
          reinterpret_cast<__nv_bfloat16*>(w.base), n, seed, (uint64_t)w.tensor_id,
          w.store_row0 * w.cols, stdv);
    } else {
      wedlm::init_normal_kernel<float><<<1184, 256>>>(reinterpret_cast<float*>(w.base), n, seed,
                                                      (uint64_t)w.tensor_id, w.store_row0 * w.cols,
                                                      stdv);
    }
  }
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return ctx->fail(Status::err(WEDLM_ERR_CUDA, cudaGetErrorString(e)));
  return WEDLM_OK;
}

int wedlm_reset_sequence(wedlm_ctx* ctx, int seq) {
  if (int rc = model_guard(ctx)) return rc;
  ModelState* m = ctx->model;
  if (seq < 0 || seq >= m->max_seqs) return ctx->fail(Status::err(WEDLM_ERR_INVALID_ARG, "bad seq"));
  m->cache_len[seq] = 0;
  m->pending_rows[seq] = 0;
  return WEDLM_OK;
}

int wedlm_cache_len(const wedlm_ctx* ctx, int seq, int32_t* out_len) {
  if (!ctx || !ctx->model || !out_len) return WEDLM_ERR_INVALID_ARG;
  if (seq < 0 || seq >= ctx->model->max_seqs) return WEDLM_ERR_INVALID_ARG;
  *out_len = ctx->model->cache_len[seq];
  return WEDLM_OK;
}

int wedlm_commit(wedlm_ctx* ctx, int seq, int n_commit) {
  if (int rc = model_guard(ctx)) return rc;
  ModelState* m = ctx->model;
  if (seq < 0 || seq >= m->max_seqs) return ctx->fail(Status::err(WEDLM_ERR_INVALID_ARG, "bad seq"));
  if (n_commit < 0 || n_commit > m->pending_rows[seq])
    return ctx->fail(Status::err(WEDLM_ERR_INVALID_ARG,
                                 "n_commit exceeds the rows written by the last forward"));
  m->cache_len[seq] += n_commit;
  m->pending_rows[seq] = 0;
  return WEDLM_OK;
}

int wedlm_truncate(wedlm_ctx* ctx, int seq, int new_len) {
  if (int rc = model_guard(ctx)) return rc;
  ModelState* m = ctx->model;
  if (seq < 0 || seq >= m->max_seqs || new_len < 0)
    return ctx->fail(Status::err(WEDLM_ERR_INVALID_ARG, "bad seq / length"));
  if (new_len < m->cache_len[seq]) m->cache_len[seq] = new_len;  // truncate_cache: no-op if >=
  m->pending_rows[seq] = 0;
  return WEDLM_OK;
}

int wedlm_prefill(wedlm_ctx* ctx, int seq, const int32_t* ids, int n, void* stream) {
  if (int rc = model_guard(ctx)) return rc;
  ModelState* m = ctx->model;
  if (seq < 0 || seq >= m->max_seqs || n < 0 || (n > 0 && !ids))
    return ctx->fail(Status::err(WEDLM_ERR_INVALID_ARG, "bad prefill arguments"));
  cudaStream_t st = pick_stream(ctx, stream);
  const int chunk = m->max_rows;
  std::vector<int> pos;
  for (int off = 0; off < n; off += chunk) {
    const int c = std::min(chunk, n - off);
    pos.resize(c);
    for (int j = 0; j < c; ++j) pos[j] = m->cache_len[seq] + j;
    std::vector<wedlm::SeqSlice> sl(1);
    sl[0].slot = seq;
    sl[0].rows = c;
    sl[0].logit_begin = c;
    Status s = wedlm::model_forward(ctx, sl, ids + off, pos.data(), nullptr, nullptr, m->dt, nullptr, st);
    if (!s.good()) return ctx->fail(s);
    m->cache_len[seq] += c;
    m->pending_rows[seq] = 0;
  }
  return WEDLM_OK;
}

int wedlm_block_forward(wedlm_ctx* ctx, int nseq, const int32_t* seq_ids, const int32_t* tokens,
                        const int32_t* positions, const int32_t* rank, int S,
                        const int32_t* logit_row_begin, void* logits_out, int logits_dtype,
                        int32_t* n_logit_rows_out, void* stream) {
  if (int rc = model_guard(ctx)) return rc;
  if (nseq < 1 || S < 0 || !seq_ids || (S > 0 && (!tokens || !positions)))
    return ctx->fail(Status::err(WEDLM_ERR_INVALID_ARG, "bad block_forward arguments"));
  std::vector<wedlm::SeqSlice> sl(nseq);
  for (int b = 0; b < nseq; ++b) {
    sl[b].slot = seq_ids[b];
    sl[b].rows = S;
    sl[b].logit_begin = logit_row_begin ? logit_row_begin[b] : 0;
    for (int c = 0; c < b; ++c)
      if (sl[c].slot == sl[b].slot)
        return ctx->fail(Status::err(WEDLM_ERR_INVALID_ARG, "a sequence appears twice"));
  }
  int nl = 0;
  Status s = wedlm::model_forward(ctx, sl, tokens, positions, rank, logits_out, logits_dtype, &nl,
                                  pick_stream(ctx, stream));
  if (!s.good()) return ctx->fail(s);
  if (n_logit_rows_out) *n_logit_rows_out = nl;
  return WEDLM_OK;
}

}  // extern "C"
