// Element-wise and row-wise kernels of the decoder layer:
//   embedding gather            src/model/backbone.rs:37-58 (on the device, no host trip)
//   RMSNorm                     src/model/attention.rs:35-50
//   QK-norm + RoPE + KV append  src/model/attention.rs:149-184, src/model/rope.rs:132-197
//   f32 attention (CUDA cores)  src/model/attention.rs:188-199 for f32 models
// Rounding follows the reference for bf16 models: RMSNorm computes in f32 and casts
// back; RoPE uses cos/sin tables rounded to the model dtype (rope.rs:94-95) and rounds
// its output.
#include "layer_ops.h"

namespace wedlm {

namespace {

template <typename T>
__device__ __forceinline__ T rnd(float v) {
  return from_f32<T>(v);
}

// ---- embedding -------------------------------------------------------------------
template <typename T>
__global__ void embed_kernel(const T* __restrict__ table, const int* __restrict__ ids, int H,
                             T* __restrict__ out, int vocab, int* err) {
  const int r = blockIdx.x;
  int id = ids[r];
  if (id < 0 || id >= vocab) {
    if (threadIdx.x == 0) atomicCAS(err, 0, 100);
    id = 0;
  }
  const T* src = table + (long)id * H;
  T* dst = out + (long)r * H;
  if ((H * sizeof(T)) % 16 == 0) {
    const uint4* s4 = reinterpret_cast<const uint4*>(src);
    uint4* d4 = reinterpret_cast<uint4*>(dst);
    for (int i = threadIdx.x; i < (int)(H * sizeof(T) / 16); i += blockDim.x) d4[i] = s4[i];
  } else {
    for (int i = threadIdx.x; i < H; i += blockDim.x) dst[i] = src[i];
  }
}

// ---- RMSNorm: out = x / sqrt(mean(x^2) + eps) * w --------------------------------
template <typename T>
__global__ void rmsnorm_kernel(const T* __restrict__ x, long ldx, const float* __restrict__ w,
                               int H, float eps, T* __restrict__ out, long ldo) {
  const int r = blockIdx.x;
  const T* xr = x + (long)r * ldx;
  float ss = 0.f;
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    float v = to_f32(xr[i]);
    ss = fmaf(v, v, ss);
  }
  __shared__ float sh[32];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? sh[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) sh[0] = v;
  }
  __syncthreads();
  const float denom = sqrtf(sh[0] / (float)H + eps);
  T* orow = out + (long)r * ldo;
  for (int i = threadIdx.x; i < H; i += blockDim.x)
    orow[i] = rnd<T>((to_f32(xr[i]) / denom) * w[i]);
}

// ---- QK-norm + RoPE + KV append ------------------------------------------------------
// One warp per (row, head) over the q, k and v heads of the fused QKV output.  Head
// dim d = 32 * E; lane holds elements lane*E .. lane*E+E-1; the rotate-half partner of
// element i (i +/- d/2) sits in lane ^ 16 at the same slot.
template <typename T, int E>
__global__ void rope_kv_kernel(RopeKvArgs a) {
  const int warps = blockDim.x >> 5;
  const int gw = blockIdx.x * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int heads = a.nh + 2 * a.nkv;
  if (gw >= a.rows * heads) return;
  const int r = gw / heads, hh = gw % heads;
  const int d = 32 * E;
  const T* src = reinterpret_cast<const T*>(a.qkv) + (long)r * a.ld_qkv + (long)hh * d;
  float x[E];
#pragma unroll
  for (int e = 0; e < E; ++e) x[e] = to_f32(src[lane * E + e]);
  const bool is_q = hh < a.nh, is_k = !is_q && hh < a.nh + a.nkv;
  if (is_q || is_k) {
    if (a.qk_norm) {
      const float* w = is_q ? a.q_norm : a.k_norm;
      float ss = 0.f;
#pragma unroll
      for (int e = 0; e < E; ++e) ss = fmaf(x[e], x[e], ss);
      ss = warp_sum(ss);
      const float denom = sqrtf(ss / (float)d + a.eps);
#pragma unroll
      for (int e = 0; e < E; ++e) x[e] = to_f32(rnd<T>((x[e] / denom) * w[lane * E + e]));
    }
    const int pos = a.positions[r];
    const float* cs = a.cos + (long)pos * (d / 2);
    const float* sn = a.sin + (long)pos * (d / 2);
    float y[E];
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const float p = __shfl_xor_sync(0xffffffffu, x[e], 16);
      const int fi = (lane & 15) * E + e;
      const float c = cs[fi], s = sn[fi];
      y[e] = lane < 16 ? x[e] * c - p * s : x[e] * c + p * s;
    }
#pragma unroll
    for (int e = 0; e < E; ++e) x[e] = to_f32(rnd<T>(y[e]));
  }
  if (is_q) {
    // group-major q: [nkv][rows * group][d], row index (r * group + h % group)
    const int g = hh / a.group, hi = hh % a.group;
    T* dst = reinterpret_cast<T*>(a.q_out) +
             (((long)g * a.rows + r) * a.group + hi) * d;
#pragma unroll
    for (int e = 0; e < E; ++e) dst[lane * E + e] = rnd<T>(x[e]);
    return;
  }
  // K / V into the paged cache at position dst_pos[r] of sequence row_seq[r]
  const int kvh = is_k ? hh - a.nh : hh - a.nh - a.nkv;
  const int seq = a.row_seq[r];
  const int tpos = a.dst_pos[r];
  const int page = a.page_table[(long)seq * a.pages_per_seq + tpos / a.page_size];
  const int off = tpos % a.page_size;
  const long page_base = (((long)a.layer * a.num_pages + page) * a.nkv + kvh) * (long)a.page_size * d;
  if (is_k) {
    T* dst = reinterpret_cast<T*>(a.kcache) + page_base + (long)off * d;
#pragma unroll
    for (int e = 0; e < E; ++e) dst[lane * E + e] = rnd<T>(x[e]);
  } else {
    // V stored transposed within a page: [d][page_size]
    T* dst = reinterpret_cast<T*>(a.vcache) + page_base + off;
#pragma unroll
    for (int e = 0; e < E; ++e) dst[(long)(lane * E + e) * a.page_size] = rnd<T>(x[e]);
  }
}

// ---- attention on CUDA cores (f32 models) -------------------------------------------
// One warp per (row, q head).  Keys: every cached key of the sequence (positions
// 0 .. cache_len-1) plus the block keys j with rank[j] <= rank[i].
__global__ void attention_f32_kernel(AttnArgs a) {
  const int warps = blockDim.x >> 5;
  const int gw = blockIdx.x * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (gw >= a.rows * a.nh) return;
  const int r = gw / a.nh, h = gw % a.nh;
  const int g = h / a.group, hi = h % a.group;
  const int d = a.head_dim;
  const int b = a.row_seq[r];
  const int slot = a.seq_slot[b];
  const int L = a.seq_cache_len[b];
  const int b0 = a.seq_row0[b], S = a.seq_rows[b];
  const int my_rank = a.rank ? a.rank[r] : r - b0;
  const float* q = reinterpret_cast<const float*>(a.q) + (((long)g * a.rows + r) * a.group + hi) * d;
  const float scale = rsqrtf((float)d);
  float m = -INFINITY, l = 0.f;
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};  // d <= 256
  const float* K = reinterpret_cast<const float*>(a.kcache);
  const float* Vt = reinterpret_cast<const float*>(a.vcache);
  for (int t = 0; t < L + S; ++t) {
    if (t >= L) {
      const int j = t - L;
      const int rk = a.rank ? a.rank[b0 + j] : j;
      if (rk > my_rank) continue;
    }
    const int page = a.page_table[(long)slot * a.pages_per_seq + t / a.page_size];
    const int off = t % a.page_size;
    const long base = (((long)a.layer * a.num_pages + page) * a.nkv + g) * (long)a.page_size * d;
    float s = 0.f;
    for (int i = lane; i < d; i += 32) s = fmaf(q[i], K[base + (long)off * d + i], s);
    s = warp_sum(s) * scale;
    const float mn = fmaxf(m, s);
    const float corr = expf(m - mn), p = expf(s - mn);
    l = l * corr + p;
    for (int k = 0; k * 32 + lane < d; ++k)
      acc[k] = acc[k] * corr + p * Vt[base + (long)(k * 32 + lane) * a.page_size + off];
    m = mn;
  }
  float* o = reinterpret_cast<float*>(a.out) + (long)r * a.ld_out + (long)h * d;
  for (int k = 0; k * 32 + lane < d; ++k) o[k * 32 + lane] = acc[k] / l;
}

}  // namespace

Status run_embed(const void* table, int dtype, const int* ids, int rows, int H, int vocab,
                 void* out, int* err, cudaStream_t st) {
  if (rows == 0) return Status::ok();
  if (dtype == WEDLM_BF16)
    embed_kernel<__nv_bfloat16><<<rows, 128, 0, st>>>((const __nv_bfloat16*)table, ids, H,
                                                      (__nv_bfloat16*)out, vocab, err);
  else
    embed_kernel<float><<<rows, 128, 0, st>>>((const float*)table, ids, H, (float*)out, vocab, err);
  WEDLM_CUDA_TRY(cudaGetLastError());
  return Status::ok();
}

Status run_rmsnorm(const void* x, long ldx, const float* w, int rows, int H, float eps, int dtype,
                   void* out, long ldo, cudaStream_t st) {
  if (rows == 0) return Status::ok();
  const int threads = H >= 1024 ? 512 : 256;
  if (dtype == WEDLM_BF16)
    rmsnorm_kernel<__nv_bfloat16><<<rows, threads, 0, st>>>(
        (const __nv_bfloat16*)x, ldx, w, H, eps, (__nv_bfloat16*)out, ldo);
  else
    rmsnorm_kernel<float><<<rows, threads, 0, st>>>((const float*)x, ldx, w, H, eps, (float*)out,
                                                    ldo);
  WEDLM_CUDA_TRY(cudaGetLastError());
  return Status::ok();
}

Status run_rope_kv(const RopeKvArgs& a, int dtype, cudaStream_t st) {
  if (a.rows == 0) return Status::ok();
  const int heads = a.nh + 2 * a.nkv;
  const long warps = (long)a.rows * heads;
  const int per_block = 8;
  const unsigned grid = (unsigned)((warps + per_block - 1) / per_block);
  const int E = a.head_dim / 32;
  WEDLM_CHECK_ARG(a.head_dim % 32 == 0 && E >= 1 && E <= 8, "head_dim must be 32..256, multiple of 32");
#define WEDLM_ROPE_CASE(EE)                                                              \
  case EE:                                                                               \
    if (dtype == WEDLM_BF16)                                                             \
      rope_kv_kernel<__nv_bfloat16, EE><<<grid, per_block * 32, 0, st>>>(a);            \
    else                                                                                 \
      rope_kv_kernel<float, EE><<<grid, per_block * 32, 0, st>>>(a);                    \
    break;
  switch (E) {
    WEDLM_ROPE_CASE(1)
    WEDLM_ROPE_CASE(2)
    WEDLM_ROPE_CASE(4)
    WEDLM_ROPE_CASE(8)
    default:
      return Status::err(WEDLM_ERR_UNSUPPORTED, "head_dim must be 32, 64, 128 or 256");
  }
#undef WEDLM_ROPE_CASE
  WEDLM_CUDA_TRY(cudaGetLastError());
  return Status::ok();
}

Status run_attention_f32(const AttnArgs& a, cudaStream_t st) {
  if (a.rows == 0) return Status::ok();
  WEDLM_CHECK_ARG(a.head_dim <= 256, "head_dim > 256");
  const long warps = (long)a.rows * a.nh;
  const unsigned grid = (unsigned)((warps + 7) / 8);
  attention_f32_kernel<<<grid, 256, 0, st>>>(a);
  WEDLM_CUDA_TRY(cudaGetLastError());
  return Status::ok();
}

}  // namespace wedlm
