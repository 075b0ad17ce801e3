// Element-wise and row-wise kernels of the decoder layer:
//   embedding gather            src/model/backbone.rs:37-58 (on the device, no host trip)
//   RMSNorm                     src/model/attention.rs:35-50
//   QK-norm + RoPE + KV append  src/model/attention.rs:149-184, src/model/rope.rs:132-197
//   f32 attention (CUDA cores)  src/model/attention.rs:188-199 for f32 models
// Rounding follows the reference for bf16 models: RMSNorm computes in f32 and casts
// back; RoPE uses cos/sin tables rounded to the model dtype (rope.rs:94-95) and rounds
// its output.
#include "layer_ops.h"
#include "layer_ops_dev.cuh"

#include <algorithm>

namespace wedlm {

namespace {

template <typename T>
__device__ __forceinline__ T rnd(float v) {
  return rnd_to<T>(v);
}

// ---- embedding -------------------------------------------------------------------
template <typename T>
__global__ void embed_kernel(const T* __restrict__ table, const int* __restrict__ ids, int H,
                             T* __restrict__ out, int vocab, int* err, const int* act) {
  pdl_trigger();
  pdl_wait();
  const int r = blockIdx.x;
  if (act && !act[r]) return;  // a padding row of the device loop
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
// One warp per (row, head) over the q, k and v heads of the fused QKV output
// (rope_kv_item, layer_ops_dev.cuh).
template <typename T, int E>
__global__ void rope_kv_kernel(RopeKvArgs a, PartialSet ps_val) {
  pdl_trigger();
  pdl_wait();
  const int warps = blockDim.x >> 5;
  const int gw = blockIdx.x * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int heads = a.nh + 2 * a.nkv;
  if (gw >= a.rows * heads) return;
  if (a.row_active && !a.row_active[gw / heads]) return;  // a padding row of the device loop
  rope_kv_item<T, E>(a, a.qkv_partials != nullptr ? &ps_val : nullptr, gw, lane);
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

// ---- residual add (from split-K partials) fused with the next RMSNorm ----------------
// The row stays in registers (two groups of four values per thread when H <= 8 *
// blockDim), so the kernel needs no row buffer in shared memory.  Wider rows keep the row
// in dynamic shared memory.  At 68 registers a 512-thread CTA does not fit on an SM beside
// a GEMM CTA (192 threads x 168 registers); making it fit, by holding this kernel to 64
// registers or the GEMM to 144, made the 8B decode step 2% slower.
template <bool kRegs>
__global__ void __launch_bounds__(512)
resid_norm_kernel(__nv_bfloat16* h, PartialSet ps, int has_ps, const float* __restrict__ w,
                  int H, float eps, __nv_bfloat16* xn, const int* act) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ float srow[];
  const int r = blockIdx.x;
  if (act && !act[r]) return;  // a padding row of the device loop
  __nv_bfloat16* hr = h + (long)r * H;
  float ss = 0.f;
  float keep[8];  // kRegs: this thread's values at i0 .. i0 + 3 and i1 .. i1 + 3
  // two float4 groups per iteration, every load of both issued before the arithmetic
  const int step = blockDim.x * 4;
  for (int i0 = threadIdx.x * 4; i0 < H; i0 += 2 * step) {
    const int i1 = i0 + step;
    const bool two = i1 < H;
    const uint2 hw0 = *reinterpret_cast<const uint2*>(hr + i0);
    const uint2 hw1 = two ? *reinterpret_cast<const uint2*>(hr + i1) : hw0;
    float4 y0 = make_float4(0.f, 0.f, 0.f, 0.f), y1 = y0;
    if (has_ps) {
      const PsTile t0 = ps_tile(ps, r, i0, 0);
      const PsTile t1 = ps_tile(ps, r, two ? i1 : i0, 0);
      y0 = ps_sum4_nb<8>(t0);
      y1 = ps_sum4_nb<8>(t1);
    }
#pragma unroll
    for (int g = 0; g < 2; ++g) {
      if (g == 1 && !two) break;
      const int i = g ? i1 : i0;
      const uint2 hw = g ? hw1 : hw0;
      const float4 y = g ? y1 : y0;
      float v[4] = {bf16_lo(hw.x), bf16_hi(hw.x), bf16_lo(hw.y), bf16_hi(hw.y)};
      if (has_ps) {
        const float ys[4] = {y.x, y.y, y.z, y.w};
        uint32_t o[2];
#pragma unroll
        for (int k = 0; k < 4; k += 2) {
          const float a0 = __bfloat162float(__float2bfloat16_rn(v[k] + __bfloat162float(__float2bfloat16_rn(ys[k]))));
          const float a1 = __bfloat162float(__float2bfloat16_rn(v[k + 1] + __bfloat162float(__float2bfloat16_rn(ys[k + 1]))));
          v[k] = a0;
          v[k + 1] = a1;
          const __nv_bfloat162 h2 = __floats2bfloat162_rn(a0, a1);
          o[k / 2] = *reinterpret_cast<const uint32_t*>(&h2);
        }
        *reinterpret_cast<uint2*>(hr + i) = make_uint2(o[0], o[1]);
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        if (kRegs) keep[g * 4 + k] = v[k];
        else srow[i + k] = v[k];
        ss = fmaf(v[k], v[k], ss);
      }
    }
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
  __nv_bfloat16* xr = xn + (long)r * H;
  if (kRegs) {
#pragma unroll
    for (int g = 0; g < 2; ++g) {
      const int i = threadIdx.x * 4 + g * step;
      if (i >= H) break;
      const float* v = keep + g * 4;
      const __nv_bfloat162 a = __floats2bfloat162_rn((v[0] / denom) * w[i], (v[1] / denom) * w[i + 1]);
      const __nv_bfloat162 b = __floats2bfloat162_rn((v[2] / denom) * w[i + 2], (v[3] / denom) * w[i + 3]);
      *reinterpret_cast<uint2*>(xr + i) =
          make_uint2(*reinterpret_cast<const uint32_t*>(&a), *reinterpret_cast<const uint32_t*>(&b));
    }
  } else {
    for (int i = threadIdx.x * 4; i < H; i += blockDim.x * 4) {
      const __nv_bfloat162 a = __floats2bfloat162_rn((srow[i] / denom) * w[i], (srow[i + 1] / denom) * w[i + 1]);
      const __nv_bfloat162 b = __floats2bfloat162_rn((srow[i + 2] / denom) * w[i + 2], (srow[i + 3] / denom) * w[i + 3]);
      *reinterpret_cast<uint2*>(xr + i) =
          make_uint2(*reinterpret_cast<const uint32_t*>(&a), *reinterpret_cast<const uint32_t*>(&b));
    }
  }
}

// ---- SwiGLU from the gate/up partials (swiglu_range, layer_ops_dev.cuh) -------------
__global__ void swiglu_kernel(PartialSet ps, int rows, int I, __nv_bfloat16* act,
                              const int* row_active) {
  pdl_trigger();
  pdl_wait();
  swiglu_range(ps, rows, I, act, blockIdx.x * (long)blockDim.x + threadIdx.x,
               (long)gridDim.x * blockDim.x, row_active);
}

}  // namespace

Status run_resid_norm(void* h, const PartialSet* ps, const float* w, int rows, int H, float eps,
                      void* xn, cudaStream_t st, const int* row_active) {
  if (rows == 0) return Status::ok();
  WEDLM_CHECK_ARG(H % 4 == 0, "hidden size must be a multiple of 4");
  const PartialSet p = ps ? *ps : PartialSet();
  if (H <= 8 * 512)
    WEDLM_CUDA_TRY(launch_pdl(resid_norm_kernel<true>, dim3(rows), dim3(512), 0, st,
                              (__nv_bfloat16*)h, p, ps ? 1 : 0, w, H, eps, (__nv_bfloat16*)xn,
                              row_active));
  else
    WEDLM_CUDA_TRY(launch_pdl(resid_norm_kernel<false>, dim3(rows), dim3(512),
                              (size_t)H * sizeof(float), st, (__nv_bfloat16*)h, p, ps ? 1 : 0, w,
                              H, eps, (__nv_bfloat16*)xn, row_active));
  return Status::ok();
}

Status run_swiglu(const PartialSet& ps, int rows, int I, void* act, cudaStream_t st,
                  const int* row_active) {
  if (rows == 0) return Status::ok();
  WEDLM_CHECK_ARG(I % 4 == 0, "intermediate size must be a multiple of 4");
  const long n4 = (long)rows * I / 4;
  const unsigned grid = (unsigned)std::min<long>((n4 + 255) / 256, 148L * 16);
  WEDLM_CUDA_TRY(launch_pdl(swiglu_kernel, dim3(grid), dim3(256), 0, st, ps, rows, I,
                            (__nv_bfloat16*)act, row_active));
  return Status::ok();
}

Status run_embed(const void* table, int dtype, const int* ids, int rows, int H, int vocab,
                 void* out, int* err, cudaStream_t st, const int* row_active) {
  if (rows == 0) return Status::ok();
  if (dtype == WEDLM_BF16)
    WEDLM_CUDA_TRY(launch_pdl(embed_kernel<__nv_bfloat16>, dim3(rows), dim3(128), 0, st,
                              (const __nv_bfloat16*)table, ids, H, (__nv_bfloat16*)out, vocab, err,
                              row_active));
  else
    WEDLM_CUDA_TRY(launch_pdl(embed_kernel<float>, dim3(rows), dim3(128), 0, st,
                              (const float*)table, ids, H, (float*)out, vocab, err, row_active));
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
  const PartialSet psv = a.qkv_partials ? *a.qkv_partials : PartialSet();
#define WEDLM_ROPE_CASE(EE)                                                              \
  case EE:                                                                               \
    if (dtype == WEDLM_BF16)                                                             \
      WEDLM_CUDA_TRY(launch_pdl(rope_kv_kernel<__nv_bfloat16, EE>, dim3(grid),          \
                                dim3(per_block * 32), 0, st, a, psv));                   \
    else                                                                                 \
      WEDLM_CUDA_TRY(launch_pdl(rope_kv_kernel<float, EE>, dim3(grid), dim3(per_block * 32), \
                                0, st, a, psv));                                         \
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
