// Device-side bodies of the per-row / per-element consumer kernels of the decoder layer,
// shared by the stand-alone kernels (layer_ops.cu) and the fused layer tail
// (layer_fused.cu) so that both compute the same values bit for bit.
//   QK-norm + RoPE + KV append  src/model/attention.rs:149-184, src/model/rope.rs:132-197
//   SwiGLU                      src/model/mlp.rs:40-43
#pragma once

#include "gemm.h"
#include "layer_ops.h"

namespace wedlm {

template <typename T>
__device__ __forceinline__ T rnd_to(float v) {
  return from_f32<T>(v);
}

// QK-norm + RoPE + KV append of row r, head hh (q heads, then k heads, then v heads)
// from its projection values x (rounded to the model dtype), by one warp.  Head dim
// d = 32 * E; lane holds elements lane*E .. lane*E+E-1; the rotate-half partner of
// element i (i +/- d/2) sits in lane ^ 16 at the same slot.
template <typename T, int E>
__device__ __forceinline__ void rope_kv_apply(const RopeKvArgs& a, float (&x)[E], int r, int hh,
                                              int lane) {
  const int d = 32 * E;
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
      for (int e = 0; e < E; ++e) x[e] = to_f32(rnd_to<T>((x[e] / denom) * w[lane * E + e]));
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
    for (int e = 0; e < E; ++e) x[e] = to_f32(rnd_to<T>(y[e]));
  }
  if (is_q) {
    // group-major q: [nkv][rows * group][d], row index (r * group + h % group)
    const int g = hh / a.group, hi = hh % a.group;
    T* dst = reinterpret_cast<T*>(a.q_out) + (((long)g * a.rows + r) * a.group + hi) * d;
#pragma unroll
    for (int e = 0; e < E; ++e) dst[lane * E + e] = rnd_to<T>(x[e]);
    return;
  }
  // K / V into the paged cache at position dst_pos[r] of sequence row_seq[r]
  const int kvh = is_k ? hh - a.nh : hh - a.nh - a.nkv;
  const int seq = a.row_seq[r];
  const int tpos = a.dst_pos[r];
  const int page = a.page_table[(long)seq * a.pages_per_seq + tpos / a.page_size];
  const int off = tpos % a.page_size;
  const long page_base =
      (((long)a.layer * a.num_pages + page) * a.nkv + kvh) * (long)a.page_size * d;
  if (is_k) {
    T* dst = reinterpret_cast<T*>(a.kcache) + page_base + (long)off * d;
#pragma unroll
    for (int e = 0; e < E; ++e) dst[lane * E + e] = rnd_to<T>(x[e]);
  } else {
    // V stored transposed within a page: [d][page_size]
    T* dst = reinterpret_cast<T*>(a.vcache) + page_base + off;
#pragma unroll
    for (int e = 0; e < E; ++e) dst[(long)(lane * E + e) * a.page_size] = rnd_to<T>(x[e]);
  }
}

// QK-norm + RoPE + KV append of one (row, head) item gw = r * heads + hh, by one warp
// (rope_kv_apply).  `ps` != NULL reads the
// QKV projection as split-K partials (summed in order, rounded to the model dtype as the
// reference's Linear returns it), else from a.qkv.
template <typename T, int E>
__device__ __forceinline__ void rope_kv_item(const RopeKvArgs& a, const PartialSet* ps, int gw,
                                             int lane) {
  const int heads = a.nh + 2 * a.nkv;
  const int r = gw / heads, hh = gw % heads;
  const int d = 32 * E;
  float x[E];
  if (ps != nullptr) {
    if (E % 4 == 0) {
#pragma unroll
      for (int e = 0; e < E; e += 4) {
        const PsTile t = ps_tile(*ps, r, hh * d + lane * E + e, 0);
        const float4 v = ps_sum4_nb<8>(t);
        x[e] = to_f32(rnd_to<T>(v.x));
        x[e + 1] = to_f32(rnd_to<T>(v.y));
        x[e + 2] = to_f32(rnd_to<T>(v.z));
        x[e + 3] = to_f32(rnd_to<T>(v.w));
      }
    } else {
#pragma unroll
      for (int e = 0; e < E; ++e)
        x[e] = to_f32(rnd_to<T>(ps_sum(*ps, r, hh * d + lane * E + e, 0)));
    }
  } else {
    const T* src = reinterpret_cast<const T*>(a.qkv) + (long)r * a.ld_qkv + (long)hh * d;
#pragma unroll
    for (int e = 0; e < E; ++e) x[e] = to_f32(src[lane * E + e]);
  }
  rope_kv_apply<T, E>(a, x, r, hh, lane);
}

// act = bf16(silu(bf16(gate)) * bf16(up)) from the gate/up partials, for the groups of
// four consecutive elements e4 = first, first + stride, ... < rows * I / 4.
__device__ __forceinline__ void swiglu_range(const PartialSet& ps, int rows, int I,
                                             __nv_bfloat16* act, long first, long stride,
                                             const int* row_active = nullptr) {
  const long n4 = (long)rows * I / 4;
  for (long e4 = first; e4 < n4; e4 += stride) {
    const long e = e4 * 4;
    const int r = (int)(e / I), j = (int)(e % I);
    if (row_active && !row_active[r]) continue;  // a padding row of the device loop
    const PsTile tg = ps_tile(ps, r, j, 0), tu = ps_tile(ps, r, j, 1);
    const float4 g4 = ps_sum4_nb<4>(tg);
    const float4 u4 = ps_sum4_nb<4>(tu);
    const float gs[4] = {g4.x, g4.y, g4.z, g4.w}, us[4] = {u4.x, u4.y, u4.z, u4.w};
    float y[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float g = __bfloat162float(__float2bfloat16_rn(gs[k]));
      const float u = __bfloat162float(__float2bfloat16_rn(us[k]));
      const float sg = __bfloat162float(__float2bfloat16_rn(g / (1.f + __expf(-g))));
      y[k] = sg * u;
    }
    const __nv_bfloat162 a = __floats2bfloat162_rn(y[0], y[1]);
    const __nv_bfloat162 b = __floats2bfloat162_rn(y[2], y[3]);
    *reinterpret_cast<uint2*>(act + e) =
        make_uint2(*reinterpret_cast<const uint32_t*>(&a), *reinterpret_cast<const uint32_t*>(&b));
  }
}

}  // namespace wedlm
