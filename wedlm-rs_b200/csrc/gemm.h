// Projection GEMMs: Y[tok, n] = sum_k X[tok, k] * W[n, k] with fused epilogues.
#pragma once

#include "common.cuh"

namespace wedlm {

enum GemmEpilogue {
  EPI_STORE_BF16 = 0,   // Y -> bf16
  EPI_STORE_F32 = 1,    // Y -> f32
  EPI_RESID_BF16 = 2,   // out = bf16(resid + bf16(Y))            (residual add)
  EPI_SWIGLU_BF16 = 3,  // out = bf16(silu(bf16(Y_gate)) * bf16(Y_up))
};

// Weight tiles pre-packed for streaming: tile (n_tile, k-block) of 128 rows x 64 columns
// is one contiguous 16 KB block at ((n_tile * (K / 64) + kb) * 16 KB) holding the
// 128-byte-swizzled shared-memory image the MMA descriptors expect, so a pipeline stage
// is one sequential 1-D bulk copy.  Rows past N are zero.
long packed_weight_elems(long N, long K);
// Pack rows [0, rows) of a row-major bf16 block (row stride ld) as global rows
// [row_off, row_off + rows) of a packed [*, K] matrix.
Status pack_weight(const void* src, long ld, long row_off, long rows, long K, void* packed,
                   cudaStream_t st);
Status unpack_weight(const void* packed, long row_off, long rows, long K, void* dst,
                     cudaStream_t st);
// N(0, std^2) values of a counter-based hash of (seed, tensor_id, logical index) written
// straight into the packed positions of rows [row_off, row_off + rows).
// The hash index of element (r, c) is hash_off + r * K + c.
Status init_normal_packed(void* packed, long row_off, long rows, long K, uint64_t seed,
                          uint64_t tensor_id, long hash_off, float stdv, cudaStream_t st);

// Split-K partial outputs consumed by the next kernel (slot mode): tile t's partial from
// its r-th contributing CTA (r = cta - first contributor) is the f32 block at
// slots + ((t * maxc + r) * na + a) * tok_tile * 128, laid out [tok][128 weight rows];
// a = 0, or 1 for the up projection of SwiGLU.  A consumer sums the contributors of a
// tile in order (deterministic) and applies the epilogue itself.
struct PartialSet {
  const float* slots = nullptr;
  long iters = 0;
  int grid = 1, kb_total = 1, t_tiles = 1, tok_tile = 16, maxc = 1, na = 1;
  int nb = 1;  // weight tiles per stream-K unit
};

struct GemmArgs {
  const void* X = nullptr;  // [M, K] (row stride ldx)
  long ldx = 0;
  const void* W = nullptr;  // [N, K] (row stride ldw), or packed tiles when w_packed
  const void* W2 = nullptr; // second [N, K] matrix (SwiGLU up projection)
  long ldw = 0;
  bool w_packed = false;
  float* slots = nullptr;   // slot mode: every tile's partials go here (out / resid unused)
  int M = 0, N = 0, K = 0;
  int epi = EPI_STORE_BF16;
  void* out = nullptr;      // [M, N] (row stride ldo)
  long ldo = 0;
  const void* resid = nullptr;  // [M, N] (row stride ldr); may alias out
  long ldr = 0;
};

struct GemmPlan {
  int tok_tile = 0, t_tiles = 0, n_tiles = 0, kb_total = 0, splits = 1, stages = 0;
  int nb = 1;  // weight tiles per stream-K unit (sharing the activation k-blocks)
  int grid = 0, nbuf = 1, maxc = 1;
  int ks = 1, kb64 = 0;  // 64-wide k-blocks per pipeline stage, k-blocks per weight row
  uint32_t stage_bytes = 0, tmem_cols = 0, smem_bytes = 0, acc_cols = 0;
  long ws_floats = 0;    // direct mode: shared-tile partials (two slots per CTA)
  long slot_floats = 0;  // slot mode: size of the partial set
  int counters = 0;
};

// bf16 tcgen05 path (K % 64 == 0).
// force_nb = 1 or 2 fixes the weight tiles per stream-K unit (0: chosen by size).
GemmPlan plan_gemm_tc(int M, int N, int K, bool dual, int num_sms, int force_nb = 0);
Status run_gemm_tc(const GemmArgs& a, const GemmPlan& g, float* ws, unsigned* counters, int* err,
                   cudaStream_t st);
void forget_tensor_maps();
PartialSet partial_set(const GemmPlan& g, const float* slots, bool dual);

// f32 path (CUDA cores, for f32 models): same epilogues with f32 storage.
Status run_gemm_f32(const GemmArgs& a, cudaStream_t st);

// ---- partial-set readers for consumer kernels ----------------------------------------
__device__ __forceinline__ long ps_owner(long x, long iters, int grid) {
  long c = ((x + 1) * grid + iters - 1) / iters - 1;
  return c < 0 ? 0 : (c >= grid ? grid - 1 : c);
}
// Sum of the contributors of output (tok, n), accumulator a, in CTA order.
__device__ __forceinline__ float ps_sum(const PartialSet& p, int tok, int n, int a) {
  const int tile = (n >> 7) * p.t_tiles + tok / p.tok_tile;
  const long x0 = (long)(((n >> 7) / p.nb) * p.t_tiles + tok / p.tok_tile) * p.kb_total;
  const int cf = (int)ps_owner(x0, p.iters, p.grid);
  const int cl = (int)ps_owner(x0 + p.kb_total - 1, p.iters, p.grid);
  const float* base = p.slots + ((long)tile * p.maxc * p.na + a) * p.tok_tile * 128 +
                      (long)(tok % p.tok_tile) * 128 + (n & 127);
  const long stride = (long)p.na * p.tok_tile * 128;
  float s = 0.f;
  for (int r = 0; r <= cl - cf; ++r) s += __ldcg(base + r * stride);
  return s;
}

// Contributor range of the tile holding output (tok, n): base of contributor 0 for
// accumulator a, the slot stride between contributors, and their count.
struct PsTile {
  const float* base;
  long stride;
  int count;
};
__device__ __forceinline__ PsTile ps_tile(const PartialSet& p, int tok, int n, int a) {
  const int tile = (n >> 7) * p.t_tiles + tok / p.tok_tile;
  // first k-step of the stream-K unit holding weight tile n >> 7 (nb tiles per unit)
  const long x0 = (long)(((n >> 7) / p.nb) * p.t_tiles + tok / p.tok_tile) * p.kb_total;
  const int cf = (int)ps_owner(x0, p.iters, p.grid);
  const int cl = (int)ps_owner(x0 + p.kb_total - 1, p.iters, p.grid);
  PsTile t;
  t.base = p.slots + ((long)tile * p.maxc * p.na + a) * p.tok_tile * 128 +
           (long)(tok % p.tok_tile) * 128 + (n & 127);
  t.stride = (long)p.na * p.tok_tile * 128;
  t.count = cl - cf + 1;
  return t;
}
// Sum of 4 consecutive outputs n .. n+3 (n % 4 == 0, same tile), contributors in order.
__device__ __forceinline__ float4 ps_sum4(const PsTile& t) {
  float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
  int r = 0;
  for (; r + 2 <= t.count; r += 2) {
    const float4 u = __ldcg(reinterpret_cast<const float4*>(t.base + r * t.stride));
    const float4 v = __ldcg(reinterpret_cast<const float4*>(t.base + (r + 1) * t.stride));
    s.x += u.x; s.y += u.y; s.z += u.z; s.w += u.w;
    s.x += v.x; s.y += v.y; s.z += v.z; s.w += v.w;
  }
  if (r < t.count) {
    const float4 u = __ldcg(reinterpret_cast<const float4*>(t.base + r * t.stride));
    s.x += u.x; s.y += u.y; s.z += u.z; s.w += u.w;
  }
  return s;
}
// Same sum with the loads of up to B contributors issued back to back before any add:
// slots past the count load contributor 0 again (in bounds, never added), so no load is
// behind a branch.  Longer contributor lists take ps_sum4.
template <int B>
__device__ __forceinline__ float4 ps_sum4_nb(const PsTile& t) {
  if (t.count > B) return ps_sum4(t);
  float4 u[B];
#pragma unroll
  for (int k = 0; k < B; ++k)
    u[k] = __ldcg(reinterpret_cast<const float4*>(t.base + (k < t.count ? k : 0) * t.stride));
  float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int k = 0; k < B; ++k)
    if (k < t.count) {
      s.x += u[k].x; s.y += u[k].y; s.z += u[k].z; s.w += u[k].w;
    }
  return s;
}

// Same sum with each of up to B loads predicated on the contributor count (no redundant
// requests), all issued before the adds; the additions run in the same order as ps_sum4.
template <int B>
__device__ __forceinline__ float4 ps_sum4_pred(const PsTile& t) {
  if (t.count > B) return ps_sum4(t);
  float4 u[B];
#pragma unroll
  for (int k = 0; k < B; ++k)
    if (k < t.count) u[k] = __ldcg(reinterpret_cast<const float4*>(t.base + k * t.stride));
  float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int k = 0; k < B; ++k)
    if (k < t.count) {
      s.x += u[k].x; s.y += u[k].y; s.z += u[k].z; s.w += u[k].w;
    }
  return s;
}

}  // namespace wedlm
