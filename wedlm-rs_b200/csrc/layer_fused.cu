// Fused layer tail of the bf16 decode step: one persistent tcgen05 kernel per layer.
//
// After the block attention of layer l, a decode window of M <= 96 token rows runs
//   phase 0  O projection            attn  x Wo^T         (src/model/attention.rs:229)
//   step  0  h += O; xn = RMSNorm(h) * ln2                 (layer.rs:72-75)
//   phase 1  gate/up projections     xn x [Wg; Wu]^T       (mlp.rs:40-41)
//   step  1  act = silu(gate) * up                         (mlp.rs:41-43)
//   phase 2  down projection         act x Wd^T            (mlp.rs:44)
//   step  2  h += down; xn = RMSNorm(h) * ln_next          (layer.rs:78, next layer's norm)
//   phase 3  QKV projection of l + 1 xn x Wqkv^T           (attention.rs:145-147)
//   step  3  QK-norm + RoPE + KV append of layer l + 1     (attention.rs:149-184)
// (the last layer stops after step 2 with the final norm).  At 96 rows every projection
// streams its weights from HBM (96 flop per byte, far under the ridge), so the kernel is
// built around one uninterrupted weight stream: the weight producer never waits for an
// activation, it runs ahead through the phases as far as its 128 KB ring allows, while
// the phase boundaries (a grid-wide data dependency each) resolve.  This replaces the
// eight launches per layer of the unfused path (four GEMMs, each followed by a kernel
// that sums its split-K partials) whose fill and drain left the HBM idle between them.
//
// Each projection keeps the stream-K schedule, partial-slot layout and consumer arithmetic
// of the stand-alone GEMM path (plan_gemm_tc, PartialSet, layer_ops_dev.cuh), so the
// fused tail computes the same bits as the unfused kernels.
//
// Warp roles (352 threads, one CTA per SM, grid = number of SMs, cooperative launch):
//   warp 0       weight producer: 1-D bulk copies of packed weight tiles into a ring of
//                four 32 KB granules (one granule per weight tile and k-step);
//   warp 1       TMEM allocator and MMA issuer (one thread), two accumulator buffers;
//   warps 2..5   epilogue (TMEM -> split-K partial slots);
//   warp 6       activation producer: TMA tiles of the phase's input into a 3-stage ring;
//                before phase k > 0 it waits until every CTA has finished step k - 1;
//   warps 2..5 and 7..10 (256 threads) run, between the phases, the consumer step of the
//                phase just finished on this CTA's share of rows or elements.  The step
//                reads the phase's split-K partials from L2 and is latency-bound, so it
//                gets eight warps with every partial load of an item issued before its adds.
// Grid-wide dependencies are counters in global memory (release add / acquire load):
//   sync[4k]     CTAs whose phase-k partials are written
//   sync[4k + 1] CTAs whose share of step k's partial sums is applied (residual added,
//                SwiGLU or RoPE written)
//   sync[4k + 2] CTAs whose rows of step k's RMSNorm are written (phases 0 and 2)
// Every wait is bounded (2 s of %globaltimer) and records a site code.
#include <cudaTypedefs.h>

#include <cstdlib>
#include <cstring>
#include <string>

#include "layer_fused.h"
#include "layer_ops_dev.cuh"
#include "sm100.cuh"
#include "tc_epilogue.cuh"

namespace wedlm {

Status cached_tmap(CUtensorMap* out, const void* base, long rows, long cols, long ld, int box_rows);

namespace {

using namespace sm100;

constexpr int kThreadsF = 352;
constexpr int kStepThreads = 256;  // warps 2..5 and 7..10
constexpr int kTileN = 128;                    // weight rows per tile (MMA M)
constexpr int kBK = 64;                        // k elements per k-block
constexpr int kKBlk = kTileN * kBK * 2;        // 16 KB: one packed tile k-block
constexpr int kGranBytes = 2 * kKBlk;          // one tile's k-step (ks <= 2 k-blocks)
constexpr int kNGran = 4;
constexpr int kXStages = 3;
constexpr int kMaxTok = 96;
constexpr int kXStageBytes = 2 * kMaxTok * kBK * 2;  // 24 KB: ks <= 2 k-blocks of <= 96 rows
constexpr int kAccStride = 256;                // TMEM columns per accumulator buffer
constexpr int kHFused = 4096;                  // hidden size of the fused norm steps
constexpr int kMaxTilesF = 256;                // weight tiles per phase (contributor table)
constexpr int kSmemF = 1024 + kNGran * kGranBytes + kXStages * kXStageBytes + 1024 +
                       4 * kMaxTilesF + 4 * 32 * 33 * 4;
constexpr int kPfDefault = 0;                  // L2 prefetch distance, in 32 KB granules

struct FPhase {
  const uint8_t* w;   // packed weight tiles
  const uint8_t* w2;  // up projection (na == 2), else == w
  int n_tiles, kb64, ks, nb, na, kb_total, maxc;
  long iters;         // units * kb_total (one token tile)
};

struct FusedParams {
  FPhase ph[4];
  PartialSet ps[4];   // readers of each phase's partial slots
  int nphase, grid, M, tok_tile, H, I;
  float eps;
  float* slots;
  int* err;
  unsigned* sync;
  __nv_bfloat16* h;
  __nv_bfloat16* xn;
  __nv_bfloat16* act;
  const float* ln2;
  const float* ln_next;
  RopeKvArgs rope;
  FPhase pf_next;     // the next layer's O projection, prefetched into L2 only
  int pf_ahead;       // L2 prefetch distance in granules (0 = off)
  int tb[4];          // token rows per block of each phase's consumer step
};

__device__ __forceinline__ long range_start(long c, long iters, int grid) {
  return c * iters / grid;
}
__device__ __forceinline__ int owner_cta(long x, long iters, int grid) {
  long c = ((x + 1) * grid + iters - 1) / iters - 1;
  return (int)(c < 0 ? 0 : (c >= grid ? grid - 1 : c));
}
__device__ __forceinline__ int unit_tiles(const FPhase& f, int u) {
  const int left = f.n_tiles - u * f.nb;
  return left < f.nb ? left : f.nb;
}

struct Seg {
  long it0, it1;
  int unit;
};
__device__ __forceinline__ Seg segment_at(long it, long end, int kb_total) {
  Seg s;
  s.unit = (int)(it / kb_total);
  const long unit_end = (long)(s.unit + 1) * kb_total;
  s.it0 = it;
  s.it1 = end < unit_end ? end : unit_end;
  return s;
}

// ---- consumer steps ---------------------------------------------------------------
// Between two phases the 256 step threads reduce the phase's split-K partials.  The
// partials (tens of MB per layer) are read with 1-D bulk copies into the activation
// ring, which is idle between phases: loads through the load/store unit are limited by
// the outstanding requests an SM can track, bulk copies are not.  A block is (weight
// tile t, token rows b0 .. b0 + ntok); contributor r's accumulator a of the block is one
// contiguous run of ntok x 128 floats in the slot layout of gemm.h (one token tile, one
// weight tile per unit), copied to stage + ((r * na + a) * tb + tok) * 128.  Contributors
// are summed in order from 0.f, as the stand-alone consumer kernels do.
enum StepOp { kOpResid = 0, kOpSwiglu = 1, kOpRope = 2 };

struct StepCtx {
  uint8_t* stage;       // kXStages stages of kXStageBytes (the activation ring)
  uint64_t* sfull;      // [kXStages] completion of each stage's copies
  const uint8_t* cnt;   // contributors per tile of this phase
  uint32_t sb;          // blocks this CTA has staged so far (stage / parity of the next)
};

__device__ __forceinline__ void step_issue(const FusedParams& p, const FPhase& f, const StepCtx& sc,
                                           int tb, int nbt, int bi, uint32_t n, uint64_t pol) {
  const int t = bi / nbt, b0 = (bi - t * nbt) * tb;
  const int ntok = min(tb, p.M - b0);
  const int c = sc.cnt[t];
  const int s = (int)(n % kXStages);
  uint8_t* dst = sc.stage + s * kXStageBytes;
  const uint32_t piece = (uint32_t)ntok * 512u;
  mbar_arrive_expect_tx(sc.sfull + s, piece * (uint32_t)(c * f.na));
  const long acc_stride = (long)p.tok_tile * 128;
  const long contrib_stride = f.na * acc_stride;
  const float* src0 = p.slots + (long)t * f.maxc * contrib_stride + (long)b0 * 128;
  for (int r = 0; r < c; ++r)
    for (int a2 = 0; a2 < f.na; ++a2)
      bulk_load_hint(dst + ((r * f.na + a2) * tb) * 512, src0 + r * contrib_stride + a2 * acc_stride,
                     piece, sc.sfull + s, pol);
}

// One phase's block reduction on this CTA's blocks (bi = cta, cta + grid, ...), pipelined
// kXStages deep.  Step thread st == 0 issues the copies.
template <int OP>
__device__ __forceinline__ void step_blocks(const FusedParams& p, int ph, StepCtx& sc, int st,
                                            int lane, int cta) {
  const FPhase& f = p.ph[ph];
  const int tb = p.tb[ph];
  const int nbt = (p.M + tb - 1) / tb;
  const int nblk = f.n_tiles * nbt;
  const int mine = cta < nblk ? (nblk - 1 - cta) / p.grid + 1 : 0;
  const uint64_t pol = policy_evict_first();  // read once
  if (st == 0)
    for (int j = 0; j < mine && j < kXStages; ++j)
      step_issue(p, f, sc, tb, nbt, cta + j * p.grid, sc.sb + j, pol);
  for (int j = 0; j < mine; ++j) {
    const uint32_t n = sc.sb + j;
    const int s = (int)(n % kXStages);
    mbar_wait(sc.sfull + s, (n / kXStages) & 1u, p.err, kErrFuStep);
    const float* stg = reinterpret_cast<const float*>(sc.stage + s * kXStageBytes);
    const int bi = cta + j * p.grid;
    const int t = bi / nbt, b0 = (bi - t * nbt) * tb;
    const int ntok = min(tb, p.M - b0);
    const int c = sc.cnt[t];
    if (OP == kOpRope) {
      const int w = st >> 5;  // one token row per warp
      if (w < ntok) {
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int r = 0; r < c; ++r) {
          const float4 u = *reinterpret_cast<const float4*>(stg + ((r * tb) + w) * 128 + lane * 4);
          acc.x += u.x; acc.y += u.y; acc.z += u.z; acc.w += u.w;
        }
        float x[4] = {to_f32(rnd_to<__nv_bfloat16>(acc.x)), to_f32(rnd_to<__nv_bfloat16>(acc.y)),
                      to_f32(rnd_to<__nv_bfloat16>(acc.z)), to_f32(rnd_to<__nv_bfloat16>(acc.w))};
        rope_kv_apply<__nv_bfloat16, 4>(p.rope, x, b0 + w, t, lane);
      }
    } else if (st < ntok * 32) {
      const int tok = st >> 5, col = (st & 31) * 4;
      float4 g = make_float4(0.f, 0.f, 0.f, 0.f), u = g;
      for (int r = 0; r < c; ++r) {
        const float4 v = *reinterpret_cast<const float4*>(stg + ((r * f.na) * tb + tok) * 128 + col);
        g.x += v.x; g.y += v.y; g.z += v.z; g.w += v.w;
        if (OP == kOpSwiglu) {
          const float4 w4 =
              *reinterpret_cast<const float4*>(stg + ((r * f.na + 1) * tb + tok) * 128 + col);
          u.x += w4.x; u.y += w4.y; u.z += w4.z; u.w += w4.w;
        }
      }
      const long e = (long)(b0 + tok) * (OP == kOpSwiglu ? p.I : kHFused) + t * 128 + col;
      const float gs[4] = {g.x, g.y, g.z, g.w};
      float yv[4];
      if (OP == kOpSwiglu) {
        const float us[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float gg = __bfloat162float(__float2bfloat16_rn(gs[k]));
          const float uu = __bfloat162float(__float2bfloat16_rn(us[k]));
          const float sg = __bfloat162float(__float2bfloat16_rn(gg / (1.f + __expf(-gg))));
          yv[k] = sg * uu;
        }
      } else {
        // residual (layer.rs:72,78): h = bf16(h + bf16(projection))
        const uint2 hw = __ldcg(reinterpret_cast<const uint2*>(p.h + e));
        const float hv[4] = {bf16_lo(hw.x), bf16_hi(hw.x), bf16_lo(hw.y), bf16_hi(hw.y)};
#pragma unroll
        for (int k = 0; k < 4; ++k) yv[k] = hv[k] + __bfloat162float(__float2bfloat16_rn(gs[k]));
      }
      const __nv_bfloat162 y0 = __floats2bfloat162_rn(yv[0], yv[1]);
      const __nv_bfloat162 y1 = __floats2bfloat162_rn(yv[2], yv[3]);
      *reinterpret_cast<uint2*>((OP == kOpSwiglu ? p.act : p.h) + e) =
          make_uint2(*reinterpret_cast<const uint32_t*>(&y0), *reinterpret_cast<const uint32_t*>(&y1));
    }
    // the stage is read (generic proxy) before the next copy (async proxy) overwrites it
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    named_bar_sync(2, kStepThreads);
    if (st == 0 && j + kXStages < mine)
      step_issue(p, f, sc, tb, nbt, cta + (j + kXStages) * p.grid, n + kXStages, pol);
  }
  sc.sb += (uint32_t)mine;
}

// RMSNorm of row r of h into xn (h already holds the residual sum), on the 256 step
// threads.  Reproduces resid_norm_kernel (512 threads) bit for bit: thread st stands for
// that kernel's threads t = st + 256 q (q = 0, 1), which own elements 4t .. 4t+3 and
// 2048 + 4t .. +3 of a 4096-wide row, and the sums of squares go through the same two
// shuffle trees (per 32-thread warp of the 512, then over the 16 warp totals).
__device__ __forceinline__ void step_row_norm(int r, const __nv_bfloat16* h,
                                              const float* __restrict__ w, float eps,
                                              __nv_bfloat16* xn, float* sred, int st) {
  const int lane = st & 31, wq = st >> 5;
  const __nv_bfloat16* hr = h + (long)r * kHFused;
  float v[16];
  float ssq[2] = {0.f, 0.f};
#pragma unroll
  for (int q = 0; q < 2; ++q)
#pragma unroll
    for (int g = 0; g < 2; ++g) {
      // h rows were just written by other CTAs: read them from L2
      const uint2 hw = __ldcg(reinterpret_cast<const uint2*>(hr + 4 * (st + 256 * q) + g * 2048));
      float* a = v + q * 8 + g * 4;
      a[0] = bf16_lo(hw.x);
      a[1] = bf16_hi(hw.x);
      a[2] = bf16_lo(hw.y);
      a[3] = bf16_hi(hw.y);
#pragma unroll
      for (int k = 0; k < 4; ++k) ssq[q] = fmaf(a[k], a[k], ssq[q]);
    }
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    const float s = warp_sum(ssq[q]);
    if (lane == 0) sred[wq + 8 * q] = s;  // warp (st + 256 q) / 32 of the 512
  }
  named_bar_sync(2, kStepThreads);
  if (wq == 0) {
    float x = lane < 16 ? sred[lane] : 0.f;
    x = warp_sum(x);
    if (lane == 0) sred[16] = x;
  }
  named_bar_sync(2, kStepThreads);
  const float denom = sqrtf(sred[16] / (float)kHFused + eps);
  __nv_bfloat16* xr = xn + (long)r * kHFused;
#pragma unroll
  for (int q = 0; q < 2; ++q)
#pragma unroll
    for (int g = 0; g < 2; ++g) {
      const int i = 4 * (st + 256 * q) + g * 2048;
      const float* a = v + q * 8 + g * 4;
      const __nv_bfloat162 b0 = __floats2bfloat162_rn((a[0] / denom) * w[i], (a[1] / denom) * w[i + 1]);
      const __nv_bfloat162 b1 = __floats2bfloat162_rn((a[2] / denom) * w[i + 2], (a[3] / denom) * w[i + 3]);
      *reinterpret_cast<uint2*>(xr + i) =
          make_uint2(*reinterpret_cast<const uint32_t*>(&b0), *reinterpret_cast<const uint32_t*>(&b1));
    }
  named_bar_sync(2, kStepThreads);  // sred is reused by the next row
}

// L2 prefetch of one granule's bytes (bulk, no shared-memory destination).
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(reinterpret_cast<uint64_t>(p)),
               "r"(bytes)
               : "memory");
}

// Walks the weight granules of this CTA in load order (phases 0 .. nphase-1, then the
// next layer's O projection) for the L2 prefetcher.
struct WCursor {
  int ph;
  long it, end;
  int j, a;  // tile within the unit, matrix within the tile
};

__device__ __forceinline__ const FPhase& cursor_phase(const FusedParams& p, int ph) {
  return ph < p.nphase ? p.ph[ph] : p.pf_next;
}

__device__ __forceinline__ void cursor_start(const FusedParams& p, WCursor& c, int ph, int cta) {
  c.ph = ph;
  c.j = c.a = 0;
  if (ph > p.nphase || (ph == p.nphase && p.pf_next.w == nullptr)) {
    c.it = c.end = 0;
    return;
  }
  const FPhase& f = cursor_phase(p, ph);
  c.it = range_start(cta, f.iters, p.grid);
  c.end = range_start(cta + 1, f.iters, p.grid);
}

// Prefetch the granule under the cursor and advance; false when nothing is left.
__device__ __forceinline__ bool cursor_prefetch(const FusedParams& p, WCursor& c, int cta) {
  while (c.it >= c.end) {
    if (c.ph >= p.nphase) return false;
    cursor_start(p, c, c.ph + 1, cta);
    if (c.it >= c.end && c.ph >= p.nphase) return false;
  }
  const FPhase& f = cursor_phase(p, c.ph);
  const int u = (int)(c.it / f.kb_total), kb = (int)(c.it % f.kb_total) * f.ks;
  const long blk = ((long)(u * f.nb + c.j) * f.kb64 + kb) * kKBlk;
  prefetch_l2((c.a ? f.w2 : f.w) + blk, (uint32_t)(f.ks * kKBlk));
  if (++c.a == f.na) {
    c.a = 0;
    if (++c.j == unit_tiles(f, u)) {
      c.j = 0;
      ++c.it;
    }
  }
  return true;
}

__global__ void __launch_bounds__(kThreadsF, 1)
layer_tail_kernel(const __grid_constant__ CUtensorMap x0, const __grid_constant__ CUtensorMap x1,
                  const __grid_constant__ CUtensorMap x2, const __grid_constant__ CUtensorMap x3,
                  const __grid_constant__ FusedParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  // layout: weight granules | activation stages | barriers (<= 1 KB) | transpose buffers
  uint8_t* gran = smem;
  uint8_t* xst = gran + kNGran * kGranBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(xst + kXStages * kXStageBytes);
  uint64_t* wfull = bars;                // [4]
  uint64_t* wempty = wfull + kNGran;     // [4]
  uint64_t* xfull = wempty + kNGran;     // [3]
  uint64_t* xempty = xfull + kXStages;   // [3]
  uint64_t* acc_full = xempty + kXStages;  // [2]
  uint64_t* acc_empty = acc_full + 2;      // [2]
  uint64_t* sfull = acc_empty + 2;         // [3] consumer-step copies
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sfull + kXStages);
  float* sred = reinterpret_cast<float*>(tmem_slot + 4);  // [17] norm reductions
  uint8_t* cnt_tab = reinterpret_cast<uint8_t*>(bars) + 1024;  // [4][kMaxTilesF]
  float* tbuf = reinterpret_cast<float*>(cnt_tab + 4 * kMaxTilesF);

  pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cta = blockIdx.x;
  if (threadIdx.x == 0) {
    for (int g = 0; g < kNGran; ++g) {
      mbar_init(wfull + g, 1);
      mbar_init(wempty + g, 1);
    }
    for (int s = 0; s < kXStages; ++s) {
      mbar_init(xfull + s, 1);
      mbar_init(xempty + s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(acc_full + b, 1);
      mbar_init(acc_empty + b, 1);
    }
    for (int s2 = 0; s2 < kXStages; ++s2) mbar_init(sfull + s2, 1);
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 2 * kAccStride);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- weight producer ----------------
      // Weights do not depend on any earlier kernel or phase: no dependency wait here.
      const uint64_t pol = policy_evict_first();
      uint32_t epar = 0, fpar = 0, armed = 0;  // per-granule phase bits
      int gi = 0;
      bool ok = true;
      // L2 prefetcher: keeps up to pf_ahead granules requested beyond the ones loaded, so
      // HBM keeps streaming while the pipeline waits at a phase boundary, and on into the
      // next layer's O projection while the attention kernel runs
      WCursor pc;
      cursor_start(p, pc, 0, cta);
      long loaded = 0, fetched = 0;
      bool more = p.pf_ahead > 0;
      for (int ph = 0; ph < p.nphase && ok; ++ph) {
        const FPhase& f = p.ph[ph];
        const long beg = range_start(cta, f.iters, p.grid), end = range_start(cta + 1, f.iters, p.grid);
        const uint32_t wbytes = (uint32_t)(f.ks * kKBlk);
        for (long it = beg; it < end; ++it) {
          const int u = (int)(it / f.kb_total), kb = (int)(it % f.kb_total) * f.ks;
          const int nv = unit_tiles(f, u);
          const int ng = nv * f.na;
          while (more && fetched < loaded + ng + p.pf_ahead) {
            more = cursor_prefetch(p, pc, cta);
            fetched += more ? 1 : 0;
          }
          loaded += ng;
          for (int m = 0; m < ng && ok; ++m) {
            const int g = (gi + m) & 3;
            ok = mbar_wait(wempty + g, ((epar >> g) & 1u) ^ 1u, p.err, kErrFuEmptyW);
            epar ^= 1u << g;
          }
          if (!ok) break;
          mbar_arrive_expect_tx(wfull + gi, (uint32_t)ng * wbytes);
          for (int j = 0; j < nv; ++j) {
            const long blk = ((long)(u * f.nb + j) * f.kb64 + kb) * kKBlk;
            for (int a = 0; a < f.na; ++a) {
              const int g = (gi + j * f.na + a) & 3;
              bulk_load_hint(gran + g * kGranBytes, (a ? f.w2 : f.w) + blk, wbytes, wfull + gi, pol);
            }
          }
          armed |= 1u << gi;
          fpar ^= 1u << gi;
          gi = (gi + ng) & 3;
        }
      }
      // the rest of the prefetch window (the next layer's first weights)
      while (more && fetched < loaded + p.pf_ahead) {
        more = cursor_prefetch(p, pc, cta);
        fetched += more ? 1 : 0;
      }
      // drain: the last copies into each granule must land before the CTA may exit
      for (int g = 0; g < kNGran; ++g)
        if (armed & (1u << g)) mbar_wait(wfull + g, ((fpar >> g) & 1u) ^ 1u, p.err, kErrFuDrainW);
    }
  } else if (warp == 6) {
    if (lane == 0) {
      // ---------------- activation producer ----------------
      long xi = 0;
      for (int ph = 0; ph < p.nphase; ++ph) {
        const FPhase& f = p.ph[ph];
        if (ph == 0) {
          pdl_wait();  // the attention output of the previous kernel
        } else {
          // every CTA has written its share of this phase's input: the RMSNorm rows
          // (gate/up, QKV) or the SwiGLU output (down).  A failed wait is recorded; the
          // pipeline still drains.
          const int k = ph == 2 ? 5 : 4 * (ph - 1) + 2;
          counter_wait(p.sync + k, (unsigned)p.grid, p.err, kErrFuGrid + k);
        }
        fence_proxy_async_global();
        const CUtensorMap* xm = ph == 0 ? &x0 : (ph == 1 ? &x1 : (ph == 2 ? &x2 : &x3));
        tma_prefetch_desc(xm);
        const long beg = range_start(cta, f.iters, p.grid), end = range_start(cta + 1, f.iters, p.grid);
        const uint32_t xbytes = (uint32_t)(f.ks * p.tok_tile * kBK * 2);
        for (long it = beg; it < end; ++it, ++xi) {
          const int s = (int)(xi % kXStages);
          if (!mbar_wait(xempty + s, ((uint32_t)(xi / kXStages) & 1u) ^ 1u, p.err, kErrFuEmptyX)) {
            ph = p.nphase;
            break;
          }
          mbar_arrive_expect_tx(xfull + s, xbytes);
          const int kb = (int)(it % f.kb_total) * f.ks;
          for (int jb = 0; jb < f.ks; ++jb)
            tma_load_2d(xst + s * kXStageBytes + jb * p.tok_tile * kBK * 2, xm, xfull + s,
                        (kb + jb) * kBK, 0);
        }
      }
      for (long s = 0; s < kXStages && s < xi; ++s) {
        const long last = s + ((xi - 1 - s) / kXStages) * kXStages;
        mbar_wait(xfull + s, (uint32_t)(last / kXStages) & 1u, p.err, kErrFuDrainX);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      const uint32_t idesc = idesc_bf16_f32(kTileN, p.tok_tile);
      uint32_t fpar = 0;
      int gi = 0, nseg = 0;
      long xi = 0;
      bool ok = true;
      for (int ph = 0; ph < p.nphase && ok; ++ph) {
        const FPhase& f = p.ph[ph];
        const long beg = range_start(cta, f.iters, p.grid), end = range_start(cta + 1, f.iters, p.grid);
        for (long it = beg; it < end && ok;) {
          const Seg sg = segment_at(it, end, f.kb_total);
          const int ng = unit_tiles(f, sg.unit) * f.na;
          const int buf = nseg & 1;
          const uint32_t use = (uint32_t)(nseg >> 1);
          if (!mbar_wait(acc_empty + buf, (use & 1u) ^ 1u, p.err, kErrFuAccEmpty)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t acc = tmem + (uint32_t)(buf * kAccStride);
          for (long j = sg.it0; j < sg.it1; ++j, ++xi) {
            if (!mbar_wait(wfull + gi, (fpar >> gi) & 1u, p.err, kErrFuFullW)) {
              ok = false;
              break;
            }
            fpar ^= 1u << gi;
            const int xs = (int)(xi % kXStages);
            if (!mbar_wait(xfull + xs, (uint32_t)(xi / kXStages) & 1u, p.err, kErrFuFullX)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t sx = smem_u32(xst + xs * kXStageBytes);
            const uint32_t ga0 = smem_u32(gran + gi * kGranBytes);
            const uint32_t ga1 = smem_u32(gran + ((gi + 1) & 3) * kGranBytes);
            const bool two = ng == 2;
#pragma unroll
            for (int jb = 0; jb < 2; ++jb) {
              if (jb >= f.ks) break;
#pragma unroll
              for (int kk = 0; kk < kBK / 16; ++kk) {
                const bool accum = (j != sg.it0) || (jb != 0) || (kk != 0);
                const uint64_t bd = smem_desc_sw128(sx + jb * p.tok_tile * kBK * 2 + kk * 32);
                tc_mma_f16(acc, smem_desc_sw128(ga0 + jb * kKBlk + kk * 32), bd, idesc, accum);
                if (two)
                  tc_mma_f16(acc + (uint32_t)p.tok_tile, smem_desc_sw128(ga1 + jb * kKBlk + kk * 32),
                             bd, idesc, accum);
              }
            }
            tc_commit(wempty + gi);
            if (two) tc_commit(wempty + ((gi + 1) & 3));
            tc_commit(xempty + xs);
            gi = (gi + ng) & 3;
          }
          tc_commit(acc_full + buf);
          it = sg.it1;
          ++nseg;
        }
      }
    }
  } else {
    // ------- epilogue (warps 2..5) and consumer steps (warps 2..5 and 7..10) -------
    pdl_wait();  // h, the slots and the KV cache may still be read by earlier kernels
    const bool epi = warp <= 5;
    const int q = warp & 3;
    const int et = threadIdx.x - 64;                         // epilogue thread 0..127
    const int st = epi ? et : 128 + (threadIdx.x - 7 * 32);  // step thread 0..255
    float* tb = tbuf + (warp - 2) * (32 * 33);
    // The split-K partials are read back by every CTA's consumer step microseconds later:
    // they are stored evict-last so that the weights streaming through L2 (evict-first)
    // do not push them out to HBM.  The slot buffer is reused by every phase, so these
    // lines stay in L2 and are overwritten in place.
    const uint64_t pol_keep = policy_evict_last();
    // contributors of every weight tile of every phase (the stream-K owners)
    for (int ph = 0; ph < p.nphase; ++ph) {
      const FPhase& f = p.ph[ph];
      for (int t = st; t < f.n_tiles; t += kStepThreads) {
        const long x0 = (long)(t / f.nb) * f.kb_total;
        cnt_tab[ph * kMaxTilesF + t] = (uint8_t)(owner_cta(x0 + f.kb_total - 1, f.iters, p.grid) -
                                                 owner_cta(x0, f.iters, p.grid) + 1);
      }
    }
    StepCtx sc;
    sc.stage = xst;
    sc.sfull = sfull;
    sc.cnt = cnt_tab;
    sc.sb = 0;
    int nseg = 0;
    for (int ph = 0; ph < p.nphase; ++ph) {
      const FPhase& f = p.ph[ph];
      if (epi) {
        const long beg = range_start(cta, f.iters, p.grid), end = range_start(cta + 1, f.iters, p.grid);
        const long slot_floats = (long)f.na * p.tok_tile * kTileN;
        for (long it = beg; it < end;) {
          const Seg sg = segment_at(it, end, f.kb_total);
          const int buf = nseg & 1;
          const uint32_t use = (uint32_t)(nseg >> 1);
          mbar_wait(acc_full + buf, use & 1u, p.err, kErrFuAccFull);
          tc_fence_after();
          const int nv = unit_tiles(f, sg.unit);
          const int rank = cta - owner_cta((long)sg.unit * f.kb_total, f.iters, p.grid);
          for (int jn = 0; jn < nv; ++jn) {
            const int nt = sg.unit * f.nb + jn;
            float* part = p.slots + ((long)nt * f.maxc + rank) * slot_floats;
            const uint32_t trow = tmem + (uint32_t)(buf * kAccStride + jn * f.na * p.tok_tile) +
                                  ((uint32_t)(q * 32) << 16);
            const int rr = q * 32 + (lane & 3) * 8;
            for (int c = 0; c < p.tok_tile; c += 32) {
              const int w = min(32, p.tok_tile - c);
              // accumulator a of the tile (gate, then up), one 32-token chunk at a time
              for (int a = 0; a < f.na; ++a) {
                float o[4][8];
                epi_transpose(trow + (uint32_t)(a * p.tok_tile + c), w, tb, lane, o);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                  if (i * 8 + (lane >> 2) >= w) continue;
                  const int tk = c + i * 8 + (lane >> 2);
                  float* dst = part + (long)(a * p.tok_tile + tk) * kTileN + rr;
                  st_v4_hint(dst, make_float4(o[i][0], o[i][1], o[i][2], o[i][3]), pol_keep);
                  st_v4_hint(dst + 4, make_float4(o[i][4], o[i][5], o[i][6], o[i][7]), pol_keep);
                }
              }
            }
          }
          tc_fence_before();
          named_bar_sync(1, 128);
          if (et == 0) mbar_arrive(acc_empty + buf);
          it = sg.it1;
          ++nseg;
        }
        // this CTA's partials of phase ph are written (the barrier above ordered them)
        if (et == 0) {
          __threadfence();
          fence_proxy_async_global();  // read back by bulk copies
          counter_arrive(p.sync + 4 * ph);
        }
      }
      // consumer step ph: this CTA's blocks of partial sums, once every CTA's phase-ph
      // partials are written
      if (st == 0) {
        counter_wait(p.sync + 4 * ph, (unsigned)p.grid, p.err, kErrFuGrid + 4 * ph);
        fence_proxy_async_global();  // the partials are read by bulk copies
      }
      named_bar_sync(2, kStepThreads);
      sc.cnt = cnt_tab + ph * kMaxTilesF;
      if (ph == 1)
        step_blocks<kOpSwiglu>(p, ph, sc, st, lane, cta);
      else if (ph == 3)
        step_blocks<kOpRope>(p, ph, sc, st, lane, cta);
      else
        step_blocks<kOpResid>(p, ph, sc, st, lane, cta);
      named_bar_sync(2, kStepThreads);
      if (st == 0 && ph + 1 < p.nphase + (ph == 2 ? 1 : 0)) {
        __threadfence();
        fence_proxy_async_global();
        counter_arrive(p.sync + 4 * ph + 1);
      }
      if (ph == 0 || ph == 2) {
        // RMSNorm of whole rows once every CTA has added its residual blocks
        if (st == 0) counter_wait(p.sync + 4 * ph + 1, (unsigned)p.grid, p.err, kErrFuGrid + 4 * ph + 1);
        named_bar_sync(2, kStepThreads);
        (void)counter_acquire(p.sync + 4 * ph + 1);  // every thread acquires the writers' release
        for (int r = cta; r < p.M; r += p.grid)
          step_row_norm(r, p.h, ph == 0 ? p.ln2 : p.ln_next, p.eps, p.xn, sred, st);
        if (st == 0 && ph + 1 < p.nphase) {
          __threadfence();
          fence_proxy_async_global();  // xn is read by TMA
          counter_arrive(p.sync + 4 * ph + 2);
        }
      }
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 2 * kAccStride);
  }
}

struct PlanSet {
  GemmPlan g[4];
  int n = 0;
};

bool make_plans(int M, int H, int I, int qdim, int qkvdim, bool with_qkv, int num_sms, PlanSet* ps) {
  // one weight tile per stream-K unit: the weight ring does not share activation blocks
  // between tiles, and single-tile units leave the fewest split-K partials to sum
  ps->g[0] = plan_gemm_tc(M, H, qdim, false, num_sms, 1);
  ps->g[1] = plan_gemm_tc(M, I, H, true, num_sms, 1);
  ps->g[2] = plan_gemm_tc(M, H, I, false, num_sms, 1);
  ps->n = 3;
  if (with_qkv) ps->g[ps->n++] = plan_gemm_tc(M, qkvdim, H, false, num_sms, 1);
  for (int k = 0; k < ps->n; ++k) {
    const GemmPlan& g = ps->g[k];
    const int na = k == 1 ? 2 : 1;
    if (g.t_tiles != 1 || g.tok_tile > kMaxTok || g.ks < 1 || g.ks > 2 || g.grid != num_sms ||
        g.nb * na > 2 || g.nb * na * g.tok_tile > kAccStride || g.n_tiles > kMaxTilesF ||
        g.maxc > 255)
      return false;
  }
  return true;
}

}  // namespace

bool fused_tail_supported(int M, int H, int I, int qdim, int qkvdim, int head_dim, int num_sms,
                          long* slot_floats) {
  // Opt-in (WEDLM_FUSED_TAIL=1): measured on B200 at the 8B shape, the stand-alone
  // kernels are faster (185 against 163 committed tok/s).  The fused tail streams each
  // projection's weights at up to 6.9 TB/s, but its four phase boundaries (split-K
  // partials summed by every CTA between grid-wide barriers) cost ~75 us a layer.
  const char* e = getenv("WEDLM_FUSED_TAIL");
  if (!e || atoi(e) == 0) return false;
  if (M < 1 || M > kMaxTok || H != kHFused || head_dim != 128 || I % 64 != 0 ||
      qdim % 64 != 0 || qkvdim % 128 != 0)
    return false;
  PlanSet ps;
  if (!make_plans(M, H, I, qdim, qkvdim, true, num_sms, &ps)) return false;
  long mx = 0;
  for (int k = 0; k < ps.n; ++k) mx = ps.g[k].slot_floats > mx ? ps.g[k].slot_floats : mx;
  if (slot_floats) *slot_floats = mx;
  return true;
}

Status run_fused_tail(const FusedTailArgs& a, int num_sms, cudaStream_t st) {
  const bool with_qkv = a.wqkv_next != nullptr;
  PlanSet ps;
  WEDLM_CHECK_ARG(a.M >= 1 && a.M <= kMaxTok && a.H == kHFused && a.rope.head_dim == 128,
                  "fused layer tail: unsupported shape");
  WEDLM_CHECK_ARG(make_plans(a.M, a.H, a.I, a.qdim, a.qkvdim, with_qkv, num_sms, &ps),
                  "fused layer tail: unsupported GEMM plan");
  FusedParams p;
  memset(&p, 0, sizeof(p));
  const void* w1[4] = {a.wo, a.wgate, a.wdown, a.wqkv_next};
  const void* w2[4] = {a.wo, a.wup, a.wdown, a.wqkv_next};
  for (int k = 0; k < ps.n; ++k) {
    const GemmPlan& g = ps.g[k];
    WEDLM_CHECK_ARG(g.slot_floats <= a.slot_floats, "fused layer tail: partial slots too small");
    FPhase& f = p.ph[k];
    f.w = reinterpret_cast<const uint8_t*>(w1[k]);
    f.w2 = reinterpret_cast<const uint8_t*>(w2[k]);
    WEDLM_CHECK_ARG(((uintptr_t)f.w % 16) == 0 && ((uintptr_t)f.w2 % 16) == 0,
                    "packed weights must be 16-byte aligned");
    f.n_tiles = g.n_tiles;
    f.kb64 = g.kb64;
    f.ks = g.ks;
    f.nb = g.nb;
    f.na = k == 1 ? 2 : 1;
    f.kb_total = g.kb_total;
    f.maxc = g.maxc;
    f.iters = (long)((g.n_tiles + g.nb - 1) / g.nb) * g.kb_total;
    p.ps[k] = partial_set(g, a.slots, k == 1);
  }
  p.nphase = ps.n;
  p.grid = num_sms;
  p.M = a.M;
  p.tok_tile = ps.g[0].tok_tile;
  for (int k = 1; k < ps.n; ++k)
    WEDLM_CHECK_ARG(ps.g[k].tok_tile == p.tok_tile, "fused layer tail: token tiles differ");
  p.H = a.H;
  p.I = a.I;
  p.eps = a.eps;
  p.slots = a.slots;
  p.err = a.err;
  p.sync = a.sync;
  p.h = reinterpret_cast<__nv_bfloat16*>(a.h);
  p.xn = reinterpret_cast<__nv_bfloat16*>(a.xn);
  p.act = reinterpret_cast<__nv_bfloat16*>(a.act);
  p.ln2 = a.ln2;
  p.ln_next = a.ln_next;
  p.rope = a.rope;
  p.rope.qkv_partials = nullptr;
  for (int k = 0; k < ps.n; ++k) {
    const int na = k == 1 ? 2 : 1;
    int tb = kXStageBytes / (ps.g[k].maxc * na * 512);
    p.tb[k] = tb > 8 ? 8 : tb;
    WEDLM_CHECK_ARG(p.tb[k] >= 1, "fused layer tail: too many split-K contributors per tile");
  }
  p.pf_ahead = kPfDefault;
  if (const char* e = getenv("WEDLM_FUSED_PF")) p.pf_ahead = atoi(e) < 0 ? 0 : atoi(e);
  if (a.wo_next) {
    p.pf_next = p.ph[0];
    p.pf_next.w = p.pf_next.w2 = reinterpret_cast<const uint8_t*>(a.wo_next);
  }
  CUtensorMap m0, m1, m2;
  WEDLM_TRY(cached_tmap(&m0, a.attn, a.M, a.qdim, a.qdim, p.tok_tile));
  WEDLM_TRY(cached_tmap(&m1, a.xn, a.M, a.H, a.H, p.tok_tile));
  WEDLM_TRY(cached_tmap(&m2, a.act, a.M, a.I, a.I, p.tok_tile));

  int dev = 0;
  WEDLM_CUDA_TRY(cudaGetDevice(&dev));
  static unsigned attr_set = 0;  // one bit per device
  if (dev < 32 && !(attr_set & (1u << dev))) {
    WEDLM_CUDA_TRY(cudaFuncSetAttribute(layer_tail_kernel,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemF));
    attr_set |= 1u << dev;
  }
  // Cooperative launch: the CTAs wait on one another through the dependency counters, so
  // all of them must be resident at once (one per SM).
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)num_sms);
  cfg.blockDim = dim3(kThreadsF);
  cfg.dynamicSmemBytes = kSmemF;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  static unsigned no_pdl = 0;  // devices where the driver refused the two attributes together
  cfg.numAttrs = (dev < 32 && (no_pdl & (1u << dev))) ? 1 : 2;
  cudaError_t e = cudaLaunchKernelEx(&cfg, layer_tail_kernel, m0, m1, m2, m1, p);
  if (e != cudaSuccess && cfg.numAttrs == 2) {
    (void)cudaGetLastError();  // a refused launch configuration is not sticky
    if (dev < 32) no_pdl |= 1u << dev;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, layer_tail_kernel, m0, m1, m2, m1, p);
  }
  if (e != cudaSuccess)
    return Status::err(WEDLM_ERR_CUDA, std::string("fused layer tail launch: ") + cudaGetErrorString(e));
  return Status::ok();
}

}  // namespace wedlm
