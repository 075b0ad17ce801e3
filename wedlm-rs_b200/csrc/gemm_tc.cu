// tcgen05 / TMEM GEMM for the projections of the decode step (bf16 in, f32 accumulate):
//   Y[tok, n] = sum_k X[tok, k] * W[n, k]      (Linear::forward, x W^T, no bias)
// Replaces the candle matmuls behind q/k/v/o (src/model/attention.rs:145-147,229),
// gate/up/down (src/model/mlp.rs:40-44) and the LM head (src/model/causal_lm.rs:77).
//
// Swap-AB: the MMA's M = 128 covers weight rows and its N covers the token rows of the
// step (96 for one block-96 window), so at batch 1 the tensor core's M side is filled
// with weights, which are what streams from HBM.  The fused gate/up projection keeps
// two accumulators side by side in TMEM and applies SwiGLU in the epilogue.
//
// Stream-K persistent schedule: the iteration space (tile, 64-wide k-block) is cut into
// one contiguous range per SM, so every SM streams the same number of weight bytes
// whatever the tile count (no wave quantisation).  A tile covered by one CTA is written
// directly by its epilogue; each CTA publishes the f32 partials of the (at most two)
// tiles it shares with neighbours, and a small follow-up kernel sums every shared tile
// in CTA order (deterministic) and applies the epilogue.
// Warp roles:
//   warp 0        TMA producer: weight / activation tiles (128-byte swizzle) into a ring
//                 of shared-memory stages, completion on "full" mbarriers;
//   warp 1        TMEM allocator and MMA issuer (one thread): 4 MMAs of K = 16 per stage,
//                 tcgen05.commit frees the stage; double-buffered accumulators;
//   warps 2..5    epilogue: tcgen05.ld (one weight row per thread), residual / SwiGLU,
//                 bf16 or f32 stores, or partial publication for shared tiles.
#include <cudaTypedefs.h>

#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>

#include "gemm.h"
#include "sm100.cuh"
#include "tc_epilogue.cuh"

namespace wedlm {

namespace {

using namespace sm100;

constexpr int kThreadsTC = 192;  // 6 warps: TMA producer, MMA issuer, 4 epilogue
constexpr int kBK = 64;              // K elements per stage (128 bytes of bf16)
constexpr int kTileN = 128;          // weight rows per tile (MMA M)
constexpr int kATileBytes = kTileN * kBK * 2;

struct TcParams {
  int N, M, K;
  int n_tiles, t_tiles, kb_total;  // kb_total: k-steps per unit (each ks 64-wide k-blocks)
  int ks, kb64;                     // k-blocks per step, 64-wide k-blocks per row
  int nb;              // weight tiles per unit: they share every activation k-block
  long iters;          // units * kb_total; unit u = (weight group u / t_tiles, token tile u % t_tiles)
  int grid;
  int tok_tile;
  int epi, dual;
  int stages, nbuf;
  uint32_t stage_bytes, tmem_cols, acc_cols;  // stage: ks k-blocks of weights + activations
  void* out;
  int ldo;
  const __nv_bfloat16* resid;
  int ldr;
  float* ws;           // [grid][2 slots][nb][na][tok_tile][128 weight rows]
  int* err;
  const uint8_t* wp;   // packed weight tiles (when packed)
  const uint8_t* wp2;
  int packed;
  float* slots;        // slot mode: [tiles][maxc][na][tok_tile][128]
  int slot_mode, maxc;
  int poll, nohint;   // tuning: spin on test_wait; weight copies evict-last, not evict-first
  int vec_ok;          // out / resid rows 16-byte aligned
};

__device__ __forceinline__ long range_start(long c, long iters, int grid) {
  return c * iters / grid;
}
// the CTA whose range holds iteration x: max c with floor(c*I/G) <= x == ceil((x+1)G/I) - 1
__device__ __forceinline__ int owner_cta(long x, long iters, int grid) {
  long c = ((x + 1) * grid + iters - 1) / iters - 1;
  return (int)(c < 0 ? 0 : (c >= grid ? grid - 1 : c));
}

__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__device__ __forceinline__ void epilogue_store(const TcParams& p, int tok, int n, float a, float a2) {
  switch (p.epi) {
    case EPI_STORE_F32:
      reinterpret_cast<float*>(p.out)[(long)tok * p.ldo + n] = a;
      break;
    case EPI_RESID_BF16: {
      // reference: residual + bf16(projection), rounded to bf16 (layer.rs:72,78)
      float r = __bfloat162float(p.resid[(long)tok * p.ldr + n]);
      reinterpret_cast<__nv_bfloat16*>(p.out)[(long)tok * p.ldo + n] =
          __float2bfloat16_rn(r + bf16r(a));
      break;
    }
    case EPI_SWIGLU_BF16: {
      // reference: silu(bf16 gate) * bf16 up, each op rounded to bf16 (mlp.rs:40-43)
      float g = bf16r(a), u = bf16r(a2);
      float s = bf16r(g / (1.f + __expf(-g)));
      reinterpret_cast<__nv_bfloat16*>(p.out)[(long)tok * p.ldo + n] = __float2bfloat16_rn(s * u);
      break;
    }
    default:
      reinterpret_cast<__nv_bfloat16*>(p.out)[(long)tok * p.ldo + n] = __float2bfloat16_rn(a);
  }
}

// Epilogue for NV consecutive weight rows n .. n+NV-1 of one token (NV = 8 or 16):
// 16-byte vector stores when the row span is in bounds and aligned.
template <int NV>
__device__ __forceinline__ void epilogue_store_vec(const TcParams& p, int tok, int n,
                                                   const float* a, const float* a2) {
  if (!p.vec_ok || n + NV > p.N) {
#pragma unroll
    for (int k = 0; k < NV; ++k)
      if (n + k < p.N) epilogue_store(p, tok, n + k, a[k], p.dual ? a2[k] : 0.f);
    return;
  }
  if (p.epi == EPI_STORE_F32) {
    float* dst = reinterpret_cast<float*>(p.out) + (long)tok * p.ldo + n;
#pragma unroll
    for (int k = 0; k < NV; k += 4)
      *reinterpret_cast<float4*>(dst + k) = make_float4(a[k], a[k + 1], a[k + 2], a[k + 3]);
    return;
  }
  float y[NV];
  if (p.epi == EPI_RESID_BF16) {
    const __nv_bfloat16* rs = p.resid + (long)tok * p.ldr + n;
#pragma unroll
    for (int k = 0; k < NV; k += 8) {
      const uint4 rv = *reinterpret_cast<const uint4*>(rs + k);
      const uint32_t w[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        y[k + 2 * u] = bf16_lo(w[u]) + bf16r(a[k + 2 * u]);
        y[k + 2 * u + 1] = bf16_hi(w[u]) + bf16r(a[k + 2 * u + 1]);
      }
    }
  } else if (p.epi == EPI_SWIGLU_BF16) {
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const float g = bf16r(a[k]), u = bf16r(a2[k]);
      y[k] = bf16r(g / (1.f + __expf(-g))) * u;
    }
  } else {
#pragma unroll
    for (int k = 0; k < NV; ++k) y[k] = a[k];
  }
  __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.out) + (long)tok * p.ldo + n;
#pragma unroll
  for (int k = 0; k < NV; k += 8) {
    uint32_t w[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const __nv_bfloat162 h2 = __floats2bfloat162_rn(y[k + 2 * u], y[k + 2 * u + 1]);
      w[u] = *reinterpret_cast<const uint32_t*>(&h2);
    }
    *reinterpret_cast<uint4*>(dst + k) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

struct Seg {
  long it0, it1;  // global iteration range of this segment
  int unit;
  bool full;      // covers the whole unit
};

__device__ __forceinline__ Seg segment_at(long it, long end, int kb_total) {
  Seg s;
  s.unit = (int)(it / kb_total);
  const long unit_end = (long)(s.unit + 1) * kb_total;
  s.it0 = it;
  s.it1 = end < unit_end ? end : unit_end;
  s.full = (it == (long)s.unit * kb_total) && (s.it1 == unit_end);
  return s;
}

// weight tiles present in unit u (the last group may hold fewer than nb)
__device__ __forceinline__ int unit_tiles(const TcParams& p, int u) {
  const int left = p.n_tiles - (u / p.t_tiles) * p.nb;
  return left < p.nb ? left : p.nb;
}

__global__ void __launch_bounds__(kThreadsTC, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmW2,
               const __grid_constant__ CUtensorMap tmX, const TcParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  // layout: stage ring | barriers (<= 1 KB) | epilogue transpose buffers
  uint8_t* tail = smem + p.stages * p.stage_bytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(tail);
  uint64_t* empty = full + p.stages;
  uint64_t* acc_full = empty + p.stages;   // [2]
  uint64_t* acc_empty = acc_full + 2;      // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  // per-epilogue-warp transpose buffers: [32 tokens][33]
  float* tbuf = reinterpret_cast<float*>(tail + 1024);

  pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cta = blockIdx.x;
  const long beg = range_start(cta, p.iters, p.grid);
  const long end = range_start(cta + 1, p.iters, p.grid);

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(acc_full + b, 1);
      mbar_init(acc_empty + b, 1);
    }
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, p.tmem_cols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer: weights (bulk) and activations ----------------
      tma_prefetch_desc(&tmX);
      if (!p.packed) {
        tma_prefetch_desc(&tmW);
        if (p.dual) tma_prefetch_desc(&tmW2);
      }
      const uint64_t pol_w = p.nohint ? policy_evict_last() : policy_evict_first();
      const int na = p.dual ? 2 : 1;
      const uint32_t wbytes = (uint32_t)(p.ks * kATileBytes);
      const uint32_t a_bytes = wbytes * na * p.nb;
      const uint32_t x_bytes = (uint32_t)(p.ks * p.tok_tile * kBK * 2);
      // weights of step `it` into ring slot s (arms the slot's full barrier for the stage);
      // stage layout: [tile j][matrix a][ks k-blocks of 16 KB] ... then the activations
      auto load_w = [&](long it, int s) {
        const int u = (int)(it / p.kb_total), kb = (int)(it % p.kb_total) * p.ks;
        const int nv = unit_tiles(p, u);
        uint8_t* st = smem + s * p.stage_bytes;
        mbar_arrive_expect_tx(full + s, (uint32_t)(nv * na) * wbytes + x_bytes);
        for (int j = 0; j < nv; ++j) {
          const int nt = (u / p.t_tiles) * p.nb + j;
          uint8_t* dw = st + (uint32_t)(j * na) * wbytes;
          if (p.packed) {
            // the ks k-blocks of this step are contiguous in the packed layout
            const long blk = ((long)nt * p.kb64 + kb) * kATileBytes;
            bulk_load_hint(dw, p.wp + blk, wbytes, full + s, pol_w);
            if (p.dual) bulk_load_hint(dw + wbytes, p.wp2 + blk, wbytes, full + s, pol_w);
          } else {
            for (int jb = 0; jb < p.ks; ++jb) {
              tma_load_2d_hint(dw + jb * kATileBytes, &tmW, full + s, (kb + jb) * kBK, nt * kTileN, pol_w);
              if (p.dual)
                tma_load_2d_hint(dw + wbytes + jb * kATileBytes, &tmW2, full + s, (kb + jb) * kBK,
                                 nt * kTileN, pol_w);
            }
          }
        }
      };
      auto load_x = [&](long it, int s) {
        const int u = (int)(it / p.kb_total), kb = (int)(it % p.kb_total) * p.ks;
        const int t0 = (u % p.t_tiles) * p.tok_tile;
        uint8_t* st = smem + s * p.stage_bytes + a_bytes;
        for (int j = 0; j < p.ks; ++j)
          tma_load_2d(st + j * p.tok_tile * kBK * 2, &tmX, full + s, (kb + j) * kBK, t0);
      };
      // The weights do not depend on the previous kernel: fill every ring slot with them
      // while that kernel finishes, then wait for it before the first activation load.
      const long pre = (end - beg) < p.stages ? (end - beg) : p.stages;
      for (long i = 0; i < pre; ++i) load_w(beg + i, (int)i);
      pdl_wait();
      for (long i = 0; i < pre; ++i) load_x(beg + i, (int)i);
      long issued = pre;
      for (long it = beg + pre; it < end; ++it) {
        const long i = it - beg;
        const int s = (int)(i % p.stages);
        const uint32_t ph = (uint32_t)(i / p.stages) & 1u;
        if (!(p.poll ? mbar_spin(empty + s, ph ^ 1u, p.err, kErrWaitEmpty)
                     : mbar_wait(empty + s, ph ^ 1u, p.err, kErrWaitEmpty)))
          break;
        issued = i + 1;
        load_w(it, s);
        load_x(it, s);
      }
      // drain: wait for the last load issued to every stage before the CTA may exit
      for (long s = 0; s < p.stages && s < issued; ++s) {
        const long last = s + ((issued - 1 - s) / p.stages) * p.stages;
        mbar_wait(full + s, (uint32_t)(last / p.stages) & 1u, p.err, kErrWaitDrain);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      const uint32_t idesc = idesc_bf16_f32(kTileN, p.tok_tile);
      const int na = p.dual ? 2 : 1;
      const uint32_t wbytes = (uint32_t)(p.ks * kATileBytes);
      const uint32_t nmat = (uint32_t)(p.nb * na);
      bool ok = true;
      int nseg = 0;
      for (long it = beg; it < end && ok;) {
        const Seg sg = segment_at(it, end, p.kb_total);
        const bool two = unit_tiles(p, sg.unit) * na == 2;
        const int buf = nseg % p.nbuf;
        const uint32_t use = (uint32_t)(nseg / p.nbuf);
        // wait until the epilogue has drained this accumulator buffer
        if (!mbar_wait(acc_empty + buf, (use & 1u) ^ 1u, p.err, kErrWaitAccumEmpty)) break;
        tc_fence_after();
        const uint32_t acc = tmem + (uint32_t)(buf * p.acc_cols);
        for (long j = sg.it0; j < sg.it1; ++j) {
          const long i = j - beg;
          const int s = (int)(i % p.stages);
          if (!(p.poll ? mbar_spin(full + s, (uint32_t)(i / p.stages) & 1u, p.err, kErrWaitFull)
                       : mbar_wait(full + s, (uint32_t)(i / p.stages) & 1u, p.err, kErrWaitFull))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + s * p.stage_bytes);
          const uint32_t sb = sa + wbytes * nmat;
          // one or two weight matrices per stage (two tiles, or gate and up): matrix m at
          // sa + m * wbytes, accumulator columns m * tok_tile; both share the activations
          for (int jb = 0; jb < p.ks; ++jb) {
            const uint32_t ja = sa + jb * kATileBytes, jx = sb + jb * p.tok_tile * kBK * 2;
#pragma unroll
            for (int kk = 0; kk < kBK / 16; ++kk) {
              const bool accum = (j != sg.it0) || (jb != 0) || (kk != 0);
              const uint64_t bd = smem_desc_sw128(jx + kk * 32);
              tc_mma_f16(acc, smem_desc_sw128(ja + kk * 32), bd, idesc, accum);
              if (two)
                tc_mma_f16(acc + (uint32_t)p.tok_tile, smem_desc_sw128(ja + wbytes + kk * 32), bd,
                           idesc, accum);
            }
          }
          tc_commit(empty + s);
          if (!ok) break;
        }
        tc_commit(acc_full + buf);
        it = sg.it1;
        ++nseg;
      }
    }
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    pdl_wait();  // outputs may still be read by the previous kernel
    const int q = warp & 3;
    const int na = p.dual ? 2 : 1;
    const long slot_floats = (long)na * p.tok_tile * kTileN;
    int nseg = 0;
    for (long it = beg; it < end;) {
      const Seg sg = segment_at(it, end, p.kb_total);
      const int buf = nseg % p.nbuf;
      const uint32_t use = (uint32_t)(nseg / p.nbuf);
      const bool ok = mbar_wait(acc_full + buf, use & 1u, p.err, kErrWaitAccum);
      tc_fence_after();
      const int nv = unit_tiles(p, sg.unit);
      const int t0 = (sg.unit % p.t_tiles) * p.tok_tile;
      const int tok_end = min(p.tok_tile, p.M - t0);
      for (int jn = 0; jn < nv; ++jn) {
        const int nt = (sg.unit / p.t_tiles) * p.nb + jn;
        const int n0 = nt * kTileN;
        const uint32_t trow = tmem + (uint32_t)(buf * p.acc_cols + jn * na * p.tok_tile) +
                              ((uint32_t)(q * 32) << 16);
        // shared unit: publish this CTA's partial of weight tile nt, layout
        // [na][tok_tile][128 weight rows] f32.  Slot mode: slot (tile, rank of this CTA among
        // the unit's contributors), summed by the consumer kernel.  Direct mode: the CTA's
        // first-segment or last-segment slot, summed by the reduce kernel.
        float* part;
        if (p.slot_mode) {
          const int rank = cta - owner_cta((long)sg.unit * p.kb_total, p.iters, p.grid);
          const long tile = (long)nt * p.t_tiles + (sg.unit % p.t_tiles);
          part = p.slots + (tile * p.maxc + rank) * slot_floats;
        } else {
          part = p.ws + (((long)cta * 2 + ((sg.it0 == beg) ? 0 : 1)) * p.nb + jn) * slot_floats;
        }
        if (!(sg.full && !p.slot_mode)) {
          // a partial: straight from TMEM, lane = weight row q * 32 + lane; for each token
          // the warp's 32 lanes write 32 consecutive floats (one 128-byte run)
          float* prow = part + q * 32 + lane;
          for (int m = 0; m < na; ++m) {
            float* pm = prow + (long)m * p.tok_tile * kTileN;
            const uint32_t tm = trow + (uint32_t)(m * p.tok_tile);
            for (int c = 0; c < p.tok_tile; c += 32) {
              float v[32];
              if (p.tok_tile - c >= 32) {
                tmem_ld32(tm + (uint32_t)c, v);
#pragma unroll
                for (int j = 0; j < 32; ++j) pm[(long)(c + j) * kTileN] = v[j];
              } else {
                float h[16];
                tmem_ld16(tm + (uint32_t)c, h);
#pragma unroll
                for (int j = 0; j < 16; ++j) pm[(long)(c + j) * kTileN] = h[j];
              }
            }
          }
          continue;
        }
        float* tb = tbuf + (warp - 2) * (32 * 33);
        const int rr = q * 32 + (lane & 3) * 8;  // this lane's first weight row in the tile
        for (int c = 0; c < p.tok_tile; c += 32) {
          const int w = min(32, p.tok_tile - c);  // tokens in this chunk (32, or 16 at the end)
          float o[4][8], o2[4][8];
          epi_transpose(trow + (uint32_t)c, w, tb, lane, o);
          if (p.dual) epi_transpose(trow + (uint32_t)(p.tok_tile + c), w, tb, lane, o2);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int tk = c + i * 8 + (lane >> 2);  // token within the tile
            if (i * 8 + (lane >> 2) >= w) continue;
            // a whole unit of direct mode: the final epilogue, 8 weight rows per lane
            if (ok && tk < tok_end) epilogue_store_vec<8>(p, t0 + tk, n0 + rr, o[i], o2[i]);
          }
        }
      }
      tc_fence_before();
      named_bar_sync(1, 128);
      if (warp == 2 && lane == 0) mbar_arrive(acc_empty + buf);
      it = sg.it1;
      ++nseg;
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, p.tmem_cols);
  }
}

// Sum the partials of every tile shared by several CTAs, in CTA order, and apply the
// epilogue.  CTA c (1 <= c < grid) owns the tile holding range boundary start(c) when
// that boundary is not a tile edge and no smaller boundary falls inside the same tile.
__global__ void __launch_bounds__(256) gemm_reduce_kernel(const TcParams p) {
  pdl_trigger();
  pdl_wait();
  const int c = blockIdx.x + 1;
  const long x = range_start(c, p.iters, p.grid);
  if (x % p.kb_total == 0) return;
  const int unit = (int)(x / p.kb_total);
  const long x0 = (long)unit * p.kb_total, x1 = x0 + p.kb_total;
  if (c > 1) {
    const long xp = range_start(c - 1, p.iters, p.grid);
    if (xp > x0) return;  // an earlier boundary lies inside this unit
  }
  const int cf = owner_cta(x0, p.iters, p.grid);
  const int cl = owner_cta(x1 - 1, p.iters, p.grid);
  const int na = p.dual ? 2 : 1;
  const long slot_floats = (long)na * p.tok_tile * kTileN;
  const int nv = unit_tiles(p, unit);
  const int t0 = (unit % p.t_tiles) * p.tok_tile;
  const int tok_end = min(p.tok_tile, p.M - t0);
  const int per_tile = tok_end * (kTileN / 8);
  for (int e = threadIdx.x; e < nv * per_tile; e += blockDim.x) {
    const int j = e / per_tile, ee = e - j * per_tile;
    const int tok = ee / (kTileN / 8), r8 = (ee % (kTileN / 8)) * 8;
    const int n0 = ((unit / p.t_tiles) * p.nb + j) * kTileN;
    float a[8] = {0, 0, 0, 0, 0, 0, 0, 0}, a2[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int k = cf; k <= cl; ++k) {
      const int sl = range_start(k, p.iters, p.grid) < x0 ? 1 : 0;
      const float* src = p.ws + (((long)k * 2 + sl) * p.nb + j) * slot_floats + (long)tok * kTileN + r8;
#pragma unroll
      for (int u = 0; u < 8; u += 4) {
        const float4 f = __ldcg(reinterpret_cast<const float4*>(src + u));
        a[u] += f.x; a[u + 1] += f.y; a[u + 2] += f.z; a[u + 3] += f.w;
        if (p.dual) {
          const float4 f2 = __ldcg(reinterpret_cast<const float4*>(src + (long)p.tok_tile * kTileN + u));
          a2[u] += f2.x; a2[u + 1] += f2.y; a2[u + 2] += f2.z; a2[u + 3] += f2.w;
        }
      }
    }
    epilogue_store_vec<8>(p, t0 + tok, n0 + r8, a, a2);
  }
}

// ---- host: tensor maps ---------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  });
  return fn;
}

struct TmapCache {
  std::mutex mu;
  std::map<std::tuple<const void*, long, long, long, int>, CUtensorMap> maps;
};
TmapCache& tmap_cache() {
  static TmapCache c;
  return c;
}

}  // namespace

// bf16 row-major [rows, cols] with row stride ld (elements); box = box_rows x 64 columns.
Status make_tmap(CUtensorMap* m, const void* base, long rows, long cols, long ld, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return Status::err(WEDLM_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  WEDLM_CHECK_ARG(((uintptr_t)base & 15) == 0, "TMA base address must be 16-byte aligned");
  WEDLM_CHECK_ARG((ld * 2) % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return Status::err(WEDLM_ERR_CUDA, "cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
  return Status::ok();
}

Status cached_tmap(CUtensorMap* out, const void* base, long rows, long cols, long ld, int box_rows) {
  TmapCache& c = tmap_cache();
  std::lock_guard<std::mutex> lk(c.mu);
  auto key = std::make_tuple(base, rows, cols, ld, box_rows);
  auto it = c.maps.find(key);
  if (it != c.maps.end()) {
    *out = it->second;
    return Status::ok();
  }
  CUtensorMap m;
  WEDLM_TRY(make_tmap(&m, base, rows, cols, ld, box_rows));
  if (c.maps.size() > 4096) c.maps.clear();
  c.maps.emplace(key, m);
  *out = m;
  return Status::ok();
}

void forget_tensor_maps() {
  TmapCache& c = tmap_cache();
  std::lock_guard<std::mutex> lk(c.mu);
  c.maps.clear();
}

// ---- packed weights ---------------------------------------------------------------------
namespace {

__device__ __forceinline__ long packed_index(long gr, long c, long kb_total) {
  const long tile = gr >> 7, r = gr & 127, kb = c >> 6, cc = c & 63;
  return ((tile * kb_total + kb) * 128 + r) * 64 + (((cc >> 3) ^ (r & 7)) << 3) + (cc & 7);
}

// one thread per 8 consecutive columns (16 bytes)
__global__ void pack_kernel(const __nv_bfloat16* src, long ld, long row_off, long rows, long K,
                            __nv_bfloat16* P, int unpack) {
  const long chunks = rows * (K / 8);
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < chunks; i += (long)gridDim.x * blockDim.x) {
    const long r = i / (K / 8), c = (i % (K / 8)) * 8;
    const long pi = packed_index(row_off + r, c, K / 64);
    if (unpack)
      *reinterpret_cast<uint4*>(const_cast<__nv_bfloat16*>(src) + r * ld + c) =
          *reinterpret_cast<const uint4*>(P + pi);
    else
      *reinterpret_cast<uint4*>(P + pi) = *reinterpret_cast<const uint4*>(src + r * ld + c);
  }
}

__device__ __forceinline__ uint64_t mix64d(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

__global__ void init_packed_kernel(__nv_bfloat16* P, long row_off, long rows, long K, uint64_t seed,
                                   uint64_t tensor_id, long hash_off, float stdv) {
  const long n = rows * K;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const long r = i / K, c = i % K;
    const uint64_t h = mix64d(seed ^ mix64d((tensor_id << 44) + (uint64_t)(i + hash_off) + 1));
    const float u1 = ((float)(uint32_t)(h >> 40) + 1.f) * (1.f / 16777216.f);
    const float u2 = (float)(uint32_t)(h & 0xFFFFFF) * (1.f / 16777216.f);
    const float z = sqrtf(-2.f * logf(u1)) * cospif(2.f * u2);
    P[packed_index(row_off + r, c, K / 64)] = __float2bfloat16_rn(z * stdv);
  }
}

}  // namespace

long packed_weight_elems(long N, long K) { return ((N + 127) / 128) * 128 * K; }

Status pack_weight(const void* src, long ld, long row_off, long rows, long K, void* packed,
                   cudaStream_t st) {
  WEDLM_CHECK_ARG(K % 64 == 0 && ld % 8 == 0 && ((uintptr_t)src % 16) == 0, "bad pack layout");
  if (rows <= 0) return Status::ok();
  pack_kernel<<<1184, 256, 0, st>>>((const __nv_bfloat16*)src, ld, row_off, rows, K,
                                    (__nv_bfloat16*)packed, 0);
  WEDLM_CUDA_TRY(cudaGetLastError());
  return Status::ok();
}

Status unpack_weight(const void* packed, long row_off, long rows, long K, void* dst,
                     cudaStream_t st) {
  WEDLM_CHECK_ARG(K % 64 == 0 && ((uintptr_t)dst % 16) == 0, "bad unpack layout");
  if (rows <= 0) return Status::ok();
  pack_kernel<<<1184, 256, 0, st>>>((const __nv_bfloat16*)dst, K, row_off, rows, K,
                                    (__nv_bfloat16*)packed, 1);
  WEDLM_CUDA_TRY(cudaGetLastError());
  return Status::ok();
}

Status init_normal_packed(void* packed, long row_off, long rows, long K, uint64_t seed,
                          uint64_t tensor_id, long hash_off, float stdv, cudaStream_t st) {
  WEDLM_CHECK_ARG(K % 64 == 0, "bad packed layout");
  init_packed_kernel<<<1184, 256, 0, st>>>((__nv_bfloat16*)packed, row_off, rows, K, seed,
                                           tensor_id, hash_off, stdv);
  WEDLM_CUDA_TRY(cudaGetLastError());
  return Status::ok();
}

PartialSet partial_set(const GemmPlan& g, const float* slots, bool dual) {
  PartialSet ps;
  ps.slots = slots;
  ps.iters = (long)((g.n_tiles + g.nb - 1) / g.nb) * g.t_tiles * g.kb_total;
  ps.nb = g.nb;
  ps.grid = g.grid;
  ps.kb_total = g.kb_total;
  ps.t_tiles = g.t_tiles;
  ps.tok_tile = g.tok_tile;
  ps.maxc = g.maxc;
  ps.na = dual ? 2 : 1;
  return ps;
}

GemmPlan plan_gemm_tc(int M, int N, int K, bool dual, int num_sms, int force_nb) {
  GemmPlan g;
  // Many token rows (prefill chunks, batched serving): the GEMM is tensor-bound and its
  // operands stream from L2.  Each unit then takes 256 token rows and two weight tiles
  // (or gate and up), 512 accumulator columns in one TMEM buffer: 131 flop per operand
  // byte against 85 with one 128 x 256 tile, at the cost of the epilogue no longer
  // overlapping the next unit's main loop.
  bool wide = M >= 512;
  if (const char* e = getenv("WEDLM_GEMM_WIDE")) wide = wide && atoi(e) != 0;
  int tt = ((M + 15) / 16) * 16;
  if (tt > 256 || (dual && !wide && tt > 128)) {
    const int cap = (dual && !wide) ? 128 : 256;
    const int nt = (M + cap - 1) / cap;
    tt = ((M + nt - 1) / nt + 15) / 16 * 16;
  }
  g.tok_tile = tt < 16 ? 16 : tt;
  g.t_tiles = (M + g.tok_tile - 1) / g.tok_tile;
  g.n_tiles = (N + kTileN - 1) / kTileN;
  // Weight tiles per unit: two tiles share each activation k-block, which halves the
  // shared memory the activations take per weight byte and so raises the weight bytes in
  // flight per SM (LM head at 96 rows: 5.8 TB/s instead of 4.2; the layer GEMMs gain less,
  // as the larger units double the split-K partials their consumers read).  Dual
  // (gate/up) already shares the activations between two matrices, and above 128 token
  // rows the accumulators of two tiles would not double-buffer in TMEM.
  // Below 48 MB of weights (the 4096 x 4096 O projection) the second tile does not pay
  // for the doubled partials of the few-row case.
  long big_mb = 48;
  if (const char* e = getenv("WEDLM_GEMM_NB_MB")) big_mb = atol(e);
  const bool big = (long)N * K * 2 >= big_mb * 1024 * 1024;
  int nb = (!dual && ((g.tok_tile <= 128 && big) || wide) && g.n_tiles >= 2) ? 2 : 1;
  const char* nb_env = getenv("WEDLM_GEMM_NB");
  if (force_nb > 0 || nb_env) {
    const int f = force_nb > 0 ? force_nb : atoi(nb_env);
    if (f == 1) nb = 1;
    if (f == 2 && !dual && g.tok_tile <= 128 && g.n_tiles >= 2) nb = 2;
  }
  g.nb = nb;
  const int na = dual ? 2 : 1;
  // k-blocks per pipeline stage: larger bulk copies per stage stream faster; keep >= 2
  // stages and enough k-steps per unit for the stream-K split
  const int kb64 = K / kBK;
  int ks = 1;
  if (const char* e = getenv("WEDLM_GEMM_KS")) ks = atoi(e);
  else ks = 4;  // largest stage that still leaves two stages in the budget (see below)
  while (ks > 1 && (kb64 % ks != 0)) ks >>= 1;
  if (ks < 1) ks = 1;
  // The k-partition follows the token-tile class (up to 128 or up to 256 rows), not the
  // exact row count: a row's split-K sums then come out the same at any row count of its
  // class (a decode window of w rows, or the same window padded to the loop's capacity).
  const int tt_class = g.tok_tile <= 128 ? 128 : 256;
  while (ks > 1 && 2u * ks * (kATileBytes * na * nb + tt_class * kBK * 2) > 192u * 1024u)
    ks >>= 1;
  g.ks = ks;
  g.kb64 = kb64;
  g.kb_total = kb64 / ks;
  const long iters = (long)((g.n_tiles + nb - 1) / nb) * g.t_tiles * g.kb_total;
  g.grid = (int)(iters < num_sms ? iters : num_sms);
  g.splits = 1;
  g.stage_bytes = (uint32_t)(ks * (kATileBytes * na * nb + g.tok_tile * kBK * 2));
  const uint32_t budget = 192 * 1024;
  int st = (int)(budget / g.stage_bytes);
  g.stages = st > 16 ? 16 : (st < 2 ? 2 : st);
  g.acc_cols = (uint32_t)(g.tok_tile * na * nb);
  g.nbuf = g.acc_cols * 2 <= 512 ? 2 : 1;
  uint32_t tc = 32;
  while (tc < g.acc_cols * g.nbuf) tc <<= 1;
  g.tmem_cols = tc;
  // stages | barriers (<= 1 KB) | epilogue transpose buffers (4 warps x 32 x 33 f32)
  g.smem_bytes = 1024 + g.stages * g.stage_bytes + 1024 + 4 * 32 * 33 * 4;
  g.ws_floats = (long)g.grid * 2 * nb * na * g.tok_tile * kTileN;
  // most CTAs a unit can be shared by: ceil(kb_total / (iters / grid)) + 1
  const long per = iters / g.grid;
  g.maxc = (int)((g.kb_total + per - 1) / (per > 0 ? per : 1)) + 1;
  if (g.maxc > g.grid) g.maxc = g.grid;
  g.slot_floats = (long)g.n_tiles * g.t_tiles * g.maxc * (dual ? 2 : 1) * g.tok_tile * kTileN;
  g.counters = 0;
  return g;
}

Status run_gemm_tc(const GemmArgs& a, const GemmPlan& g, float* ws, unsigned* counters, int* err,
                   cudaStream_t st) {
  WEDLM_CHECK_ARG(a.K % kBK == 0, "tcgen05 GEMM needs K % 64 == 0");
  WEDLM_CHECK_ARG(a.M > 0 && a.N > 0, "empty GEMM");
  WEDLM_CHECK_ARG(ws != nullptr || a.slots != nullptr, "the GEMM needs its workspace");
  (void)counters;
  const bool dual = a.epi == EPI_SWIGLU_BF16;
  WEDLM_CHECK_ARG(!dual || a.W2, "SwiGLU GEMM needs the second weight matrix");
  CUtensorMap mW, mW2, mX;
  WEDLM_TRY(cached_tmap(&mX, a.X, a.M, a.K, a.ldx, g.tok_tile));
  if (a.w_packed) {
    WEDLM_CHECK_ARG(((uintptr_t)a.W % 16 == 0) && (!dual || (uintptr_t)a.W2 % 16 == 0),
                    "packed weights must be 16-byte aligned");
    mW = mX;
    mW2 = mX;
  } else {
    WEDLM_TRY(cached_tmap(&mW, a.W, a.N, a.K, a.ldw, kTileN));
    WEDLM_TRY(cached_tmap(&mW2, dual ? a.W2 : a.W, a.N, a.K, a.ldw, kTileN));
  }
  TcParams p;
  p.N = a.N;
  p.M = a.M;
  p.K = a.K;
  p.n_tiles = g.n_tiles;
  p.t_tiles = g.t_tiles;
  p.kb_total = g.kb_total;
  p.ks = g.ks;
  p.kb64 = g.kb64;
  p.iters = (long)((g.n_tiles + g.nb - 1) / g.nb) * g.t_tiles * g.kb_total;
  p.nb = g.nb;
  p.grid = g.grid;
  p.tok_tile = g.tok_tile;
  p.epi = a.epi;
  p.dual = dual ? 1 : 0;
  p.stages = g.stages;
  p.nbuf = g.nbuf;
  p.stage_bytes = g.stage_bytes;
  p.tmem_cols = g.tmem_cols;
  p.acc_cols = g.acc_cols;
  p.out = a.out;
  p.ldo = (int)a.ldo;
  p.resid = reinterpret_cast<const __nv_bfloat16*>(a.resid);
  p.ldr = (int)a.ldr;
  p.ws = ws;
  p.err = err;
  p.wp = reinterpret_cast<const uint8_t*>(a.W);
  p.wp2 = reinterpret_cast<const uint8_t*>(dual ? a.W2 : a.W);
  p.packed = a.w_packed ? 1 : 0;
  p.slots = a.slots;
  p.slot_mode = a.slots ? 1 : 0;
  p.maxc = g.maxc;
  p.poll = getenv("WEDLM_GEMM_POLL") ? atoi(getenv("WEDLM_GEMM_POLL")) : 0;
  p.nohint = getenv("WEDLM_GEMM_NOHINT") ? atoi(getenv("WEDLM_GEMM_NOHINT")) : 0;
  const int osz = a.epi == EPI_STORE_F32 ? 4 : 2;
  p.vec_ok = ((uintptr_t)a.out % 16 == 0) && ((a.ldo * osz) % 16 == 0) &&
             (a.epi != EPI_RESID_BF16 || (((uintptr_t)a.resid % 16 == 0) && (a.ldr * 2) % 16 == 0));
  int dev = 0;
  WEDLM_CUDA_TRY(cudaGetDevice(&dev));
  static unsigned attr_set = 0;  // one bit per device
  if (dev < 32 && !(attr_set & (1u << dev))) {
    WEDLM_CUDA_TRY(cudaFuncSetAttribute(gemm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        227 * 1024));
    attr_set |= 1u << dev;
  }
  WEDLM_CUDA_TRY(launch_pdl(gemm_tc_kernel, dim3((unsigned)g.grid), dim3(kThreadsTC),
                            g.smem_bytes, st, mW, mW2, mX, p));
  if (g.grid > 1 && !p.slot_mode)
    WEDLM_CUDA_TRY(launch_pdl(gemm_reduce_kernel, dim3((unsigned)(g.grid - 1)), dim3(256), 0, st, p));
  return Status::ok();
}

}  // namespace wedlm
