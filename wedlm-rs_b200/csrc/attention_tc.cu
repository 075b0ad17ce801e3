// Block attention of the reordered window against the committed-prefix KV cache, on
// the tcgen05 tensor cores (bf16 in, f32 accumulate in TMEM).
// Replaces softmax(QK^T / sqrt(d) + mask) V with GQA (src/model/attention.rs:188-221)
// and the host-built causal mask (src/model/attention.rs:255-279,
// src/model/backbone.rs:158-178): the mask is evaluated in-kernel from a per-row rank,
// key j of the window is visible to query i iff rank[j] <= rank[i] (rank = window
// index reproduces the reference), every cached key is visible.
//
// Work item = (sequence b, kv head g, 128-row query tile t, range of 128-key chunks).
// The query tile holds the `group` q heads of kv head g for 128/group window rows, so
// K and V of that kv head are read once for the whole group (GQA without repeat_kv).
//   S[q][key]  = Q[q][d] . K[key][d]      A = Q   (K-major), B = K page tiles (K-major)
//   O[q][d]   += P[q][key] . V[key][d]    A = P   (K-major), B = V^T page tiles (K-major,
//                                          the cache stores V transposed within a page)
// Both accumulators have TMEM lane = query row, so the thread that owns a query row does
// its online softmax, rescales its O row when the running max grows, and writes it out.
// Warp roles: warp 0 TMA producer of Q (once) and the K chunks, warp 10 TMA producer of
// the V chunks (K and V have rings of their own: a K stage is free as soon as its QK^T
// has run, long before the PV of the same chunk, so K(i+2) loads while the softmax of
// chunk i runs), warp 1 TMEM allocator + MMA issuer, warps 2..9 softmax / correction /
// epilogue, two threads per query row (64 key columns and 64 O columns each).  S has two
// TMEM buffers, so QK^T of chunk i+1 runs while the softmax reads chunk i.
// A work item covering only part of the keys writes (m, l, O) partials; a combine
// kernel merges them (flash-decoding split-KV).
#include <cudaTypedefs.h>

#include <cfloat>
#include <cstring>
#include <mutex>
#include <vector>

#include "layer_ops.h"
#include "sm100.cuh"

namespace wedlm {

Status make_tmap(CUtensorMap* m, const void* base, long rows, long cols, long ld, int box_rows);

namespace {

using namespace sm100;

constexpr int kThreadsAT = 352;   // warp 0 TMA Q/K, warp 1 MMA, warps 2..9 softmax, warp 10 TMA V
constexpr int kSoftThreads = 256;
constexpr int kQT = 128;        // query rows per tile
constexpr int kKC = 128;        // keys per chunk (two 64-key pages)
constexpr int kD = 128;         // head dim (this kernel)
constexpr int kBlk = 128 * 128; // bytes of one [128 rows x 64 bf16] K-block
constexpr int kKStages = 3;  // K ring
constexpr int kVStages = 2;  // V ring
constexpr float kLog2e = 1.4426950408889634f;

struct AttnWork {
  int b, g, t, c0, c1, split;  // chunk range [c0, c1)
  int part;                    // partial slot, -1 = final output written directly
};

struct AtParams {
  int rows, nh, nkv, group, page_size, pages_per_seq, num_pages, layer;
  const int* page_table;
  const int* row_seq;
  const int* seq_row0;
  const int* seq_rows;
  const int* seq_cache_len;
  const int* seq_slot;
  const int* rank;
  const AttnWork* work;
  __nv_bfloat16* out;
  long ld_out;
  float* part_o;   // [parts][128][128]
  float* part_ml;  // [parts][128][2]
  float scale_log2;
  int* err;
  // device-built plans: the live item counts (work, combine); NULL = the launch's own
  const int* n_work_dev;
  const int* n_comb_dev;
};

// 32 consecutive 32-bit columns of this thread's TMEM lane (P as packed bf16 pairs).
__device__ __forceinline__ void tmem_st32u(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]),
      "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]),
      "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]),
      "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15]))
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__global__ void __launch_bounds__(kThreadsAT, 1)
attention_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const AtParams p) {
  pdl_trigger();
  pdl_wait();
  // a device-built plan launches its upper bound of items
  if (p.n_work_dev && (int)blockIdx.x >= *p.n_work_dev) return;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  // layout: Q (2 blocks) | K stages (2 blocks each) | V stages (2 blocks each)
  //         | barriers (15) | TMEM slot | ranks      (P lives in tensor memory)
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + 2 * kBlk;
  uint8_t* sV = sK + kKStages * 2 * kBlk;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + kVStages * 2 * kBlk);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;            // [kKStages]
  uint64_t* k_empty = k_full + kKStages;  // [kKStages]
  uint64_t* v_full = k_empty + kKStages;  // [kVStages]
  uint64_t* v_empty = v_full + kVStages;  // [kVStages]
  uint64_t* s_full = v_empty + kVStages;  // [2]: S buffers
  uint64_t* p_full = s_full + 2;
  uint64_t* o_done = p_full + 1;          // bars + 14
  // fixed offsets after the barriers, so that s_krank (read as int4) stays 16-byte
  // aligned: slot at byte 128, ranks from byte 144
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);
  int* s_rank = reinterpret_cast<int*>(tmem_slot + 4);  // window ranks of sequence b
  int* s_krank = s_rank + 4096;                          // key ranks of the current chunk
  float* s_red = reinterpret_cast<float*>(s_krank + kKC);  // [4][128]: row max / sum halves

  const AttnWork w = p.work[blockIdx.x];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = w.b, g = w.g;
  const int row0 = p.seq_row0[b], S = p.seq_rows[b], L = p.seq_cache_len[b];
  const int slot = p.seq_slot[b];
  const int nchunks = w.c1 - w.c0;

  for (int j = threadIdx.x; j < S; j += blockDim.x) s_rank[j] = p.rank ? p.rank[row0 + j] : j;
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kKStages; ++s) {
      mbar_init(k_full + s, 1);
      mbar_init(k_empty + s, 1);
    }
    for (int s = 0; s < kVStages; ++s) {
      mbar_init(v_full + s, 1);
      mbar_init(v_empty + s, 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_full + 1, 1);
    mbar_init(p_full, 1);
    mbar_init(o_done, 1);
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // two S buffers (S of chunk i in buffer i % 2, so that the next chunk's QK^T runs while
  // the softmax reads this one), the O accumulator, and two P buffers (bf16 pairs, 64
  // columns each; P of chunk i in buffer i % 2), the A operand of PV
  const uint32_t tS = tmem, tO = tmem + 256, tP = tmem + 384;

  if (warp == 0 || warp == 10) {
    if (lane == 0) {
      // ---------------- TMA producers: Q and K (warp 0), V (warp 10) ----------------
      const bool kside = warp == 0;
      uint64_t* full = kside ? k_full : v_full;
      uint64_t* empty = kside ? k_empty : v_empty;
      const int nst = kside ? kKStages : kVStages;
      if (kside) {
        tma_prefetch_desc(&tmQ);
        tma_prefetch_desc(&tmK);
        // Q tile: rows (g * rows + row0) * group + t * 128 of the group-major q buffer
        const int qrow = (g * p.rows + row0) * p.group + w.t * kQT;
        mbar_arrive_expect_tx(q_full, 2 * kBlk);
        tma_load_2d(sQ, &tmQ, q_full, 0, qrow);
        tma_load_2d(sQ + kBlk, &tmQ, q_full, 64, qrow);
      } else {
        tma_prefetch_desc(&tmV);
      }
      int issued = 0;
      for (int i = 0; i < nchunks; ++i) {
        const int s = i % nst;
        const uint32_t ph = (uint32_t)(i / nst) & 1u;
        if (!mbar_wait(empty + s, ph ^ 1u, p.err, kErrAtKvEmpty)) break;
        issued = i + 1;
        uint8_t* st = (kside ? sK : sV) + s * 2 * kBlk;
        mbar_arrive_expect_tx(full + s, 2 * kBlk);
        const int c = w.c0 + i;
        for (int pg = 0; pg < 2; ++pg) {
          const int page = p.page_table[(long)slot * p.pages_per_seq + 2 * c + pg];
          if (kside) {
            // K: two d-halves (K-blocks), keys of page pg at rows 64 * pg
            const int krow = ((p.layer * p.num_pages + page) * p.nkv + g) * p.page_size;
            tma_load_2d(st + pg * (kBlk / 2), &tmK, full + s, 0, krow);
            tma_load_2d(st + kBlk + pg * (kBlk / 2), &tmK, full + s, 64, krow);
          } else {
            // V^T page: [128 d rows x 64 keys] = K-block pg of the B operand
            const int vrow = ((p.layer * p.num_pages + page) * p.nkv + g) * kD;
            tma_load_2d(st + pg * kBlk, &tmV, full + s, 0, vrow);
          }
        }
      }
      if (kside) mbar_wait(q_full, 0, p.err, kErrAtDrainQ);
      for (int s = 0; s < nst && s < issued; ++s) {
        const int last = s + ((issued - 1 - s) / nst) * nst;
        mbar_wait(full + s, (uint32_t)(last / nst) & 1u, p.err, kErrAtDrainKv);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      const uint32_t idesc = idesc_bf16_f32(128, 128);
      const uint32_t aq = smem_u32(sQ);
      bool ok = mbar_wait(q_full, 0, p.err, kErrAtMmaQ);
      // O += P(j) . V(j), once the softmax has published P(j) (in TMEM: keys 16 kk ..
      // 16 kk + 15 in columns 8 kk .. 8 kk + 7) and V(j) has landed
      auto pv = [&](int j, int code) -> bool {
        const int sv = j % kVStages;
        if (!mbar_wait(p_full, (uint32_t)j & 1u, p.err, code)) return false;
        if (!mbar_wait(v_full + sv, (uint32_t)(j / kVStages) & 1u, p.err, kErrAtMmaKv)) return false;
        tc_fence_after();
        const uint32_t bv = smem_u32(sV + sv * 2 * kBlk);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          tc_mma_f16_ts(tO, tP + (uint32_t)((j & 1) * 64 + kk * 8),
                        smem_desc_sw128(bv + (kk >> 2) * kBlk + (kk & 3) * 32), idesc,
                        j > 0 || kk > 0);
        tc_commit(o_done);
        tc_commit(v_empty + sv);
        return true;
      };
      bool all_pv = nchunks > 0;  // every PV issued (each commits o_done once)
      for (int i = 0; i < nchunks && ok; ++i) {
        const int s = i % kKStages;
        if (!mbar_wait(k_full + s, (uint32_t)(i / kKStages) & 1u, p.err, kErrAtMmaKv)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t bk = smem_u32(sK + s * 2 * kBlk);
        // S(i) = Q . K(i)^T into S buffer i % 2, issued as soon as K(i) has landed, so it
        // runs while the softmax works on S(i-1) (buffer i % 2 was freed when the softmax
        // of chunk i - 2 published P, which this thread waited for before PV(i-2))
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          tc_mma_f16(tS + (uint32_t)((i & 1) * 128),
                     smem_desc_sw128(aq + (kk >> 2) * kBlk + (kk & 3) * 32),
                     smem_desc_sw128(bk + (kk >> 2) * kBlk + (kk & 3) * 32), idesc, kk > 0);
        tc_commit(s_full + (i & 1));
        tc_commit(k_empty + s);  // K(i) is read once QK^T(i) completes
        if (i > 0 && !pv(i - 1, kErrAtMmaP)) {
          ok = false;
          break;
        }
      }
      all_pv = all_pv && ok && pv(nchunks - 1, kErrAtMmaPLast);
      // without a last PV (no chunk, or a wait gave up) one commit still lets the softmax
      // warps' final o_done wait end; after a last PV, a second commit would complete the
      // barrier's next phase and alias the parity they wait for
      if (!all_pv) tc_commit(o_done);
    }
  } else {
    // ---------------- softmax / correction / epilogue (warps 2..9) ----------------
    // Two threads per query row: warp w reads TMEM lanes (w % 4) * 32 .. + 31 and, with
    // half = (w - 2) / 4, the key / O columns half * 64 .. + 63 of those rows.  The two
    // halves of a row exchange their maxima and sums through shared memory (s_red).
    const int q4 = warp & 3;
    const int half = (warp - 2) >> 2;
    const int qr = q4 * 32 + lane;                 // query row within the tile (TMEM lane)
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    const uint32_t col0 = (uint32_t)(half * 64);
    const int qi = w.t * kQT + qr;                 // query index within (b, g)
    const bool qvalid = qi < S * p.group;
    const int r_local = qvalid ? qi / p.group : 0;
    const int my_rank = s_rank[r_local];
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int i = 0; i < nchunks && ok; ++i) {
      ok = mbar_wait(s_full + (i & 1), (uint32_t)(i >> 1) & 1u, p.err, kErrAtSoftS);
      tc_fence_after();
      const int kbase = (w.c0 + i) * kKC;
      // this half's 64 scores of the query row, after one TMEM wait; masked keys become
      // -inf (log2 units after the scale)
      float sv[64];
      tmem_ld64(tS + (uint32_t)((i & 1) * 128) + lane_off + col0, sv);
      float cm = -INFINITY;
      if (kbase + kKC <= L) {  // chunk inside the committed prefix: every key visible
#pragma unroll
        for (int j = 0; j < 64; ++j) {
          sv[j] *= p.scale_log2;
          cm = fmaxf(cm, sv[j]);
        }
      } else {
        // the chunk's key ranks, one key per first-half thread: cached keys rank below
        // every query, keys past the window above; key j is visible iff its rank <= mine
        if (half == 0) {
          const int t = qr - (L - kbase);  // window index of key qr of this chunk
          s_krank[qr] = t < 0 ? INT_MIN : (t < S ? s_rank[t] : INT_MAX);
        }
        named_bar_sync(1, kSoftThreads);
        const int4* kr4 = reinterpret_cast<const int4*>(s_krank + half * 64);
#pragma unroll
        for (int j4 = 0; j4 < 16; ++j4) {
          const int4 rk = kr4[j4];
          const int r4[4] = {rk.x, rk.y, rk.z, rk.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int j = j4 * 4 + e;
            sv[j] = r4[e] <= my_rank ? sv[j] * p.scale_log2 : -INFINITY;
            cm = fmaxf(cm, sv[j]);
          }
        }
      }
      // the row's maximum over both halves
      s_red[half * kQT + qr] = cm;
      named_bar_sync(1, kSoftThreads);
      cm = fmaxf(s_red[qr], s_red[kQT + qr]);
      const float mn = fmaxf(m, cm);
      const float base = mn == -INFINITY ? 0.f : mn;
      float ps = 0.f;
      // P = 2^(s - max) as bf16 pairs into this half's 32 columns of P buffer i % 2 in the
      // row's TMEM lane (2^-inf = 0 for masked keys).  The buffer's last reader, PV(i-2),
      // completed before the previous iteration rescaled O, so this runs while PV(i-1)
      // still accumulates.
      {
        uint32_t pk[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const __nv_bfloat162 h2 = __floats2bfloat162_rn(fast_exp2(sv[2 * j] - base),
                                                          fast_exp2(sv[2 * j + 1] - base));
          ps += __low2float(h2) + __high2float(h2);
          pk[j] = *reinterpret_cast<const uint32_t*>(&h2);
        }
        tmem_st32u(tP + (uint32_t)((i & 1) * 64) + lane_off + (uint32_t)(half * 32), pk);
      }
      // the row's sum over both halves (first half + second half)
      s_red[(2 + half) * kQT + qr] = ps;
      named_bar_sync(1, kSoftThreads);
      ps = s_red[2 * kQT + qr] + s_red[3 * kQT + qr];
      // PV(i-1) must be complete before O is rescaled (and PV(i) accumulates into it)
      if (i > 0) ok = ok && mbar_wait(o_done, (uint32_t)(i - 1) & 1u, p.err, kErrAtSoftO);
      tc_fence_after();
      // Rescale this half of the O row when its running max grew.  tcgen05.ld / st are
      // warp-wide (.sync.aligned), so the whole warp takes the branch when any of its rows
      // needs it; rows that do not keep the factor 1.
      const bool grow = i > 0 && mn > m && m != -INFINITY;
      if (__any_sync(0xffffffffu, grow)) {
        const float f = grow ? fast_exp2(m - mn) : 1.f;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          float v[16];
          tmem_ld16(tO + lane_off + col0 + c * 16, v);
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] *= f;
          tmem_st16(tO + lane_off + col0 + c * 16, v);
        }
      }
      l = (m == -INFINITY ? 0.f : l * fast_exp2(m - base)) + ps;
      m = mn;
      tc_fence_before();
      ok = named_bar_and(1, kSoftThreads, ok);  // the eight warps leave the loop together
      if (warp == 2 && lane == 0) mbar_arrive(p_full);
    }
    ok = ok && mbar_wait(o_done, (uint32_t)(nchunks > 0 ? nchunks - 1 : 0) & 1u, p.err,
                         kErrAtSoftOLast);
    tc_fence_after();
    const int r = row0 + r_local;
    const int h = g * p.group + (qi % p.group);
    const float inv = l > 0.f ? 1.f / l : 0.f;
    float ov[64];
    tmem_ld64(tO + lane_off + col0, ov);
    if (ok && qvalid) {
      if (w.part < 0) {
        __nv_bfloat16* dst = p.out + (long)r * p.ld_out + (long)h * kD + half * 64;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          uint32_t pk[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const __nv_bfloat162 h2 =
                __floats2bfloat162_rn(ov[c * 8 + 2 * j] * inv, ov[c * 8 + 2 * j + 1] * inv);
            pk[j] = *reinterpret_cast<const uint32_t*>(&h2);
          }
          *reinterpret_cast<uint4*>(dst + c * 8) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        }
      } else {
        float* po = p.part_o + ((long)w.part * kQT + qr) * kD + half * 64;
#pragma unroll
        for (int c = 0; c < 16; ++c)
          *reinterpret_cast<float4*>(po + 4 * c) =
              make_float4(ov[4 * c], ov[4 * c + 1], ov[4 * c + 2], ov[4 * c + 3]);
      }
    }
    if (ok && qvalid && w.part >= 0 && half == 0) {
      p.part_ml[((long)w.part * kQT + qr) * 2] = m;
      p.part_ml[((long)w.part * kQT + qr) * 2 + 1] = l;
    }
    tc_fence_before();
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Merge the split-KV partials of one (b, g, t) tile: one warp per query row.
struct CombineItem {
  int b, g, t, part0, nparts;
};

__global__ void attention_combine_kernel(const CombineItem* items, int nitems, AtParams p) {
  pdl_trigger();
  pdl_wait();
  const int wid = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (wid >= nitems * kQT) return;
  if (p.n_comb_dev && wid >= *p.n_comb_dev * kQT) return;
  const CombineItem it = items[wid / kQT];
  const int qr = wid % kQT;
  const int S = p.seq_rows[it.b];
  const int qi = it.t * kQT + qr;
  if (qi >= S * p.group) return;
  // (m, l) of up to 32 parts at once: lane k holds part k; then the O rows of 8 parts
  // per round, every load of a round in flight together
  float M = -INFINITY;
  for (int k0 = 0; k0 < it.nparts; k0 += 32) {
    const int k = k0 + lane;
    if (k < it.nparts) {
      const float* ml = p.part_ml + ((long)(it.part0 + k) * kQT + qr) * 2;
      if (ml[1] > 0.f) M = fmaxf(M, ml[0]);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
  float acc[4] = {0.f, 0.f, 0.f, 0.f}, lsum = 0.f;
  for (int k0 = 0; k0 < it.nparts; k0 += 32) {
    const int nk = min(32, it.nparts - k0);
    float f = 0.f, lk = 0.f;
    if (lane < nk) {
      const long pi = (long)(it.part0 + k0 + lane) * kQT + qr;
      const float mk = p.part_ml[pi * 2];
      lk = p.part_ml[pi * 2 + 1];
      f = lk > 0.f ? fast_exp2(mk - M) : 0.f;
    }
    float fl = f * lk;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) fl += __shfl_xor_sync(0xffffffffu, fl, o);
    lsum += fl;
    for (int j0 = 0; j0 < nk; j0 += 8) {
      float4 v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int kk = k0 + (j0 + j < nk ? j0 + j : j0);
        v[j] = *reinterpret_cast<const float4*>(p.part_o + ((long)(it.part0 + kk) * kQT + qr) * kD +
                                                lane * 4);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float fj = __shfl_sync(0xffffffffu, f, (j0 + j) & 31);
        if (j0 + j < nk) {
          acc[0] += fj * v[j].x;
          acc[1] += fj * v[j].y;
          acc[2] += fj * v[j].z;
          acc[3] += fj * v[j].w;
        }
      }
    }
  }
  const float inv = lsum > 0.f ? 1.f / lsum : 0.f;
  const int r = p.seq_row0[it.b] + qi / p.group;
  const int h = it.g * p.group + qi % p.group;
  __nv_bfloat16* dst = p.out + (long)r * p.ld_out + (long)h * kD + lane * 4;
  const __nv_bfloat162 a = __floats2bfloat162_rn(acc[0] * inv, acc[1] * inv);
  const __nv_bfloat162 c = __floats2bfloat162_rn(acc[2] * inv, acc[3] * inv);
  uint2 pk;
  pk.x = *reinterpret_cast<const uint32_t*>(&a);
  pk.y = *reinterpret_cast<const uint32_t*>(&c);
  *reinterpret_cast<uint2*>(dst) = pk;
}

}  // namespace

// ---- host: plan once per forward, run once per layer ------------------------------------
// Workspace layout (floats): [AttnWork table | CombineItem table | part_o | part_ml].
long attention_ws_floats(const AttnArgs& a) {
  const long tiles = (long)a.nkv * (((long)a.rows * a.group + kQT - 1) / kQT + a.nseq);
  const long chunks = (a.max_kv + kKC - 1) / kKC + 1;
  const long items = tiles * chunks;
  return items * 8 + items * 6 + items * (long)kQT * (kD + 2) + 1024;
}

Status plan_attention_tc(const AttnArgs& a, const int* h_seq_rows, const int* h_cache_len,
                         int num_sms, float* ws, long ws_floats, void* h_staging,
                         size_t staging_bytes, AttnPlan* plan, cudaStream_t st) {
  WEDLM_CHECK_ARG(a.head_dim == kD, "tensor-core attention needs head_dim 128");
  WEDLM_CHECK_ARG(a.page_size == 64, "tensor-core attention needs 64-token pages");
  WEDLM_CHECK_ARG(kQT % a.group == 0, "query tile must hold whole GQA groups");
  std::vector<AttnWork> work;
  std::vector<CombineItem> comb;
  long base = 0;
  for (int b = 0; b < a.nseq; ++b) {
    WEDLM_CHECK_ARG(h_seq_rows[b] <= 4096, "window longer than 4096 rows");
    base += (long)a.nkv * ((h_seq_rows[b] * a.group + kQT - 1) / kQT);
  }
  // Split the key range so that all work items run in one wave (one CTA per SM: the
  // kernel's shared memory holds Q, two K/V stages and P): a second wave would double
  // the fixed cost per item (TMEM allocation, Q load, first K/V latency, epilogue).
  int part = 0;
  for (int b = 0; b < a.nseq; ++b) {
    const int S = h_seq_rows[b], L = h_cache_len[b];
    if (S == 0) continue;
    const int tiles = (S * a.group + kQT - 1) / kQT;
    const int chunks = (L + S + kKC - 1) / kKC;
    int splits = base > 0 ? (int)(num_sms / base) : 1;
    splits = splits < 1 ? 1 : (splits > chunks ? chunks : splits);
    for (int g = 0; g < a.nkv; ++g)
      for (int t = 0; t < tiles; ++t) {
        if (splits > 1) comb.push_back(CombineItem{b, g, t, part, splits});
        for (int s2 = 0; s2 < splits; ++s2) {
          AttnWork w;
          w.b = b;
          w.g = g;
          w.t = t;
          w.c0 = (int)((long)chunks * s2 / splits);
          w.c1 = (int)((long)chunks * (s2 + 1) / splits);
          w.split = s2;
          w.part = splits > 1 ? part++ : -1;
          work.push_back(w);
        }
      }
  }
  plan->n_work = (int)work.size();
  plan->n_comb = (int)comb.size();
  if (work.empty()) return Status::ok();
  const long need = (long)work.size() * 8 + (long)comb.size() * 6 + 4 + (long)part * kQT * (kD + 2);
  WEDLM_CHECK_ARG(need <= ws_floats, "attention workspace too small");
  // the combine table starts 8 floats per work item into the workspace
  static_assert(sizeof(AttnWork) <= 8 * sizeof(float), "AttnWork slot");
  static_assert(sizeof(CombineItem) <= 6 * sizeof(float), "CombineItem slot");
  const size_t wbytes = work.size() * sizeof(AttnWork), cbytes = comb.size() * sizeof(CombineItem);
  const size_t coff = work.size() * 8 * sizeof(float);
  WEDLM_CHECK_ARG(coff + cbytes <= staging_bytes, "attention staging too small");
  uint8_t* hs = reinterpret_cast<uint8_t*>(h_staging);
  memcpy(hs, work.data(), wbytes);
  memcpy(hs + coff, comb.data(), cbytes);
  WEDLM_CUDA_TRY(cudaMemcpyAsync(ws, hs, coff + cbytes, cudaMemcpyHostToDevice, st));
  plan->work = ws;
  plan->comb = ws + work.size() * 8;
  float* po = ws + work.size() * 8 + comb.size() * 6;
  po = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(po) + 15) & ~uintptr_t(15));
  plan->part_o = po;
  plan->part_ml = po + (long)part * kQT * kD;
  return Status::ok();
}

// ---- the same plan built on the device -------------------------------------------------
// For the decode loop that keeps its bookkeeping on the device (the window rows and cache
// lengths of a step exist only there): one CTA computes exactly the items
// plan_attention_tc computes from host copies of the same lengths, in the same order.
struct AttnDevPlan {
  int nseq, nkv, group, num_sms, max_work, max_comb;
  const int* seq_rows;
  const int* seq_cache_len;
  AttnWork* work;
  CombineItem* comb;
  int* counts;  // [2]: work items, combine items
  int* err;
};

__device__ __forceinline__ int last_le(const int* off, int n, int v) {
  int lo = 0, hi = n - 1;  // the last index b in [0, n) with off[b] <= v
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (off[mid] <= v) lo = mid; else hi = mid - 1;
  }
  return lo;
}

__global__ void attention_plan_kernel(AttnDevPlan a) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ int sh_off[];  // [3][nseq + 1]: work, combine and part offsets
  int* wo = sh_off;
  int* co = wo + a.nseq + 1;
  int* po = co + a.nseq + 1;
  __shared__ long s_base;
  __shared__ int s_nw, s_nc;
  auto tiles_of = [&](int S) { return (S * a.group + kQT - 1) / kQT; };
  auto splits_of = [&](long base, int S, int L) {
    const int chunks = (L + S + kKC - 1) / kKC;
    int splits = base > 0 ? (int)(a.num_sms / base) : 1;
    return splits < 1 ? 1 : (splits > chunks ? chunks : splits);
  };
  if (threadIdx.x == 0) {
    long base = 0;
    for (int b = 0; b < a.nseq; ++b) base += (long)a.nkv * tiles_of(a.seq_rows[b]);
    int nw = 0, nc = 0, np = 0;
    for (int b = 0; b < a.nseq; ++b) {
      wo[b] = nw;
      co[b] = nc;
      po[b] = np;
      const int S = a.seq_rows[b];
      if (S == 0) continue;
      const int tiles = tiles_of(S), splits = splits_of(base, S, a.seq_cache_len[b]);
      nw += a.nkv * tiles * splits;
      if (splits > 1) {
        nc += a.nkv * tiles;
        np += a.nkv * tiles * splits;
      }
    }
    wo[a.nseq] = nw;
    co[a.nseq] = nc;
    po[a.nseq] = np;
    if (nw > a.max_work || nc > a.max_comb) {  // outside the launch bound: run nothing
      nw = nc = 0;
      if (a.err) atomicCAS(a.err, 0, kErrAtPlan);
    }
    s_base = base;
    s_nw = nw;
    s_nc = nc;
    a.counts[0] = nw;
    a.counts[1] = nc;
  }
  __syncthreads();
  const long base = s_base;
  for (int i = threadIdx.x; i < s_nw; i += blockDim.x) {
    const int b = last_le(wo, a.nseq, i);
    const int S = a.seq_rows[b], L = a.seq_cache_len[b];
    const int tiles = tiles_of(S), splits = splits_of(base, S, L);
    const int chunks = (L + S + kKC - 1) / kKC;
    const int local = i - wo[b];
    const int s2 = local % splits, gt = local / splits;
    AttnWork w;
    w.b = b;
    w.g = gt / tiles;
    w.t = gt % tiles;
    w.c0 = (int)((long)chunks * s2 / splits);
    w.c1 = (int)((long)chunks * (s2 + 1) / splits);
    w.split = s2;
    w.part = splits > 1 ? po[b] + local : -1;
    a.work[i] = w;
  }
  for (int j = threadIdx.x; j < s_nc; j += blockDim.x) {
    const int b = last_le(co, a.nseq, j);
    const int S = a.seq_rows[b];
    const int tiles = tiles_of(S), splits = splits_of(base, S, a.seq_cache_len[b]);
    const int local = j - co[b];
    a.comb[j] = CombineItem{b, local / tiles, local % tiles, po[b] + local * splits, splits};
  }
}

long attention_ws_floats_device(int max_work, int max_comb) {
  return (long)max_work * 8 + (long)max_comb * 6 + 4 + (long)max_work * kQT * (kD + 2) + 64;
}

Status plan_attention_tc_device(const AttnArgs& a, int num_sms, float* ws, long ws_floats,
                                int max_work, int max_comb, int* counts, int* err,
                                AttnPlan* plan, cudaStream_t st) {
  WEDLM_CHECK_ARG(a.head_dim == kD, "tensor-core attention needs head_dim 128");
  WEDLM_CHECK_ARG(a.page_size == 64, "tensor-core attention needs 64-token pages");
  WEDLM_CHECK_ARG(kQT % a.group == 0, "query tile must hold whole GQA groups");
  WEDLM_CHECK_ARG(a.nseq >= 1 && a.nseq <= 4000, "bad number of sequences");
  WEDLM_CHECK_ARG(max_work >= 1 && max_comb >= 1 && counts, "bad plan bounds");
  WEDLM_CHECK_ARG(attention_ws_floats_device(max_work, max_comb) <= ws_floats,
                  "attention workspace too small");
  AttnDevPlan d;
  d.nseq = a.nseq;
  d.nkv = a.nkv;
  d.group = a.group;
  d.num_sms = num_sms;
  d.max_work = max_work;
  d.max_comb = max_comb;
  d.seq_rows = a.seq_rows;
  d.seq_cache_len = a.seq_cache_len;
  d.work = reinterpret_cast<AttnWork*>(ws);
  d.comb = reinterpret_cast<CombineItem*>(ws + (long)max_work * 8);
  d.counts = counts;
  d.err = err;
  const size_t smem = sizeof(int) * 3 * (a.nseq + 1);
  WEDLM_CUDA_TRY(launch_pdl(attention_plan_kernel, dim3(1), dim3(512), smem, st, d));
  plan->n_work = max_work;
  plan->n_comb = max_comb;
  plan->work = ws;
  plan->comb = ws + (long)max_work * 8;
  float* po = ws + (long)max_work * 8 + (long)max_comb * 6;
  po = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(po) + 15) & ~uintptr_t(15));
  plan->part_o = po;
  plan->part_ml = po + (long)max_work * kQT * kD;
  plan->n_work_dev = counts;
  plan->n_comb_dev = counts + 1;
  return Status::ok();
}

Status run_attention_tc(const AttnArgs& a, const AttnPlan& plan, int* err, cudaStream_t st) {
  if (plan.n_work == 0) return Status::ok();
  CUtensorMap mQ, mK, mV;
  WEDLM_TRY(make_tmap(&mQ, a.q, (long)a.nkv * a.rows * a.group, kD, kD, kQT));
  WEDLM_TRY(make_tmap(&mK, a.kcache, (long)a.num_layers * a.num_pages * a.nkv * a.page_size, kD, kD, 64));
  WEDLM_TRY(make_tmap(&mV, a.vcache, (long)a.num_layers * a.num_pages * a.nkv * kD, a.page_size,
                      a.page_size, kD));
  AtParams p;
  p.rows = a.rows;
  p.nh = a.nh;
  p.nkv = a.nkv;
  p.group = a.group;
  p.page_size = a.page_size;
  p.pages_per_seq = a.pages_per_seq;
  p.num_pages = a.num_pages;
  p.layer = a.layer;
  p.page_table = a.page_table;
  p.row_seq = a.row_seq;
  p.seq_row0 = a.seq_row0;
  p.seq_rows = a.seq_rows;
  p.seq_cache_len = a.seq_cache_len;
  p.seq_slot = a.seq_slot;
  p.rank = a.rank;
  p.work = reinterpret_cast<const AttnWork*>(plan.work);
  p.out = reinterpret_cast<__nv_bfloat16*>(a.out);
  p.ld_out = a.ld_out;
  p.part_o = plan.part_o;
  p.part_ml = plan.part_ml;
  p.scale_log2 = kLog2e / sqrtf((float)kD);
  p.err = err;
  p.n_work_dev = plan.n_work_dev;
  p.n_comb_dev = plan.n_comb_dev;
  const size_t smem =
      1024 + (2 + kKStages * 2 + kVStages * 2) * kBlk + 18 * 8 + 4096 * 4 + kKC * 4 + 4 * kQT * 4;
  int dev = 0;
  WEDLM_CUDA_TRY(cudaGetDevice(&dev));
  static unsigned attr_set = 0;
  if (dev < 32 && !(attr_set & (1u << dev))) {
    WEDLM_CUDA_TRY(cudaFuncSetAttribute(attention_tc_kernel,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    attr_set |= 1u << dev;
  }
  WEDLM_CUDA_TRY(launch_pdl(attention_tc_kernel, dim3((unsigned)plan.n_work), dim3(kThreadsAT),
                            smem, st, mQ, mK, mV, p));
  if (plan.n_comb > 0) {
    const long warps = (long)plan.n_comb * kQT;
    WEDLM_CUDA_TRY(launch_pdl(attention_combine_kernel, dim3((unsigned)((warps + 7) / 8)), dim3(256),
                              0, st, reinterpret_cast<const CombineItem*>(plan.comb), plan.n_comb, p));
  }
  return Status::ok();
}

}  // namespace wedlm
