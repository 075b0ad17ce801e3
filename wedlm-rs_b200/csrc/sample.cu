// Seeded T > 0 sampling of the selected mask rows (sample_from_probs / sample_nucleus,
// src/decoding/sampler.rs:306-351) with one 1024-thread CTA per row.
//
// p = softmax(x / T) is handled unnormalised as e_i = exp((x_i - max) / T) <= 1, held in
// 2^-40 fixed point: every sum below is an exact 64-bit integer sum, so the result does
// not depend on the order of the additions (the row's chunks, the warps, the shared
// memory atomics, the ranks of a split vocabulary) and a row always samples the same
// token for the same draw.
//   multinomial (top_p >= 1): the first index whose running sum exceeds u * S (the row's
//     chunk sums are scanned across the block, and the one thread whose chunk holds the
//     crossing walks it);
//   nucleus (top_p < 1): tokens in descending probability, ties in index order (the
//     reference's stable sort).  A radix select over an order-preserving key of the
//     logit (8 bits per level, MSB first, bucket counts and fixed-point sums in shared
//     memory) finds the cutoff value whose running sum first reaches top_p * S and how
//     many of its ties the nucleus keeps; a second radix walk over the nucleus finds the
//     value where u * total is crossed, and a block scan of per-thread tie counts finds
//     the tie in index order.
// The split-vocabulary sampler (run_shard_sample) runs the same steps as phases, each
// rank over its own shard, with the per-row maxima, sums, bucket tables and tie counts
// all-gathered between phases; the decisions use the same helpers as the single kernel.
#include <algorithm>
#include <cmath>
#include <cstdint>

#include "sample.cuh"

namespace wedlm {

namespace {

constexpr int kST = 1024;
constexpr int kSW = kST / 32;
constexpr float kFix = 1099511627776.0f;  // 2^40

// Logit access and an order-preserving unsigned key (larger logit -> larger key).
template <typename T>
struct Row;
template <>
struct Row<__nv_bfloat16> {
  static constexpr int kBits = 16;
  __device__ static float x(const __nv_bfloat16* r, int i) { return __bfloat162float(r[i]); }
  __device__ static uint32_t key(const __nv_bfloat16* r, int i) {
    const uint32_t b = __bfloat16_as_ushort(r[i]);
    return (b & 0x8000u) ? (~b & 0xFFFFu) : (b | 0x8000u);
  }
  __device__ static float x_of_key(uint32_t k) {
    const uint32_t b = (k & 0x8000u) ? (k & 0x7FFFu) : (~k & 0xFFFFu);
    return __uint_as_float(b << 16);
  }
};
template <>
struct Row<float> {
  static constexpr int kBits = 32;
  __device__ static float x(const float* r, int i) { return r[i]; }
  __device__ static uint32_t key(const float* r, int i) {
    const uint32_t b = __float_as_uint(r[i]);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  }
  __device__ static float x_of_key(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
  }
};

__device__ __forceinline__ uint64_t fix_of(float x, float mx, float sc) {
  return __float2ull_rn(exp2f((x - mx) * sc) * kFix);
}

__device__ float block_max(float v, float* sh) {
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    float w = sh[threadIdx.x];
    for (int o = 16; o; o >>= 1) w = fmaxf(w, __shfl_xor_sync(0xffffffffu, w, o));
    if (threadIdx.x == 0) sh[0] = w;
  }
  __syncthreads();
  const float r = sh[0];
  __syncthreads();
  return r;
}

// Exclusive block scan of one value per thread; *total receives the block sum.
__device__ uint64_t block_scan(uint64_t v, uint64_t* sh, uint64_t* total) {
  const int l = threadIdx.x & 31, w = threadIdx.x >> 5;
  uint64_t inc = v;
  for (int o = 1; o < 32; o <<= 1) {
    const uint64_t n = __shfl_up_sync(0xffffffffu, inc, o);
    if (l >= o) inc += n;
  }
  if (l == 31) sh[w] = inc;
  __syncthreads();
  if (w == 0) {
    const uint64_t t = sh[l];
    uint64_t ti = t;
    for (int o = 1; o < 32; o <<= 1) {
      const uint64_t n = __shfl_up_sync(0xffffffffu, ti, o);
      if (l >= o) ti += n;
    }
    sh[l] = ti - t;
    if (l == 31) sh[kSW] = ti;
  }
  __syncthreads();
  const uint64_t pre = sh[w] + inc - v;
  *total = sh[kSW];
  __syncthreads();
  return pre;
}

// One radix level's decision (one thread): the buckets are visited from the largest key
// down, and the walk enters the bucket whose running sum first reaches `target` (>= when
// `inclusive`, the nucleus cutoff; > otherwise, the draw).  acc = fixed-point sum of the
// members above the entered bucket; n = members in it.
struct RadixPick {
  uint32_t key;
  uint64_t acc;
  unsigned n;
};
__device__ RadixPick radix_pick(const unsigned* cnt, const unsigned long long* sum,
                                uint64_t target, bool inclusive, uint32_t prefix, int shift,
                                uint64_t acc) {
  int sel = -1, low = -1;
  uint64_t acc_low = 0;
  for (int b = 255; b >= 0; --b) {
    if (!cnt[b]) continue;
    const uint64_t nxt = acc + sum[b];
    if (inclusive ? nxt >= target : nxt > target) {
      sel = b;
      break;
    }
    acc_low = acc;
    low = b;
    acc = nxt;
  }
  if (sel < 0) {  // not reached (only when rounding put the target past the end)
    sel = low;
    acc = acc_low;
  }
  if (sel < 0) sel = 0;  // no member at all: cannot happen, keeps the index in range
  RadixPick p;
  p.key = prefix | ((uint32_t)sel << shift);
  p.acc = acc;
  p.n = cnt[sel];
  return p;
}

// How many of the n_eq ties at the cutoff value (fixed-point weight q_star each) the
// nucleus keeps, in index order, for its sum to reach TA; and the nucleus total.
__device__ void nucleus_cut(uint64_t TA, uint64_t acc_a, unsigned n_eq, uint64_t q_star,
                            uint64_t* j_out, uint64_t* total) {
  uint64_t j = n_eq;
  if (q_star > 0) {
    const uint64_t need = TA > acc_a ? TA - acc_a : 0;
    j = (need + q_star - 1) / q_star;
  }
  j = j < 1 ? 1 : (j > n_eq ? n_eq : j);
  *j_out = j;
  *total = acc_a + j * q_star;
}

// Which of `cap` ties of weight q (after `acc` of heavier members) holds the draw TB.
__device__ uint64_t tie_index(uint64_t TB, uint64_t acc, uint64_t q, uint64_t cap) {
  uint64_t i = q > 0 ? (TB - acc) / q : 0;
  return i > cap - 1 ? cap - 1 : i;
}

struct Shared {
  float f[kSW];
  uint64_t scan[kSW + 1];
  unsigned cnt[256];
  unsigned long long sum[256];
  float u;
  int skip, tok;
  uint32_t key;
  unsigned n;
  unsigned long long acc;
};

// Bucket table of one radix level over columns [c0, c1) of `row`: members are the keys
// that match `prefix` under `pmask` and, when `above`, exceed `floor_key`.
template <typename R, typename T>
__device__ void radix_buckets(Shared& s, const T* row, int c0, int c1, uint32_t prefix,
                              uint32_t pmask, int shift, bool above, uint32_t floor_key,
                              float mx, float sc) {
  for (int b = threadIdx.x; b < 256; b += kST) {
    s.cnt[b] = 0u;
    s.sum[b] = 0ull;
  }
  __syncthreads();
  for (int i = c0; i < c1; ++i) {
    const uint32_t k = R::key(row, i);
    if ((k & pmask) != prefix || (above && k <= floor_key)) continue;
    const int b = (k >> shift) & 255;
    atomicAdd(&s.cnt[b], 1u);
    atomicAdd(&s.sum[b], (unsigned long long)fix_of(R::x(row, i), mx, sc));
  }
  __syncthreads();
}

template <typename T>
__global__ void __launch_bounds__(kST) sample_kernel(SampleArgs a) {
  using R = Row<T>;
  __shared__ Shared s;
  const int r = blockIdx.x;
  if (threadIdx.x == 0) {
    int skip = 0;
    float u;
    if (a.u) {
      u = a.u[r];
    } else {
      // the sequence of row r: the last b with seq_rows[b] <= r
      int lo = 0, hi = a.nseq - 1;
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (a.seq_rows[mid] <= r) lo = mid; else hi = mid - 1;
      }
      const int rel = r - a.seq_rows[lo];
      skip = 1;
      for (int i = 0; i < a.n_selected[lo]; ++i)
        if (a.selected[a.seq_rows[lo] + i] == rel) {
          skip = 0;
          break;
        }
      u = sample_draw(a.seed, (uint64_t)a.seq_key[lo], (uint64_t)a.seq_step[lo], (uint64_t)rel);
    }
    s.u = u;
    s.skip = skip;
    s.tok = 0;
  }
  __syncthreads();
  if (s.skip) return;

  const T* row = reinterpret_cast<const T*>(a.logits) + (long)r * a.ld;
  const int V = a.V;
  const int C = (V + kST - 1) / kST;
  const int c0 = min(V, (int)threadIdx.x * C), c1 = min(V, c0 + C);
  const float sc = 1.4426950408889634f / a.temperature;
  float mx = -INFINITY;
  for (int i = c0; i < c1; ++i) mx = fmaxf(mx, R::x(row, i));
  mx = block_max(mx, s.f);
  auto fix = [&](float x) -> uint64_t { return fix_of(x, mx, sc); };

  uint64_t cs = 0;
  for (int i = c0; i < c1; ++i) cs += fix(R::x(row, i));
  uint64_t S;
  const uint64_t pre = block_scan(cs, s.scan, &S);

  if (a.top_p >= 1.f) {
    // sample_from_probs: first index whose running sum exceeds u * S (sampler.rs:306-317);
    // the last token when none does
    const uint64_t target = (uint64_t)((double)s.u * (double)S);
    if (threadIdx.x == 0) s.tok = V - 1;
    __syncthreads();
    if (target >= pre && target < pre + cs) {
      uint64_t acc = pre;
      for (int i = c0; i < c1; ++i) {
        acc += fix(R::x(row, i));
        if (target < acc) {
          s.tok = i;
          break;
        }
      }
    }
    __syncthreads();
    if (threadIdx.x == 0) a.tokens[r] = s.tok;
    return;
  }

  // ---- sample_nucleus (sampler.rs:320-351) ----
  // Radix walk, MSB first; returns the final key, s.acc = fixed-point sum of the members
  // above it, s.n = members equal to it.
  auto walk = [&](uint64_t target, bool inclusive, bool above, uint32_t floor_key) {
    uint32_t prefix = 0, pmask = 0;
    uint64_t acc = 0;
    for (int shift = R::kBits - 8; shift >= 0; shift -= 8) {
      radix_buckets<R>(s, row, c0, c1, prefix, pmask, shift, above, floor_key, mx, sc);
      if (threadIdx.x == 0) {
        const RadixPick p = radix_pick(s.cnt, s.sum, target, inclusive, prefix, shift, acc);
        s.key = p.key;
        s.acc = p.acc;
        s.n = p.n;
      }
      __syncthreads();
      prefix = s.key;
      acc = s.acc;
      pmask |= 0xFFu << shift;
      __syncthreads();
    }
    return prefix;
  };

  // cutoff: the first value whose running sum (descending) reaches top_p * S
  const uint64_t TA = (uint64_t)ceil((double)a.top_p * (double)S);
  const uint32_t vstar = walk(TA, true, false, 0u);
  const uint64_t acc_a = s.acc;
  const unsigned n_eq = s.n;
  const uint64_t q_star = fix(R::x_of_key(vstar));
  // ties at the cutoff join in index order until the sum reaches top_p * S
  uint64_t j, total;
  nucleus_cut(TA, acc_a, n_eq, q_star, &j, &total);

  // the crossing of u * total in the nucleus
  const uint64_t TB = (uint64_t)((double)s.u * (double)total);
  uint32_t w;
  uint64_t i_tie;
  if (TB >= acc_a) {
    w = vstar;
    i_tie = tie_index(TB, acc_a, q_star, j);
  } else {
    w = walk(TB, false, true, vstar);
    i_tie = tie_index(TB, s.acc, fix(R::x_of_key(w)), s.n);
  }
  // the i_tie-th token (index order) whose key is w
  uint64_t n = 0;
  for (int i = c0; i < c1; ++i) n += (R::key(row, i) == w);
  uint64_t tot;
  const uint64_t tpre = block_scan(n, s.scan, &tot);
  if (i_tie >= tpre && i_tie < tpre + n) {
    uint64_t c = tpre;
    for (int i = c0; i < c1; ++i)
      if (R::key(row, i) == w) {
        if (c == i_tie) {
          s.tok = i;
          break;
        }
        ++c;
      }
  }
  __syncthreads();
  if (threadIdx.x == 0) a.tokens[r] = s.tok;
}

// ---------------------------------------------------------------------------------------
// Split-vocabulary phases.  One CTA per row r = k * rmax + j (mask row j of rank k).  A
// phase reads the previous gather (recv: [nranks][stride bytes]) and writes this rank's
// payload (send); every rank derives the same ShardSampleRow state.
//   Max      : send f32 max[rows] (this shard's maximum), int flag[rmax] (own rows picked
//              by the commit rule)
//   Sum      : send u64 sum[rows] (this shard's fixed-point sum under the global maximum)
//   Pick     : (multinomial) send int token[rows] (the global token where this shard holds
//              the crossing of u * S, else -1)
//   RadixA0  : (nucleus) S, TA; bucket table of walk A's first level
//   Radix    : decide the previous level of walk `walk`; bucket table of level `shift`
//   AB       : decide walk A's last level (cutoff, ties kept, total, TB); walk B's first
//              bucket table when the draw falls above the cutoff value
//   Tie      : decide walk B's last level (or take the cutoff value); send u64 count of
//              this shard's keys equal to the drawn value
//   TiePick  : send int token[rows] (the global token where this shard holds the tie)
enum { kPhMax, kPhSum, kPhPick, kPhRadixA0, kPhRadix, kPhAB, kPhTie, kPhTiePick };
constexpr int kBucketBytes = 256 * 4 + 256 * 8;

struct ShardPhase {
  int phase = kPhMax;
  int shift = 0;     // bucket level of this phase (Radix / RadixA0 / AB)
  int walk_b = 0;    // Radix: which walk
  size_t stride = 0; // per-rank bytes of the previous gather
};

template <typename U>
__device__ __forceinline__ U& at(void* base, size_t off) {
  return *reinterpret_cast<U*>(reinterpret_cast<char*>(base) + off);
}
template <typename U>
__device__ __forceinline__ U at(const void* base, size_t off) {
  return *reinterpret_cast<const U*>(reinterpret_cast<const char*>(base) + off);
}

template <typename T>
__global__ void __launch_bounds__(kST) shard_sample_kernel(ShardSampleArgs a, ShardPhase ph) {
  using R = Row<T>;
  __shared__ Shared s;
  __shared__ int s_go;
  const int r = blockIdx.x;
  const int rows = a.nranks * a.rmax;
  const int k = r / a.rmax, jr = r - k * a.rmax;
  const int V = a.V;
  const int C = (V + kST - 1) / kST;
  const int c0 = min(V, (int)threadIdx.x * C), c1 = min(V, c0 + C);
  const T* row = reinterpret_cast<const T*>(a.logits) + (long)r * a.ld;
  const float sc = 1.4426950408889634f / a.temperature;
  ShardSampleRow& q = a.state[r];
  const void* rv = a.xrecv;
  void* sd = a.xsend;

  if (ph.phase == kPhMax) {
    const bool valid = jr < a.hdr[4 * k + 1];
    if (threadIdx.x == 0 && k == a.me) {
      // own row jr: picked by the commit rule?
      int flag = 0;
      if (valid) {
        int lo = 0, hi = a.nseq - 1;
        while (lo < hi) {
          const int mid = (lo + hi + 1) >> 1;
          if (a.seq_rows[mid] <= jr) lo = mid; else hi = mid - 1;
        }
        const int rel = jr - a.seq_rows[lo];
        for (int i = 0; i < a.n_selected[lo]; ++i)
          if (a.selected[a.seq_rows[lo] + i] == rel) {
            flag = 1;
            break;
          }
      }
      at<int>(sd, (size_t)rows * 4 + (size_t)jr * 4) = flag;
    }
    float mx = -INFINITY;
    if (valid)
      for (int i = c0; i < c1; ++i) mx = fmaxf(mx, R::x(row, i));
    mx = block_max(mx, s.f);
    if (threadIdx.x == 0) at<float>(sd, (size_t)r * 4) = mx;
    return;
  }

  if (ph.phase == kPhSum) {
    if (threadIdx.x == 0) {
      const int sel = at<int>(rv, (size_t)k * ph.stride + (size_t)rows * 4 + (size_t)jr * 4);
      float mx = -INFINITY;
      for (int kk = 0; kk < a.nranks; ++kk)
        mx = fmaxf(mx, at<float>(rv, (size_t)kk * ph.stride + (size_t)r * 4));
      q.sel = sel;
      q.mx = mx;
      q.walk_b = 0;
      s_go = sel;
      s.f[0] = mx;
      if (!sel) at<unsigned long long>(sd, (size_t)r * 8) = 0ull;
    }
    __syncthreads();
    if (!s_go) return;
    const float mx = s.f[0];
    uint64_t cs = 0;
    for (int i = c0; i < c1; ++i) cs += fix_of(R::x(row, i), mx, sc);
    uint64_t S;
    block_scan(cs, s.scan, &S);
    if (threadIdx.x == 0) at<unsigned long long>(sd, (size_t)r * 8) = S;
    return;
  }

  if (ph.phase == kPhPick || ph.phase == kPhTiePick) {
    // Which shard holds the target: the exclusive prefix of the gathered per-shard values
    // (sums for the multinomial target, tie counts for the nucleus tie index).
    if (threadIdx.x == 0) {
      s_go = 0;
      s.tok = -1;
      if (q.sel) {
        uint64_t tot = 0, pre = 0, mine = 0;
        for (int kk = 0; kk < a.nranks; ++kk) {
          const uint64_t v = at<unsigned long long>(rv, (size_t)kk * ph.stride + (size_t)r * 8);
          if (kk < a.me) pre += v;
          if (kk == a.me) mine = v;
          tot += v;
        }
        uint64_t target;
        if (ph.phase == kPhPick) {
          q.S = tot;
          target = (uint64_t)((double)a.u[r] * (double)tot);
          // the last token when no index crosses (sample_from_probs' fallback)
          if (target >= tot && a.me == a.nranks - 1) s.tok = a.V_total - 1;
        } else {
          target = q.i_tie;
        }
        if (target >= pre && target < pre + mine) {
          s_go = 1;
          s.acc = target - pre;
        }
      }
    }
    __syncthreads();
    if (s_go) {
      const float mx = q.mx;
      const uint64_t t = s.acc;
      if (ph.phase == kPhPick) {
        uint64_t cs = 0;
        for (int i = c0; i < c1; ++i) cs += fix_of(R::x(row, i), mx, sc);
        uint64_t S;
        const uint64_t pre = block_scan(cs, s.scan, &S);
        if (t >= pre && t < pre + cs) {
          uint64_t acc = pre;
          for (int i = c0; i < c1; ++i) {
            acc += fix_of(R::x(row, i), mx, sc);
            if (t < acc) {
              s.tok = a.vocab_begin + i;
              break;
            }
          }
        }
      } else {
        const uint32_t w = q.w;
        uint64_t n = 0;
        for (int i = c0; i < c1; ++i) n += (R::key(row, i) == w);
        uint64_t tot;
        const uint64_t tpre = block_scan(n, s.scan, &tot);
        if (t >= tpre && t < tpre + n) {
          uint64_t c = tpre;
          for (int i = c0; i < c1; ++i)
            if (R::key(row, i) == w) {
              if (c == t) {
                s.tok = a.vocab_begin + i;
                break;
              }
              ++c;
            }
        }
      }
    }
    __syncthreads();
    if (threadIdx.x == 0) at<int>(sd, (size_t)r * 4) = s.tok;
    return;
  }

  // ---- nucleus radix phases: decide from the gathered tables, then bucket this level ----
  if (threadIdx.x == 0) {
    s_go = q.sel;
    if (ph.phase == kPhRadix && ph.walk_b && !q.walk_b) s_go = 0;
    if (ph.phase == kPhTie) s_go = q.sel;
  }
  __syncthreads();
  const bool go = s_go != 0;
  // the previous level's decision needs the summed tables of all ranks
  const bool decide = go && ph.phase != kPhRadixA0 &&
                      !(ph.phase == kPhTie && !q.walk_b);
  if (decide) {
    for (int b = threadIdx.x; b < 256; b += kST) {
      unsigned c = 0;
      unsigned long long sm = 0;
      for (int kk = 0; kk < a.nranks; ++kk) {
        const size_t base = (size_t)kk * ph.stride + (size_t)r * kBucketBytes;
        c += at<unsigned>(rv, base + (size_t)b * 4);
        sm += at<unsigned long long>(rv, base + 1024 + (size_t)b * 8);
      }
      s.cnt[b] = c;
      s.sum[b] = sm;
    }
    __syncthreads();
  }
  if (threadIdx.x == 0 && go) {
    const float mx = q.mx;
    if (ph.phase == kPhRadixA0) {
      uint64_t tot = 0;
      for (int kk = 0; kk < a.nranks; ++kk)
        tot += at<unsigned long long>(rv, (size_t)kk * ph.stride + (size_t)r * 8);
      q.S = tot;
      q.TA = (uint64_t)ceil((double)a.top_p * (double)tot);
      q.prefix = 0u;
      q.pmask = 0u;
      q.acc = 0ull;
    } else if (decide) {
      const int lvl = ph.phase == kPhRadix ? ph.shift + 8 : 0;  // AB / Tie: the last level
      const bool wb = ph.phase == kPhRadix ? ph.walk_b != 0 : ph.phase == kPhTie;
      const RadixPick p = radix_pick(s.cnt, s.sum, wb ? q.TB : q.TA, !wb, q.prefix, lvl, q.acc);
      q.prefix = p.key;
      q.acc = p.acc;
      q.n = p.n;
      q.pmask |= 0xFFu << lvl;
    }
    if (ph.phase == kPhAB) {
      q.vstar = q.prefix;
      q.acc_a = q.acc;
      q.n_eq = q.n;
      const uint64_t q_star = fix_of(R::x_of_key(q.vstar), mx, sc);
      uint64_t j, total;
      nucleus_cut(q.TA, q.acc_a, q.n_eq, q_star, &j, &total);
      q.j = j;
      q.total = total;
      q.TB = (uint64_t)((double)a.u[r] * (double)total);
      q.walk_b = q.TB < q.acc_a;
      q.prefix = 0u;
      q.pmask = 0u;
      q.acc = 0ull;
    }
    if (ph.phase == kPhTie) {
      if (q.walk_b) {
        q.w = q.prefix;
        q.i_tie = tie_index(q.TB, q.acc, fix_of(R::x_of_key(q.w), mx, sc), q.n);
      } else {
        q.w = q.vstar;
        q.i_tie = tie_index(q.TB, q.acc_a, fix_of(R::x_of_key(q.vstar), mx, sc), q.j);
      }
    }
    s_go = ph.phase == kPhAB ? (int)q.walk_b : 1;
  }
  __syncthreads();
  const bool emit = go && s_go;

  if (ph.phase == kPhTie) {
    uint64_t n = 0;
    if (emit) {
      const uint32_t w = q.w;
      for (int i = c0; i < c1; ++i) n += (R::key(row, i) == w);
    }
    uint64_t tot;
    block_scan(n, s.scan, &tot);
    if (threadIdx.x == 0) at<unsigned long long>(sd, (size_t)r * 8) = emit ? tot : 0ull;
    return;
  }

  // bucket table of level ph.shift (zeros when this row has nothing to walk)
  const size_t base = (size_t)r * kBucketBytes;
  if (emit) {
    const bool above = ph.phase == kPhAB || (ph.phase == kPhRadix && ph.walk_b);
    radix_buckets<R>(s, row, c0, c1, q.prefix, q.pmask, ph.shift, above, q.vstar, q.mx, sc);
  }
  for (int b = threadIdx.x; b < 256; b += kST) {
    at<unsigned>(sd, base + (size_t)b * 4) = emit ? s.cnt[b] : 0u;
    at<unsigned long long>(sd, base + 1024 + (size_t)b * 8) = emit ? s.sum[b] : 0ull;
  }
}

// Own rows: the token of each row the commit rule picked (the one rank that found it).
__global__ void shard_sample_finish(ShardSampleArgs a, size_t stride) {
  const int own = a.hdr[4 * a.me + 1];
  for (int j = threadIdx.x; j < own; j += blockDim.x) {
    const int r = a.me * a.rmax + j;
    if (!a.state[r].sel) continue;
    int tok = -1;
    for (int kk = 0; kk < a.nranks; ++kk)
      tok = max(tok, at<int>(a.xrecv, (size_t)kk * stride + (size_t)r * 4));
    a.tokens[j] = tok < 0 ? 0 : tok;
  }
}

size_t pad16(size_t b) { return (b + 15) / 16 * 16; }

}  // namespace

Status run_sample(const SampleArgs& a, cudaStream_t st) {
  WEDLM_CHECK_ARG(a.logits && a.tokens, "logits and tokens are required");
  WEDLM_CHECK_ARG(a.dtype == WEDLM_BF16 || a.dtype == WEDLM_F32, "logits dtype must be F32 or BF16");
  WEDLM_CHECK_ARG(a.rows >= 0 && a.V > 0 && a.ld >= a.V, "bad rows / V / ld");
  WEDLM_CHECK_ARG(a.temperature > 0.f && std::isfinite(a.temperature), "temperature must be > 0");
  WEDLM_CHECK_ARG(a.top_p > 0.f, "top_p must be > 0");
  WEDLM_CHECK_ARG(a.u || (a.nseq >= 1 && a.seq_rows && a.selected && a.n_selected && a.seq_key &&
                          a.seq_step),
                  "either draws u or the selection (seq_rows, selected, n_selected, keys, steps)");
  if (a.rows == 0) return Status::ok();
  if (a.dtype == WEDLM_BF16)
    sample_kernel<__nv_bfloat16><<<a.rows, kST, 0, st>>>(a);
  else
    sample_kernel<float><<<a.rows, kST, 0, st>>>(a);
  WEDLM_CUDA_TRY(cudaGetLastError());
  return Status::ok();
}

size_t shard_sample_xbytes(int rows, int rmax, bool nucleus) {
  size_t b = pad16(((size_t)rows + rmax) * 4);
  b = std::max(b, pad16((size_t)rows * 8));
  if (nucleus) b = std::max(b, pad16((size_t)rows * kBucketBytes));
  return b;
}

Status run_shard_sample(const ShardSampleArgs& a, const ShardGather& g, cudaStream_t st) {
  WEDLM_CHECK_ARG(a.logits && a.tokens && a.hdr && a.u && a.state && a.xsend && a.xrecv && g.fn,
                  "sharded sampling: missing buffers");
  WEDLM_CHECK_ARG(a.dtype == WEDLM_BF16 || a.dtype == WEDLM_F32, "logits dtype must be F32 or BF16");
  WEDLM_CHECK_ARG(a.nranks >= 1 && a.me >= 0 && a.me < a.nranks && a.rmax >= 1, "bad ranks / rows");
  WEDLM_CHECK_ARG(a.V > 0 && a.ld >= a.V && a.vocab_begin >= 0 && a.vocab_begin + a.V <= a.V_total,
                  "bad shard");
  WEDLM_CHECK_ARG(a.temperature > 0.f && std::isfinite(a.temperature), "temperature must be > 0");
  WEDLM_CHECK_ARG(a.top_p > 0.f, "top_p must be > 0");
  const int rows = a.nranks * a.rmax;
  const bool nucleus = a.top_p < 1.f;
  const int bits = a.dtype == WEDLM_BF16 ? 16 : 32;
  auto kern = a.dtype == WEDLM_BF16 ? shard_sample_kernel<__nv_bfloat16> : shard_sample_kernel<float>;
  size_t stride = 0;
  auto step = [&](int phase, int shift, int walk_b, size_t out_bytes) -> Status {
    ShardPhase ph;
    ph.phase = phase;
    ph.shift = shift;
    ph.walk_b = walk_b;
    ph.stride = stride;
    kern<<<rows, kST, 0, st>>>(a, ph);
    WEDLM_CUDA_TRY(cudaGetLastError());
    WEDLM_TRY(g.fn(g.user, a.xsend, a.xrecv, out_bytes, st));
    stride = out_bytes;
    return Status::ok();
  };
  const size_t b_max = pad16(((size_t)rows + a.rmax) * 4), b_u64 = pad16((size_t)rows * 8),
               b_int = pad16((size_t)rows * 4), b_bkt = pad16((size_t)rows * kBucketBytes);
  WEDLM_TRY(step(kPhMax, 0, 0, b_max));
  WEDLM_TRY(step(kPhSum, 0, 0, b_u64));
  if (!nucleus) {
    WEDLM_TRY(step(kPhPick, 0, 0, b_int));
  } else {
    WEDLM_TRY(step(kPhRadixA0, bits - 8, 0, b_bkt));
    for (int sh = bits - 16; sh >= 0; sh -= 8) WEDLM_TRY(step(kPhRadix, sh, 0, b_bkt));
    WEDLM_TRY(step(kPhAB, bits - 8, 1, b_bkt));
    for (int sh = bits - 16; sh >= 0; sh -= 8) WEDLM_TRY(step(kPhRadix, sh, 1, b_bkt));
    WEDLM_TRY(step(kPhTie, 0, 1, b_u64));
    WEDLM_TRY(step(kPhTiePick, 0, 1, b_int));
  }
  shard_sample_finish<<<1, 256, 0, st>>>(a, stride);
  WEDLM_CUDA_TRY(cudaGetLastError());
  return Status::ok();
}

}  // namespace wedlm
