// Seeded T > 0 sampling of the selected mask rows (sample_from_probs / sample_nucleus,
// src/decoding/sampler.rs:306-351) with one 1024-thread CTA per row.
//
// p = softmax(x / T) is handled unnormalised as e_i = exp((x_i - max) / T) <= 1, held in
// 2^-40 fixed point: every sum below is an exact 64-bit integer sum, so the result does
// not depend on the order of the additions (the row's chunks, the warps, the shared
// memory atomics) and a row always samples the same token for the same draw.
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
// Draws: SplitMix64 (Steele, Lea and Flood, OOPSLA 2014) chained over (seed, sequence,
// step, row), 24 bits, the precision of rand's gen::<f32>().
#include <cmath>
#include <cstdint>

#include "sample.cuh"

namespace wedlm {

namespace {

constexpr int kST = 1024;
constexpr int kSW = kST / 32;
constexpr float kFix = 1099511627776.0f;  // 2^40

__device__ __forceinline__ uint64_t mix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

__device__ float draw(uint64_t seed, uint64_t seq, uint64_t step, uint64_t row) {
  uint64_t h = mix64(seed);
  h = mix64(h ^ seq);
  h = mix64(h ^ step);
  h = mix64(h ^ row);
  return (float)(h >> 40) * 5.9604644775390625e-08f;  // 2^-24
}

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
      u = draw(a.seed, (uint64_t)a.seq_key[lo], (uint64_t)a.seq_step[lo], (uint64_t)rel);
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
  auto fix = [&](float x) -> uint64_t { return __float2ull_rn(exp2f((x - mx) * sc) * kFix); };

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
  // Radix walk, MSB first, over the keys that match the bits decided so far and exceed
  // `floor_key` (when `above`): in each level the buckets are visited from the largest
  // key down, and the walk enters the bucket whose running sum first reaches `target`
  // (>= when `inclusive`, the nucleus cutoff; > otherwise, the draw).  Returns the final
  // key; s.acc = fixed-point sum of the members above it, s.n = members equal to it.
  auto walk = [&](uint64_t target, bool inclusive, bool above, uint32_t floor_key) {
    uint32_t prefix = 0, pmask = 0;
    uint64_t acc = 0;
    for (int shift = R::kBits - 8; shift >= 0; shift -= 8) {
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
        atomicAdd(&s.sum[b], (unsigned long long)fix(R::x(row, i)));
      }
      __syncthreads();
      if (threadIdx.x == 0) {
        int sel = -1, low = -1;
        uint64_t acc_low = 0;
        for (int b = 255; b >= 0; --b) {
          if (!s.cnt[b]) continue;
          const uint64_t nxt = acc + s.sum[b];
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
        s.key = prefix | ((uint32_t)sel << shift);
        s.acc = acc;
        s.n = s.cnt[sel];
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
  uint64_t j = n_eq;
  if (q_star > 0) {
    const uint64_t need = TA > acc_a ? TA - acc_a : 0;
    j = (need + q_star - 1) / q_star;
  }
  j = j < 1 ? 1 : (j > n_eq ? n_eq : j);
  const uint64_t total = acc_a + j * q_star;

  // the crossing of u * total in the nucleus
  const uint64_t TB = (uint64_t)((double)s.u * (double)total);
  uint32_t w;
  uint64_t i_tie;
  if (TB >= acc_a) {
    w = vstar;
    i_tie = q_star > 0 ? (TB - acc_a) / q_star : 0;
    if (i_tie > j - 1) i_tie = j - 1;
  } else {
    w = walk(TB, false, true, vstar);
    const uint64_t q_w = fix(R::x_of_key(w));
    i_tie = q_w > 0 ? (TB - s.acc) / q_w : 0;
    if (i_tie > (uint64_t)s.n - 1) i_tie = (uint64_t)s.n - 1;
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

}  // namespace wedlm
