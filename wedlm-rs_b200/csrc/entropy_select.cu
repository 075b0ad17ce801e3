// Fused vocab-wide entropy / argmax / max-prob pass plus the WeDLM commit rule.
//
// Replaces, on the device and in one read of the logits:
//   compute_entropies_with_probs     src/decoding/sampler.rs:125-154
//   sample_from_probs_at_indices     src/decoding/sampler.rs:160-200 (T = 0 branch)
//   select_by_entropy_with_distance  src/decoding/sampler.rs:446-493
//
// Per row the pass keeps the online-softmax state (m, s, u, idx) in log2 units:
//   z = x / T (x when T is 0 or 1), m = max z, t = (z - m) * log2(e),
//   s = sum 2^t, u = sum 2^t * t, idx = largest column holding the max.
// Then H = -sum p ln p = ln(2) * (log2 s - u / s) and max-prob = 1 / s.  Argmax over
// probabilities with `Iterator::max_by` (last maximum wins) equals argmax over z with
// ties resolved to the largest column, which is what idx tracks.
//
// Layout: grid = rows x splits CTAs; each CTA reduces one column range of one row to a
// partial.  The last CTA to finish within a sequence (an atomic counter per sequence,
// no waiting) combines that sequence's partials and applies the commit rule, so one
// launch does the whole stage.  The counters reset themselves for the next launch.
#include "common.cuh"
#include "entropy_select.cuh"

#include <cfloat>

namespace wedlm {

namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 4;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

struct Acc {
  float m;  // running max (units set by the caller)
  float s;  // sum 2^t
  float u;  // sum 2^t * t
  int idx;  // column of the max (largest on ties)
};

__device__ __forceinline__ void acc_init(Acc& a) {
  a.m = -FLT_MAX;
  a.s = 0.f;
  a.u = 0.f;
  a.idx = -1;
}

// Merge b into a; k converts a difference of maxima to log2 units.
__device__ __forceinline__ void acc_merge(Acc& a, const Acc& b, float k) {
  if (b.s <= 0.f) return;
  if (a.s <= 0.f) {
    a = b;
    return;
  }
  if (b.m > a.m || (b.m == a.m && b.idx > a.idx)) {
    // rebase a onto b's max
    float d = (a.m - b.m) * k;
    float f = fast_exp2(d);
    float s = fmaf(f, a.s, b.s);
    float u = fmaf(f, fmaf(d, a.s, a.u), b.u);
    a.m = b.m;
    a.idx = b.idx;
    a.s = s;
    a.u = u;
  } else {
    float d = (b.m - a.m) * k;
    float f = fast_exp2(d);
    a.s = fmaf(f, b.s, a.s);
    a.u = fmaf(f, fmaf(d, b.s, b.u), a.u);
  }
}

__device__ __forceinline__ Acc acc_shfl(const Acc& a, int o) {
  Acc b;
  b.m = __shfl_xor_sync(0xffffffffu, a.m, o);
  b.s = __shfl_xor_sync(0xffffffffu, a.s, o);
  b.u = __shfl_xor_sync(0xffffffffu, a.u, o);
  b.idx = __shfl_xor_sync(0xffffffffu, a.idx, o);
  return b;
}

__device__ __forceinline__ void acc_warp_reduce(Acc& a, float k) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    Acc b = acc_shfl(a, o);
    acc_merge(a, b, k);
  }
}

// Accumulate NV values x[0..NV) at columns col..col+NV-1.  `a` = invT * log2(e).
template <int NV>
__device__ __forceinline__ void acc_values(Acc& st, float& nb, const float* x, int col, float a) {
  float cm = x[0];
#pragma unroll
  for (int j = 1; j < NV; ++j) cm = fmaxf(cm, x[j]);
  if (cm >= st.m) {
    int j0 = 0;
#pragma unroll
    for (int j = 0; j < NV; ++j)
      if (x[j] == cm) j0 = j;
    st.idx = col + j0;
    if (cm > st.m) {
      if (st.s > 0.f) {
        float d = (st.m - cm) * a;
        float f = fast_exp2(d);
        st.u = f * fmaf(d, st.s, st.u);
        st.s = f * st.s;
      }
      st.m = cm;
      nb = -cm * a;
    }
  }
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    float t = fmaxf(fmaf(x[j], a, nb), -128.f);
    float e = fast_exp2(t);
    st.s += e;
    st.u = fmaf(e, t, st.u);
  }
}

__device__ __forceinline__ void unpack(const uint4& v, float (&x)[8]) {
  x[0] = bf16_lo(v.x); x[1] = bf16_hi(v.x);
  x[2] = bf16_lo(v.y); x[3] = bf16_hi(v.y);
  x[4] = bf16_lo(v.z); x[5] = bf16_hi(v.z);
  x[6] = bf16_lo(v.w); x[7] = bf16_hi(v.w);
}
__device__ __forceinline__ void unpack(const uint4& v, float (&x)[4]) {
  x[0] = __uint_as_float(v.x); x[1] = __uint_as_float(v.y);
  x[2] = __uint_as_float(v.z); x[3] = __uint_as_float(v.w);
}

// Reduce columns [c0, c1) of one row into st (raw-logit units for st.m).
template <typename T, bool kVec>
__device__ __forceinline__ void reduce_range(const T* __restrict__ row, int c0, int c1, float a,
                                             Acc& st) {
  float nb = 0.f;
  int c = c0;
  if (kVec) {
    constexpr int VEC = 16 / sizeof(T);
    const int nvec = (c1 - c0) / VEC;
    const uint4* p = reinterpret_cast<const uint4*>(row + c0);
    for (int base = 0; base < nvec; base += kThreads * kUnroll) {
      uint4 v[kUnroll];
#pragma unroll
      for (int k = 0; k < kUnroll; ++k) {
        int i = base + k * kThreads + threadIdx.x;
        if (i < nvec) v[k] = ld_stream_v4(p + i);
      }
#pragma unroll
      for (int k = 0; k < kUnroll; ++k) {
        int i = base + k * kThreads + threadIdx.x;
        if (i < nvec) {
          float x[VEC];
          unpack(v[k], x);
          acc_values<VEC>(st, nb, x, c0 + i * VEC, a);
        }
      }
    }
    c = c0 + nvec * VEC;
  }
  for (int i = c + threadIdx.x; i < c1; i += kThreads) {
    float x[1] = {to_f32(row[i])};
    acc_values<1>(st, nb, x, i, a);
  }
}

// CTA-wide merge; result valid in thread 0.
__device__ __forceinline__ Acc block_reduce(Acc st, float k) {
  __shared__ Acc sh[kThreads / 32];
  acc_warp_reduce(st, k);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) sh[w] = st;
  __syncthreads();
  if (w == 0) {
    Acc v;
    if (l < kThreads / 32) v = sh[l];
    else acc_init(v);
    acc_warp_reduce(v, k);
    st = v;
  }
  return st;
}

__device__ __forceinline__ Acc load_partial(const float* p) {
  float4 v = __ldcg(reinterpret_cast<const float4*>(p));
  Acc a;
  a.m = v.x;
  a.s = v.y;
  a.u = v.z;
  a.idx = __float_as_int(v.w);
  return a;
}

__device__ void commit_rule(int b, int r0, int r1, float tau, float lambda,
                            const int* __restrict__ mask_pos, const int* __restrict__ caps,
                            const float* row_H, int* selected, int* n_selected, float* running,
                            const int* running_idx);

// Combine partials of every row of sequence [r0, r1) (partial (r, k) at
// part + (r * rs + k * ks) * 4), write per-row results, then the commit rule.
// Runs on one whole CTA of kThreads threads.
__device__ void finalize_sequence(int b, int r0, int r1, const float* part, long rs, long ks,
                                  int nk, float tau, float lambda, const int* __restrict__ mask_pos,
                                  const int* __restrict__ caps, float* row_H, float* H,
                                  int* argmax, float* maxprob, int* selected, int* n_selected,
                                  float* running, const int* running_idx) {
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  for (int r = r0 + w; r < r1; r += kThreads / 32) {
    Acc st;
    acc_init(st);
    for (int k = l; k < nk; k += 32) {
      Acc p = load_partial(part + ((long)r * rs + (long)k * ks) * 4);
      acc_merge(st, p, kLog2e);
    }
    acc_warp_reduce(st, kLog2e);
    if (l == 0) {
      float h = kLn2 * (log2f(st.s) - st.u / st.s);
      row_H[r] = h;
      if (H) H[r] = h;
      if (argmax) argmax[r] = st.idx;
      if (maxprob) maxprob[r] = 1.f / st.s;
    }
  }
  __syncthreads();
  __threadfence_block();
  commit_rule(b, r0, r1, tau, lambda, mask_pos, caps, row_H, selected, n_selected, running,
              running_idx);
}

// The commit rule of sequence b over its rows' entropies row_H[r0 .. r1): entropy EMA and
// dynamic cap, then select_by_entropy_with_distance (sampler.rs:446-493).  One whole CTA.
// The positions and entropies are staged in shared memory (sequences up to kRuleRows
// rows; longer ones read them from global memory).
constexpr int kRuleRows = 1024;
__device__ void commit_rule(int b, int r0, int r1, float tau, float lambda,
                            const int* __restrict__ mask_pos, const int* __restrict__ caps,
                            const float* row_H, int* selected, int* n_selected, float* running,
                            const int* running_idx) {
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  const int M = r1 - r0;
  __shared__ int s_pos[kRuleRows];
  __shared__ float s_adj[kRuleRows];
  __shared__ float s_h[kRuleRows];
  const bool staged = M <= kRuleRows;
  if (staged)
    for (int i = threadIdx.x; i < M; i += kThreads) {
      s_pos[i] = mask_pos[r0 + i];
      s_h[i] = __ldcg(row_H + r0 + i);
    }
  __syncthreads();
  auto pos_of = [&](int i) { return staged ? s_pos[i] : mask_pos[r0 + i]; };
  auto h_of = [&](int i) { return staged ? s_h[i] : __ldcg(row_H + r0 + i); };
  __shared__ int sh_i[kThreads / 32];
  __shared__ float sh_f[kThreads / 32];
  __shared__ int sh_r[kThreads / 32];
  // leftmost = min logical position
  int mn = INT_MAX;
  for (int i = threadIdx.x; i < M; i += kThreads) mn = min(mn, pos_of(i));
  mn = warp_min_i(mn);
  if (l == 0) sh_i[w] = mn;
  __syncthreads();
  if (threadIdx.x == 0) {
    int v = sh_i[0];
    for (int k = 1; k < kThreads / 32; ++k) v = min(v, sh_i[k]);
    sh_i[0] = v;
  }
  __syncthreads();
  const int leftmost = sh_i[0];
  __shared__ int sh_cap;
  if (threadIdx.x == 0) {
    int cap0 = caps[b];
    if (running != nullptr && M > 0) {
      // entropy EMA and dynamic cap, f32 in the reference's operation order
      // (wedlm.rs:517-535): sequential sum, mean, 0.3 * mean + (1 - 0.3) * r
      float sum = 0.f;
      for (int i = 0; i < M; ++i) sum = __fadd_rn(sum, h_of(i));
      const float mean = __fdiv_rn(sum, (float)M);
      const float a = 0.3f;
      const int ri = running_idx ? running_idx[b] : b;
      const float r = __fadd_rn(__fmul_rn(a, mean), __fmul_rn(__fsub_rn(1.f, a), running[ri]));
      running[ri] = r;
      if (r < __fmul_rn(tau, 0.4f)) cap0 = cap0 * 2;
      else if (r < __fmul_rn(tau, 0.7f)) cap0 = (cap0 * 3 + 1) / 2;
    }
    sh_cap = cap0;
  }
  if (staged)
    for (int i = threadIdx.x; i < M; i += kThreads)
      s_adj[i] = __fadd_rn(s_h[i], __fmul_rn(lambda, (float)(s_pos[i] - leftmost)));
  __syncthreads();
  const int cap = sh_cap;
  int npass = 0;
  float best_adj = FLT_MAX;
  int best_rank = INT_MAX, best_i = -1;
  for (int i = threadIdx.x; i < M; i += kThreads) {
    const int pi = pos_of(i);
    const float adj_i =
        staged ? s_adj[i] : __fadd_rn(h_of(i), __fmul_rn(lambda, (float)(pi - leftmost)));
    const bool pass_i = adj_i < tau;
    // rank of row i in (logical position, row) order, and how many passing rows precede it
    int rank = 0, before = 0;
    if (staged) {
      // branch-free over shared memory
#pragma unroll 4
      for (int j = 0; j < M; ++j) {
        const int pj = s_pos[j];
        const int earlier = (pj < pi) | ((pj == pi) & (j < i));
        rank += earlier;
        before += earlier & (s_adj[j] < tau);
      }
    } else {
      for (int j = 0; j < M; ++j) {
        const int pj = mask_pos[r0 + j];
        const bool earlier = pj < pi || (pj == pi && j < i);
        if (earlier) {
          ++rank;
          const float adj_j = __fadd_rn(__ldcg(row_H + r0 + j), __fmul_rn(lambda, (float)(pj - leftmost)));
          before += (adj_j < tau);
        }
      }
    }
    if (pass_i) {
      ++npass;
      if (before < cap) selected[r0 + before] = i;
    }
    if (adj_i < best_adj || (adj_i == best_adj && rank < best_rank)) {
      best_adj = adj_i;
      best_rank = rank;
      best_i = i;
    }
  }
  npass = warp_sum_i(npass);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float a2 = __shfl_xor_sync(0xffffffffu, best_adj, o);
    int r2 = __shfl_xor_sync(0xffffffffu, best_rank, o);
    int i2 = __shfl_xor_sync(0xffffffffu, best_i, o);
    if (a2 < best_adj || (a2 == best_adj && r2 < best_rank)) {
      best_adj = a2;
      best_rank = r2;
      best_i = i2;
    }
  }
  __shared__ int sh_rank[kThreads / 32];
  __syncthreads();
  if (l == 0) {
    sh_i[w] = npass;
    sh_f[w] = best_adj;
    sh_r[w] = best_i;
    sh_rank[w] = best_rank;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int tot = 0;
    float ba = FLT_MAX;
    int br = INT_MAX, bi = -1;
    for (int k = 0; k < kThreads / 32; ++k) {
      tot += sh_i[k];
      if (sh_f[k] < ba || (sh_f[k] == ba && sh_rank[k] < br)) {
        ba = sh_f[k];
        br = sh_rank[k];
        bi = sh_r[k];
      }
    }
    int nsel = min(tot, max(cap, 0));
    if (nsel == 0 && M > 0) {
      selected[r0] = bi;
      nsel = 1;
    }
    n_selected[b] = nsel;
  }
}

__device__ __forceinline__ int find_seq(const int* __restrict__ seq_rows, int nseq, int row) {
  int lo = 0, hi = nseq - 1;
  while (lo < hi) {
    int mid = (lo + hi + 1) >> 1;
    if (seq_rows[mid] <= row) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

template <typename T, bool kVec>
__global__ void __launch_bounds__(kThreads)
entropy_select_kernel(const T* __restrict__ logits, int V, long ld, int splits, int split_cols,
                      float invT, float* __restrict__ part, unsigned* __restrict__ row_count,
                      unsigned* __restrict__ seq_count, int nseq, const int* __restrict__ seq_rows, const int* __restrict__ mask_pos,
                      const int* __restrict__ caps, float tau, float lambda,
                      float* __restrict__ row_H, float* H, int* argmax, float* maxprob,
                      int* selected, int* n_selected, float* running, const int* running_idx) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x / splits;
  const int split = blockIdx.x - row * splits;
  const int c0 = split * split_cols;
  const int c1 = min(V, c0 + split_cols);
  const T* rp = logits + (long)row * ld;
  if (blockIdx.x == 0) {
    // sequences without mask rows get no CTA; they select nothing (sampler.rs:452-454)
    for (int b = threadIdx.x; b < nseq; b += kThreads)
      if (seq_rows[b + 1] == seq_rows[b]) n_selected[b] = 0;
  }
  // rows past the last sequence's end: a launch sized for more rows than this step holds
  // (the device-resident decode loop launches its row capacity)
  if (row >= seq_rows[nseq]) return;
  const float a = invT * kLog2e;

  Acc st;
  acc_init(st);
  reduce_range<T, kVec>(rp, c0, c1, a, st);
  st = block_reduce(st, a);

  // Two-level finish, no waiting: the last CTA of a row merges the row's splits and
  // writes its statistics; the last row of a sequence to finish applies the commit rule.
  __shared__ int s_last, s_seq;
  if (threadIdx.x == 0) {
    int last = 1;
    if (splits > 1) {
      // partial in scaled units: m_scaled = m_raw * invT (st is in log2 units)
      float4 v = make_float4(st.m * invT, st.s, st.u, __int_as_float(st.idx));
      *reinterpret_cast<float4*>(part + ((long)row * splits + split) * 4) = v;
      __threadfence();
      last = (atomicAdd(row_count + row, 1u) + 1 == (unsigned)splits);
    }
    s_last = last;
  }
  __syncthreads();
  if (!s_last) return;
  if (splits > 1) {
    __threadfence();
    if (threadIdx.x < 32) {
      Acc m;
      acc_init(m);
      for (int k = threadIdx.x; k < splits; k += 32)
        acc_merge(m, load_partial(part + ((long)row * splits + k) * 4), kLog2e);
      acc_warp_reduce(m, kLog2e);
      if (threadIdx.x == 0) {
        st = m;
        row_count[row] = 0u;
      }
    }
  } else if (threadIdx.x == 0) {
    st.m *= invT;  // scaled units, as the merged partials
  }
  if (threadIdx.x == 0) {
    const float h = kLn2 * (log2f(st.s) - st.u / st.s);
    row_H[row] = h;
    if (H) H[row] = h;
    if (argmax) argmax[row] = st.idx;
    if (maxprob) maxprob[row] = 1.f / st.s;
    __threadfence();
    const int b = find_seq(seq_rows, nseq, row);
    const unsigned need = (unsigned)(seq_rows[b + 1] - seq_rows[b]);
    s_last = (atomicAdd(seq_count + b, 1u) + 1 == need);
    s_seq = b;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  const int b = s_seq;
  commit_rule(b, seq_rows[b], seq_rows[b + 1], tau, lambda, mask_pos, caps, row_H, selected,
              n_selected, running, running_idx);
  if (threadIdx.x == 0) seq_count[b] = 0u;
}

template <typename T, bool kVec>
__global__ void __launch_bounds__(kThreads)
entropy_partials_kernel(const T* __restrict__ logits, int V, long ld, int splits,
                        int split_cols, int vocab_offset, float invT, float* __restrict__ tmp,
                        unsigned* __restrict__ row_count, float* __restrict__ out) {
  const int row = blockIdx.x / splits;
  const int split = blockIdx.x - row * splits;
  const int c0 = split * split_cols;
  const int c1 = min(V, c0 + split_cols);
  const float a = invT * kLog2e;
  Acc st;
  acc_init(st);
  reduce_range<T, kVec>(logits + (long)row * ld, c0, c1, a, st);
  st = block_reduce(st, a);
  __shared__ int s_last;
  if (threadIdx.x == 0) {
    float4 v = make_float4(st.m * invT, st.s, st.u,
                           __int_as_float(st.idx < 0 ? -1 : st.idx + vocab_offset));
    *reinterpret_cast<float4*>(tmp + ((long)row * splits + split) * 4) = v;
    __threadfence();
    s_last = (atomicAdd(row_count + row, 1u) + 1 == (unsigned)splits);
  }
  __syncthreads();
  if (!s_last || threadIdx.x >= 32) return;
  __threadfence();
  Acc r;
  acc_init(r);
  for (int k = threadIdx.x; k < splits; k += 32)
    acc_merge(r, load_partial(tmp + ((long)row * splits + k) * 4), kLog2e);
  acc_warp_reduce(r, kLog2e);
  if (threadIdx.x == 0) {
    *reinterpret_cast<float4*>(out + (long)row * 4) =
        make_float4(r.m, r.s, r.u, __int_as_float(r.idx));
    row_count[row] = 0u;
  }
}

__global__ void __launch_bounds__(kThreads)
entropy_combine_kernel(const float* __restrict__ part, int nshards, long shard_stride,
                       const int* seq_rows, const int* mask_pos, const int* caps, float tau,
                       float lambda, float* row_H, float* H, int* argmax, float* maxprob,
                       int* selected, int* n_selected, float* running, const int* running_idx) {
  const int b = blockIdx.x;
  finalize_sequence(b, seq_rows[b], seq_rows[b + 1], part, 1, shard_stride, nshards, tau, lambda,
                    mask_pos, caps, row_H, H, argmax, maxprob, selected, n_selected, running,
                    running_idx);
}

int pick_splits(int rows, int V, int num_sms) {
  // No rows: no launch follows; one split keeps the plan's arithmetic defined.
  if (rows <= 0 || V <= 0) return 1;
  // Aim for >= 4 CTAs per SM in total, with >= 8K columns per CTA.
  int target = num_sms * 4;
  int splits = (target + rows - 1) / rows;
  int max_splits = (V + 8191) / 8192;
  splits = splits < 1 ? 1 : splits;
  splits = splits > max_splits ? max_splits : splits;
  return splits < 1 ? 1 : splits;
}

template <typename T>
cudaError_t launch_select(const EntropyArgs& A, const EntropyScratch& W, int splits,
                          int split_cols, float invT, bool vec, cudaStream_t st) {
  const dim3 grid((unsigned)(A.rows * splits));
  auto kern = vec ? entropy_select_kernel<T, true> : entropy_select_kernel<T, false>;
  return launch_pdl(kern, grid, dim3(kThreads), 0, st, (const T*)A.logits, A.V, A.ld, splits,
                    split_cols, invT, W.partials, W.row_count, W.seq_count, A.nseq, A.seq_rows,
                    A.mask_pos,
                    A.caps, A.tau, A.lambda, W.row_H, A.H, A.argmax, A.maxprob, A.selected,
                    A.n_selected, A.running, (const int*)A.running_idx);
}

template <typename T>
void launch_partials(const EntropyArgs& A, const EntropyScratch& W, int splits, int split_cols,
                     float invT, bool vec, int vocab_offset, float* out, cudaStream_t st) {
  dim3 grid((unsigned)(A.rows * splits));
  if (vec)
    entropy_partials_kernel<T, true><<<grid, kThreads, 0, st>>>(
        (const T*)A.logits, A.V, A.ld, splits, split_cols, vocab_offset, invT, W.partials,
        W.row_count, out);
  else
    entropy_partials_kernel<T, false><<<grid, kThreads, 0, st>>>(
        (const T*)A.logits, A.V, A.ld, splits, split_cols, vocab_offset, invT, W.partials,
        W.row_count, out);
}

float inv_temperature(float T) { return (T > 0.f && T != 1.f) ? (float)(1.0 / (double)T) : 1.f; }

}  // namespace

EntropyPlan plan_entropy(int rows, int V, int dtype, int num_sms) {
  EntropyPlan p;
  p.splits = pick_splits(rows, V, num_sms);
  const int vec = 16 / dtype_size(dtype);
  int cols = (V + p.splits - 1) / p.splits;
  cols = (cols + vec - 1) / vec * vec;
  p.split_cols = cols;
  p.splits = (V + cols - 1) / cols;
  return p;
}

Status check_entropy_args(const EntropyArgs& A) {
  WEDLM_CHECK_ARG(A.logits != nullptr || A.rows == 0, "logits is NULL");
  WEDLM_CHECK_ARG(A.dtype == WEDLM_F32 || A.dtype == WEDLM_BF16, "logits dtype must be F32 or BF16");
  WEDLM_CHECK_ARG(A.rows >= 0 && A.V > 0 && A.ld >= A.V, "bad rows / V / ld");
  return Status::ok();
}

Status run_entropy_select(const EntropyArgs& A, const EntropyScratch& W, int num_sms,
                          cudaStream_t st) {
  WEDLM_TRY(check_entropy_args(A));
  WEDLM_CHECK_ARG(A.nseq >= 1, "nseq must be >= 1");
  WEDLM_CHECK_ARG(A.n_selected != nullptr, "n_selected is required");
  if (A.rows == 0) {
    // no mask rows: every sequence selects nothing (the per-row outputs are empty)
    WEDLM_CUDA_TRY(cudaMemsetAsync(A.n_selected, 0, sizeof(int) * A.nseq, st));
    return Status::ok();
  }
  WEDLM_CHECK_ARG(A.seq_rows && A.mask_pos && A.caps && A.selected,
                  "seq_rows, mask_pos, caps, selected and n_selected are required");
  EntropyPlan p = plan_entropy(A.plan_rows > 0 ? A.plan_rows : A.rows, A.V, A.dtype, num_sms);
  WEDLM_CHECK_ARG((long)A.rows * p.splits * 4 <= W.partial_capacity, "entropy scratch too small");
  WEDLM_CHECK_ARG(A.rows <= W.row_capacity && A.nseq <= W.seq_capacity, "entropy scratch too small");
  const bool vec = ((uintptr_t)A.logits % 16 == 0) && ((A.ld * dtype_size(A.dtype)) % 16 == 0);
  const float invT = inv_temperature(A.temperature);
  if (A.dtype == WEDLM_BF16)
    WEDLM_CUDA_TRY(launch_select<__nv_bfloat16>(A, W, p.splits, p.split_cols, invT, vec, st));
  else
    WEDLM_CUDA_TRY(launch_select<float>(A, W, p.splits, p.split_cols, invT, vec, st));
  return Status::ok();
}

Status run_entropy_partials(const EntropyArgs& A, const EntropyScratch& W, int vocab_offset,
                            float* out, int num_sms, cudaStream_t st) {
  WEDLM_TRY(check_entropy_args(A));
  if (A.rows == 0) return Status::ok();  // nothing to reduce (the buffers may be empty)
  WEDLM_CHECK_ARG(out != nullptr, "partials output is NULL");
  EntropyPlan p = plan_entropy(A.rows, A.V, A.dtype, num_sms);
  WEDLM_CHECK_ARG((long)A.rows * p.splits * 4 <= W.partial_capacity, "entropy scratch too small");
  WEDLM_CHECK_ARG(A.rows <= W.row_capacity, "entropy scratch too small");
  const bool vec = ((uintptr_t)A.logits % 16 == 0) && ((A.ld * dtype_size(A.dtype)) % 16 == 0);
  const float invT = inv_temperature(A.temperature);
  if (A.dtype == WEDLM_BF16)
    launch_partials<__nv_bfloat16>(A, W, p.splits, p.split_cols, invT, vec, vocab_offset, out, st);
  else
    launch_partials<float>(A, W, p.splits, p.split_cols, invT, vec, vocab_offset, out, st);
  WEDLM_CUDA_TRY(cudaGetLastError());
  return Status::ok();
}

Status run_entropy_combine(const float* partials, int nshards, const EntropyArgs& A,
                           const EntropyScratch& W, cudaStream_t st, long shard_stride) {
  WEDLM_CHECK_ARG(partials != nullptr && nshards >= 1, "bad partials");
  WEDLM_CHECK_ARG(A.nseq >= 1 && A.seq_rows && A.mask_pos && A.caps && A.selected && A.n_selected,
                  "seq_rows, mask_pos, caps, selected and n_selected are required");
  WEDLM_CHECK_ARG(A.rows <= W.row_capacity, "entropy scratch too small");
  if (shard_stride <= 0) shard_stride = A.rows;
  WEDLM_CHECK_ARG(shard_stride >= A.rows, "shard stride shorter than the rows");
  entropy_combine_kernel<<<A.nseq, kThreads, 0, st>>>(partials, nshards, shard_stride, A.seq_rows,
                                                      A.mask_pos, A.caps, A.tau, A.lambda, W.row_H,
                                                      A.H, A.argmax, A.maxprob, A.selected,
                                                      A.n_selected, A.running, A.running_idx);
  WEDLM_CUDA_TRY(cudaGetLastError());
  return Status::ok();
}

}  // namespace wedlm
