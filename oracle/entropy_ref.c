/*
 * Plain-C restatement of the reference's CPU commit-rule stage.
 * TEST INFRASTRUCTURE ONLY (the checker and the timed CPU baseline), never linked
 * into the product library.
 *
 * Follows, row by row:
 *   compute_entropies_with_probs   src/decoding/sampler.rs:125-154
 *     scaled = logits / T iff T > 0 && T != 1; p = softmax(scaled) materialised as f32
 *     (candle softmax: max, exp(x - max), sum, divide); H = sum_{p > 0} -p * ln p with
 *     a sequential f32 sum.
 *   select_by_entropy_with_distance src/decoding/sampler.rs:446-493
 *   sample_from_probs_at_indices   src/decoding/sampler.rs:160-200, T = 0 branch:
 *     argmax over the f32 probabilities, last maximum wins (Iterator::max_by).
 * Rows are processed in parallel with POSIX threads (nthreads <= 0: all cores).
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

static float load(const void* base, int dtype, long i) {
  if (dtype == 0) return ((const float*)base)[i];
  uint32_t w = (uint32_t)((const uint16_t*)base)[i] << 16;
  float f;
  memcpy(&f, &w, 4);
  return f;
}

/* Entropy and greedy token for each row; probs scratch is one row per thread. */
static void row_pass(const void* logits, int dtype, long off, int V, float T, float* p,
                     float* H_out, int* tok_out) {
  const int scale = (T > 0.f && T != 1.f);
  const float invT = scale ? (float)(1.0 / (double)T) : 1.f;
  float m = -INFINITY;
  for (int i = 0; i < V; ++i) {
    float x = load(logits, dtype, off + i);
    if (scale) x *= invT;
    p[i] = x;
    if (x > m) m = x;
  }
  float s = 0.f;
  for (int i = 0; i < V; ++i) {
    p[i] = expf(p[i] - m);
    s += p[i];
  }
  for (int i = 0; i < V; ++i) p[i] = p[i] / s;
  float h = 0.f;
  for (int i = 0; i < V; ++i)
    if (p[i] > 0.f) h += -p[i] * logf(p[i]);
  *H_out = h;
  int best = 0;
  float bv = p[0];
  for (int i = 1; i < V; ++i)
    if (!(p[i] < bv)) { /* >= : last maximum wins */
      bv = p[i];
      best = i;
    }
  *tok_out = best;
}

static int select_rule(const float* H, const int* pos, int M, float tau, float lambda, int cap,
                       int* sel) {
  if (M <= 0) return 0;
  int leftmost = pos[0];
  for (int i = 1; i < M; ++i)
    if (pos[i] < leftmost) leftmost = pos[i];
  /* stable sort of row indices by logical position (insertion sort, M is small) */
  int* ord = (int*)malloc(sizeof(int) * M);
  float* adj = (float*)malloc(sizeof(float) * M);
  for (int i = 0; i < M; ++i) {
    volatile float d = (float)(pos[i] - leftmost);
    volatile float pen = lambda * d;
    adj[i] = H[i] + pen;
    int j = i;
    while (j > 0 && pos[ord[j - 1]] > pos[i]) {
      ord[j] = ord[j - 1];
      --j;
    }
    ord[j] = i;
  }
  int n = 0;
  for (int k = 0; k < M && n < cap; ++k)
    if (adj[ord[k]] < tau) sel[n++] = ord[k];
  if (n == 0) {
    int b = ord[0];
    for (int k = 1; k < M; ++k)
      if (adj[ord[k]] < adj[b]) b = ord[k];
    sel[n++] = b;
  }
  free(ord);
  free(adj);
  return n;
}

struct job {
  const void* logits;
  int dtype, V, rows, nthreads, tid;
  long ld;
  float T;
  float* H;
  int* tokens;
};

static void* worker(void* arg) {
  struct job* j = (struct job*)arg;
  float* p = (float*)malloc(sizeof(float) * (size_t)j->V);
  for (int r = j->tid; r < j->rows; r += j->nthreads)
    row_pass(j->logits, j->dtype, (long)r * j->ld, j->V, j->T, p, j->H + r, j->tokens + r);
  free(p);
  return NULL;
}

/* Returns 0.  H, tokens: [rows]; selected: [rows] (per-sequence blocks as in the CUDA
 * ABI); n_selected: [nseq]. */
int oracle_entropy_select(const void* logits, int dtype, int rows, int V, long ld, float T,
                          float tau, float lambda, int nseq, const int* seq_rows,
                          const int* mask_pos, const int* caps, float* H, int* tokens,
                          int* selected, int* n_selected, int nthreads) {
  if (nthreads <= 0) nthreads = (int)sysconf(_SC_NPROCESSORS_ONLN);
  if (nthreads > rows) nthreads = rows > 0 ? rows : 1;
  pthread_t th[256];
  struct job jobs[256];
  if (nthreads > 256) nthreads = 256;
  for (int t = 0; t < nthreads; ++t) {
    jobs[t] = (struct job){logits, dtype, V, rows, nthreads, t, ld, T, H, tokens};
    pthread_create(&th[t], NULL, worker, &jobs[t]);
  }
  for (int t = 0; t < nthreads; ++t) pthread_join(th[t], NULL);
  for (int b = 0; b < nseq; ++b) {
    int r0 = seq_rows[b], r1 = seq_rows[b + 1];
    n_selected[b] = select_rule(H + r0, mask_pos + r0, r1 - r0, tau, lambda, caps[b], selected + r0);
  }
  return 0;
}
