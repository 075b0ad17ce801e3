/*
 * wedlm_b200_kernels.h -- kernel-level entry points of libwedlm_b200.so.
 *
 * These expose single kernels of the decode step for tests, profiling and callers
 * that drive the forward pass themselves.  They have no counterpart in the reference
 * (whose kernels are candle ops); the conventions of wedlm_b200.h apply.
 */
#ifndef WEDLM_B200_KERNELS_H
#define WEDLM_B200_KERNELS_H

#include "wedlm_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Epilogues of wedlm_kernel_gemm. */
enum wedlm_gemm_epilogue {
  WEDLM_EPI_STORE = 0,       /* out = Y (model dtype)                            */
  WEDLM_EPI_STORE_F32 = 1,   /* out = Y (f32)                                    */
  WEDLM_EPI_RESIDUAL = 2,    /* out = resid + Y (bf16: rounded as the reference) */
  WEDLM_EPI_SWIGLU = 3       /* out = silu(X W^T) * (X W2^T)                     */
};

/* Y[m, n] = sum_k X[m, k] * W[n, k] (Linear::forward without bias) plus epilogue.
 * All pointers are device pointers of `dtype` (WEDLM_BF16: tcgen05 tensor cores,
 * K % 64 == 0, 16-byte aligned rows; WEDLM_F32: CUDA cores).  Row strides are in
 * elements.  `resid` may alias `out`.  w_layout 0: W (and W2) row-major with stride ldw;
 * w_layout 1 (bf16 only): W and W2 packed by wedlm_kernel_pack_weight. */
WEDLM_API int wedlm_kernel_gemm(wedlm_ctx* ctx, const void* X, int64_t ldx, const void* W,
                                const void* W2, int64_t ldw, int w_layout, int M, int N, int K,
                                int dtype, int epilogue, void* out, int64_t ldo,
                                const void* resid, int64_t ldr, void* stream);

/* Pack a row-major bf16 weight [N, K] (row stride ld, K % 64 == 0) into GEMM tiles:
 * `packed` (device, 16-byte aligned) must hold ceil(N / 128) * 128 * K elements; rows
 * past N are left as they are (zero them first).  Tile (n_tile, k-block) of 128 rows x
 * 64 columns is one contiguous 16 KB block holding the 128-byte-swizzled image the tensor
 * cores read, so the GEMM streams each pipeline stage with one sequential bulk copy. */
WEDLM_API int wedlm_kernel_pack_weight(wedlm_ctx* ctx, const void* W, int64_t ld, int N, int K,
                                       void* packed, void* stream);

/* Block attention of one S-row window against L cached tokens, the attention of the
 * decode step on caller buffers: softmax(Q K^T / sqrt(128) + mask) V with GQA
 * (src/model/attention.rs:188-221), every cached key visible and window key j visible
 * to window query i iff rank[j] <= rank[i] (rank = window index is the reference's
 * create_causal_mask, attention.rs:255-279; rank = position is causal over explicit
 * positions).  Tensor cores, head_dim 128, bf16.
 *   q     device bf16 [S, nh, 128]         queries after QK-norm and RoPE
 *   k, v  device bf16 [L + S, nkv, 128]    keys (after RoPE) and values: the L cached
 *                                          tokens, then the S window tokens
 *   rank  device int32 [S] or NULL (window index)
 * prepare copies them into the paged cache layout the model uses, inside the context,
 * and plans the split-KV work (1 <= S <= 4096, nh % nkv == 0, 128 % (nh / nkv) == 0);
 * run writes out (device bf16 [S, nh * 128], head h at column h * 128) and can be
 * repeated on the prepared inputs. */
WEDLM_API int wedlm_kernel_attention_prepare(wedlm_ctx* ctx, const void* q, const void* k,
                                             const void* v, int L, int S, int nh, int nkv,
                                             const int32_t* rank, void* stream);
WEDLM_API int wedlm_kernel_attention_run(wedlm_ctx* ctx, void* out, void* stream);

/* The T > 0 branches of sample_from_probs_at_indices (src/decoding/sampler.rs:160-200,
 * 306-351) on caller buffers, with the draw given: row r of softmax(logits / T) is
 * sampled with u[r] in [0, 1) (device f32 [rows]) and its token written to tokens[r]
 * (device int32 [rows]).  top_p >= 1: the first token whose running probability sum
 * exceeds u (sample_from_probs); top_p < 1: the nucleus, i.e. the most probable tokens
 * (ties in index order) until their sum reaches top_p, renormalised, then the same rule
 * in that order (sample_nucleus).  Sums are exact in 2^-40 fixed point, so a row and a
 * draw always give the same token.  temperature > 0. */
WEDLM_API int wedlm_kernel_sample(wedlm_ctx* ctx, const void* logits, int dtype, int rows, int V,
                                  int ld, float temperature, float top_p, const float* u,
                                  int32_t* tokens, void* stream);

/* Synchronises `stream`, then reports (and clears) a device-side wait that gave up
 * inside a kernel since the last check: WEDLM_ERR_TIMEOUT, else WEDLM_OK. */
WEDLM_API int wedlm_check_device_error(wedlm_ctx* ctx, void* stream);

/* Test of the bounded device wait (no counterpart in the reference, whose host code
 * has no device waits): launches one CTA whose consumer warp waits, with the helper the
 * tcgen05 kernels use, on an mbarrier phase that nothing completes (no arrival, no copy
 * in flight).  After limit_ns (0 < limit_ns <= 2e9) the wait gives up, records wait site
 * 1 in the context's error word and the kernel returns; wedlm_check_device_error then
 * reports WEDLM_ERR_TIMEOUT.  out: device int32[2] = {wait succeeded (0 expected),
 * microseconds waited}. */
WEDLM_API int wedlm_kernel_wait_probe(wedlm_ctx* ctx, int64_t limit_ns, int32_t* out,
                                      void* stream);

/* Kernel classes of the profiler. */
enum wedlm_kernel_class {
  WEDLM_KC_GEMM = 0,       /* projection GEMMs (tcgen05) incl. their shared-tile reduce */
  WEDLM_KC_ATTENTION = 1,  /* block attention incl. the split-KV combine               */
  WEDLM_KC_ENTROPY = 2,    /* fused entropy-select and the T > 0 sampling kernels       */
  WEDLM_KC_OTHER = 3,      /* embedding, RMSNorm, RoPE/KV append, row gather            */
  WEDLM_KC_COMM = 4        /* NCCL all-gathers of the vocabulary-sharded decode (not
                              kernels of this library: counted as 0 launches)          */
};

/* Time every launch of the model forward and the entropy stage with CUDA events on the
 * launching stream, per kernel class (on = 1 clears the totals).  Events sit between
 * launches, so keep it off for headline timings. */
WEDLM_API int wedlm_profile_enable(wedlm_ctx* ctx, int on);
/* Totals of class `cls` since profiling was enabled: device milliseconds, algorithmic
 * bytes and flops (the minimum a launch must move / compute), number of kernels. */
WEDLM_API int wedlm_profile_read(wedlm_ctx* ctx, int cls, double* ms, double* bytes,
                                 double* flops, int64_t* launches);
/* Kernels this context has launched for forwards and entropy passes so far. */
WEDLM_API int wedlm_launch_count(const wedlm_ctx* ctx, int64_t* out);

#ifdef __cplusplus
}
#endif

#endif /* WEDLM_B200_KERNELS_H */
