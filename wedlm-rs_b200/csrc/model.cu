// Model state and the block forward (filled in by the forward kernels).
#include "model.h"

namespace wedlm {

Status model_create(wedlm_ctx* ctx, const wedlm_config& cfg, int max_seqs, int max_ctx) {
  (void)ctx; (void)cfg; (void)max_seqs; (void)max_ctx;
  return Status::err(WEDLM_ERR_UNSUPPORTED, "model contexts are not built yet");
}

void model_destroy(wedlm_ctx* ctx) { (void)ctx; }

}  // namespace wedlm

extern "C" {

#define WEDLM_NOT_YET(ctx) \
  ((ctx) ? (ctx)->fail(wedlm::Status::err(WEDLM_ERR_UNSUPPORTED, "not built yet")) : WEDLM_ERR_INVALID_ARG)

int wedlm_set_weight(wedlm_ctx* ctx, const char*, const void*, int, const int64_t*, int) { return WEDLM_NOT_YET(ctx); }
int wedlm_init_random(wedlm_ctx* ctx, uint64_t, float) { return WEDLM_NOT_YET(ctx); }
int wedlm_get_weight(wedlm_ctx* ctx, const char*, void*, int64_t) { return WEDLM_NOT_YET(ctx); }
int wedlm_reset_sequence(wedlm_ctx* ctx, int) { return WEDLM_NOT_YET(ctx); }
int wedlm_cache_len(const wedlm_ctx* ctx, int, int32_t*) { return ctx ? WEDLM_ERR_UNSUPPORTED : WEDLM_ERR_INVALID_ARG; }
int wedlm_commit(wedlm_ctx* ctx, int, int) { return WEDLM_NOT_YET(ctx); }
int wedlm_truncate(wedlm_ctx* ctx, int, int) { return WEDLM_NOT_YET(ctx); }
int wedlm_prefill(wedlm_ctx* ctx, int, const int32_t*, int, void*) { return WEDLM_NOT_YET(ctx); }
int wedlm_block_forward(wedlm_ctx* ctx, int, const int32_t*, const int32_t*, const int32_t*,
                        const int32_t*, int, const int32_t*, void*, int, int32_t*, void*) {
  return WEDLM_NOT_YET(ctx);
}
int wedlm_generate_streaming(wedlm_ctx* ctx, int, const int32_t*, int, int, int,
                             const wedlm_sampling_params*, int32_t*, int32_t*, wedlm_block_stats*,
                             void*) {
  return WEDLM_NOT_YET(ctx);
}
int wedlm_generate_streaming_batch(wedlm_ctx* ctx, int, const int32_t*, int, int, int,
                                   const wedlm_sampling_params*, int32_t*, int32_t*, int64_t*,
                                   void*) {
  return WEDLM_NOT_YET(ctx);
}

}  // extern "C"
