// Model state: weights, paged KV cache, activation buffers and the forward pass.
#pragma once

#include "context.h"

namespace wedlm {

Status model_create(wedlm_ctx* ctx, const wedlm_config& cfg, int max_seqs, int max_ctx);
void model_destroy(wedlm_ctx* ctx);

}  // namespace wedlm
