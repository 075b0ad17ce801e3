// The wedlm_ctx object behind the C ABI: device, model shape, weights, the paged KV
// cache, scratch buffers and the last error message.
#pragma once

#include <map>
#include <string>
#include <vector>

#include "common.cuh"
#include "entropy_select.cuh"

struct wedlm_ctx {
  int device = 0;
  int num_sms = 148;
  bool has_model = false;
  wedlm_config cfg{};
  int max_seqs = 0;
  int max_ctx = 0;
  std::string last_error;

  wedlm::EntropyScratch ent{};

  // model state lives in ModelState (model.cu); opaque here
  struct ModelState* model = nullptr;

  int fail(const wedlm::Status& s) {
    last_error = s.msg;
    return s.code;
  }
};

namespace wedlm {

// Grow the entropy scratch to hold `rows` rows, `nseq` sequences and `partial_floats`
// partial words.  Synchronises the device when it reallocates.
Status ensure_entropy_scratch(wedlm_ctx* ctx, int rows, int nseq, long partial_floats);
void free_entropy_scratch(wedlm_ctx* ctx);

}  // namespace wedlm
