// The wedlm_ctx object behind the C ABI: device, model shape, weights, the paged KV
// cache, scratch buffers and the last error message.
#pragma once

#include <map>
#include <string>
#include <vector>

#include "common.cuh"
#include "entropy_select.cuh"

namespace wedlm {
struct ModelState;
}

struct wedlm_ctx {
  int device = 0;
  int num_sms = 148;
  bool has_model = false;
  wedlm_config cfg{};
  int max_seqs = 0;
  int max_ctx = 0;
  std::string last_error;

  wedlm::EntropyScratch ent{};

  // split-K GEMM workspace and the device error word of the bounded waits
  float* gemm_ws = nullptr;
  long gemm_ws_floats = 0;
  unsigned* gemm_counters = nullptr;
  int gemm_n_counters = 0;
  int* dev_err = nullptr;

  // model state (model.cu); opaque here
  wedlm::ModelState* model = nullptr;

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
// Grow the split-K workspace / tile counters (synchronises when it reallocates).
Status ensure_gemm_scratch(wedlm_ctx* ctx, long ws_floats, int counters);
void free_gemm_scratch(wedlm_ctx* ctx);
// Read and clear the device error word; a non-zero code means a bounded wait gave up.
Status check_device_error(wedlm_ctx* ctx, cudaStream_t st);

}  // namespace wedlm
