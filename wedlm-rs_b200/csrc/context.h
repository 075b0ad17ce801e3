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
struct DecodeSession;
struct AttnKernelScratch;
struct Comm;
}

// Optional per-kernel-class timing with CUDA events on the launching stream
// (enabled around a measured region; the events are recorded between launches).
struct WedlmProfiler {
  enum { kGemm = 0, kAttention = 1, kEntropy = 2, kOther = 3, kComm = 4, kClasses = 5 };
  bool on = false;
  std::vector<cudaEvent_t> ev;
  struct Rec {
    int cls, e0, e1;
    double bytes, flops;
  };
  std::vector<Rec> pending;
  int next = 0;
  double ms[kClasses] = {}, bytes[kClasses] = {}, flops[kClasses] = {};
  int64_t launches[kClasses] = {};
};

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

  // kernels launched by this context (always counted) and the optional profiler
  int64_t launches = 0;
  WedlmProfiler prof;

  // model state (model.cu); opaque here
  wedlm::ModelState* model = nullptr;
  // step-wise streaming decode (decode.cu); at most one per context
  wedlm::DecodeSession* session = nullptr;
  // stand-alone block attention (attention_kernel.cu)
  wedlm::AttnKernelScratch* att = nullptr;
  // NCCL communicator of the vocabulary-sharded decode (comm.cu); NULL on one GPU
  wedlm::Comm* comm = nullptr;
  // seed of the T > 0 draws (sample.cu)
  unsigned long long sample_seed = 0;

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
void session_free(wedlm_ctx* ctx);
void free_attention_kernel_scratch(wedlm_ctx* ctx);
// Profiler: mark the start of a launch group; returns a handle (or -1 when off).
int prof_begin(wedlm_ctx* ctx, cudaStream_t st);
// End the group started by prof_begin: `nlaunch` kernels of class `cls` that moved
// `bytes` algorithmic bytes and did `flops` algorithmic flops.
void prof_end(wedlm_ctx* ctx, cudaStream_t st, int h, int cls, double bytes, double flops,
              int nlaunch);
// Fold completed event pairs into the totals (call after the stream synchronised).
void prof_collect(wedlm_ctx* ctx);

}  // namespace wedlm
