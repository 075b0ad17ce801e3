// Communicator of a context that takes part in a vocabulary-sharded decode (comm.cu).
//
// Each rank is one process driving one GPU.  The ranks' contexts hold the LM-head rows
// [vocab_shard_begin, vocab_shard_end) of their configs; together, in rank order, these
// tile [0, V).  NCCL is loaded at run time (dlopen of libnccl.so.2, the copy already in the
// process when there is one), so a context that never joins a communicator does not need
// it.  The communicator is non-blocking: every host wait on it polls the stream and
// ncclCommGetAsyncError and gives up after the communicator's timeout, aborting the
// communicator (which ends NCCL's kernels) and returning WEDLM_ERR_TIMEOUT.
#pragma once

#include <vector>

#include "common.cuh"

struct wedlm_ctx;

namespace wedlm {

struct Comm;

// One all-gather of a group: `count` elements of `dtype` (WEDLM_BF16, WEDLM_F32 or the
// int32 code below) from every rank's send into recv ([nranks, count], rank order).
constexpr int kCommInt32 = 100;
struct GatherPiece {
  const void* send = nullptr;
  void* recv = nullptr;
  size_t count = 0;
  int dtype = WEDLM_F32;
};

int comm_rank(const Comm* c);
int comm_size(const Comm* c);
// LM-head rows held by rank r.
int comm_shard_begin(const Comm* c, int r);
int comm_shard_end(const Comm* c, int r);
// Enqueue one NCCL group of all-gathers on `st`.
Status comm_all_gather(Comm* c, const GatherPiece* pieces, int n, cudaStream_t st);
// Wait for `st` with the communicator's timeout (see above).
Status comm_sync(Comm* c, cudaStream_t st);
void comm_free(wedlm_ctx* ctx);

}  // namespace wedlm
