// NCCL communicator of a context (the multi-GPU seam of the C ABI): unique id, init
// with a bounded wait, the vocabulary-shard table of the ranks, grouped all-gathers and
// the bounded stream wait used by the vocabulary-sharded decode step (decode.cu).
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstring>
#include <mutex>
#include <thread>
#include <type_traits>

#include "comm.h"
#include "context.h"
#include "model.h"

namespace wedlm {

namespace {

// The NCCL entry points used here, resolved from libnccl.so.2 at run time.
struct NcclApi {
  bool ok = false;
  std::string why;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*CommFinalize)(ncclComm_t) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*GroupStart)() = nullptr;
  ncclResult_t (*GroupEnd)() = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

const NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    // Prefer the NCCL already loaded in the process (one NCCL per process).
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_LOCAL);
    if (!h) {
      const char* e = dlerror();
      api.why = std::string("cannot load libnccl.so.2: ") + (e ? e : "unknown error");
      return;
    }
    bool all = true;
    auto sym = [&](auto& fn, const char* name) {
      fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
      if (!fn) {
        all = false;
        api.why = std::string("libnccl.so.2 lacks ") + name;
      }
    };
    sym(api.GetUniqueId, "ncclGetUniqueId");
    sym(api.CommInitRankConfig, "ncclCommInitRankConfig");
    sym(api.CommGetAsyncError, "ncclCommGetAsyncError");
    sym(api.CommAbort, "ncclCommAbort");
    sym(api.CommFinalize, "ncclCommFinalize");
    sym(api.CommDestroy, "ncclCommDestroy");
    sym(api.AllGather, "ncclAllGather");
    sym(api.GroupStart, "ncclGroupStart");
    sym(api.GroupEnd, "ncclGroupEnd");
    sym(api.GetErrorString, "ncclGetErrorString");
    api.ok = all;
  });
  return api;
}

Status nccl_err(ncclResult_t r, const char* what) {
  const NcclApi& a = nccl();
  std::string m = std::string(what) + ": " + (a.GetErrorString ? a.GetErrorString(r) : "error");
  return Status::err(r == ncclSystemError || r == ncclRemoteError ? WEDLM_ERR_IO : WEDLM_ERR_CUDA,
                     m);
}

using Clock = std::chrono::steady_clock;

}  // namespace

struct Comm {
  ncclComm_t comm = nullptr;
  int rank = 0, nranks = 1;
  int timeout_ms = 0;
  bool broken = false;
  std::vector<int> lo, hi;  // vocabulary shard of every rank
  int* dbuf = nullptr;      // small device buffer of the init exchange
};

int comm_rank(const Comm* c) { return c->rank; }
int comm_size(const Comm* c) { return c->nranks; }
int comm_shard_begin(const Comm* c, int r) { return c->lo[r]; }
int comm_shard_end(const Comm* c, int r) { return c->hi[r]; }

namespace {

// Abort the communicator after a failed or timed-out wait; later calls fail.
Status comm_fail(Comm* c, Status s) {
  if (!c->broken && c->comm) nccl().CommAbort(c->comm);
  c->comm = nullptr;
  c->broken = true;
  return s;
}

// Poll ncclCommGetAsyncError until the communicator leaves ncclInProgress.
Status wait_ready(Comm* c, const char* what) {
  const NcclApi& a = nccl();
  const auto deadline = Clock::now() + std::chrono::milliseconds(c->timeout_ms);
  for (;;) {
    ncclResult_t r = ncclSuccess;
    ncclResult_t q = a.CommGetAsyncError(c->comm, &r);
    if (q != ncclSuccess) return comm_fail(c, nccl_err(q, "ncclCommGetAsyncError"));
    if (r == ncclSuccess) return Status::ok();
    if (r != ncclInProgress) return comm_fail(c, nccl_err(r, what));
    if (Clock::now() > deadline)
      return comm_fail(c, Status::err(WEDLM_ERR_TIMEOUT,
                                      std::string(what) + ": no answer from the other ranks"));
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

}  // namespace

Status comm_all_gather(Comm* c, const GatherPiece* pieces, int n, cudaStream_t st) {
  if (c->broken) return Status::err(WEDLM_ERR_STATE, "the communicator was aborted");
  const NcclApi& a = nccl();
  ncclResult_t r = a.GroupStart();
  if (r != ncclSuccess) return comm_fail(c, nccl_err(r, "ncclGroupStart"));
  for (int i = 0; i < n; ++i) {
    const GatherPiece& p = pieces[i];
    const ncclDataType_t t = p.dtype == WEDLM_BF16  ? ncclBfloat16
                             : p.dtype == kCommInt32 ? ncclInt32
                                                     : ncclFloat32;
    r = a.AllGather(p.send, p.recv, p.count, t, c->comm, st);
    if (r != ncclSuccess && r != ncclInProgress) {
      a.GroupEnd();
      return comm_fail(c, nccl_err(r, "ncclAllGather"));
    }
  }
  r = a.GroupEnd();
  if (r == ncclInProgress) return wait_ready(c, "ncclAllGather");
  if (r != ncclSuccess) return comm_fail(c, nccl_err(r, "ncclGroupEnd"));
  return Status::ok();
}

Status comm_sync(Comm* c, cudaStream_t st) {
  if (c->broken) return Status::err(WEDLM_ERR_STATE, "the communicator was aborted");
  const NcclApi& a = nccl();
  const auto deadline = Clock::now() + std::chrono::milliseconds(c->timeout_ms);
  for (int spin = 0;; ++spin) {
    cudaError_t e = cudaStreamQuery(st);
    if (e == cudaSuccess) return Status::ok();
    if (e != cudaErrorNotReady) return Status::err(WEDLM_ERR_CUDA, cudaGetErrorString(e));
    ncclResult_t r = ncclSuccess;
    a.CommGetAsyncError(c->comm, &r);
    if (r != ncclSuccess && r != ncclInProgress)
      return comm_fail(c, nccl_err(r, "collective failed"));
    if (Clock::now() > deadline) {
      Status s = comm_fail(c, Status::err(WEDLM_ERR_TIMEOUT,
                                          "a collective of the decode step did not finish within "
                                          "the communicator timeout"));
      // The abort ends NCCL's kernels and this context's own waits are bounded, so the
      // stream drains; wait for it (bounded again) before the caller reuses its buffers.
      const auto drain = Clock::now() + std::chrono::milliseconds(c->timeout_ms);
      while (cudaStreamQuery(st) == cudaErrorNotReady && Clock::now() < drain)
        std::this_thread::sleep_for(std::chrono::microseconds(200));
      return s;
    }
    if (spin > 2000) std::this_thread::yield();
  }
}

void comm_free(wedlm_ctx* ctx) {
  Comm* c = ctx->comm;
  if (!c) return;
  if (c->comm && !c->broken) {
    const NcclApi& a = nccl();
    // Finalize flushes outstanding work; its wait is bounded like every other one and
    // aborts the communicator when it gives up.
    const ncclResult_t r = a.CommFinalize(c->comm);
    if (r == ncclSuccess || r == ncclInProgress) {
      if (wait_ready(c, "ncclCommFinalize").good()) a.CommDestroy(c->comm);
    } else {
      a.CommAbort(c->comm);
    }
  }
  cudaFree(c->dbuf);
  delete c;
  ctx->comm = nullptr;
}

}  // namespace wedlm

using wedlm::Status;

extern "C" {

int wedlm_comm_unique_id(void* out, int nbytes) {
  if (!out || nbytes < (int)sizeof(ncclUniqueId)) return WEDLM_ERR_INVALID_ARG;
  const wedlm::NcclApi& a = wedlm::nccl();
  if (!a.ok) return WEDLM_ERR_UNSUPPORTED;
  ncclUniqueId id;
  if (a.GetUniqueId(&id) != ncclSuccess) return WEDLM_ERR_IO;
  std::memcpy(out, &id, sizeof(id));
  return WEDLM_OK;
}

int wedlm_comm_init(wedlm_ctx* ctx, const void* unique_id, int rank, int nranks, int timeout_ms) {
  if (!ctx) return WEDLM_ERR_INVALID_ARG;
  if (!ctx->model) return ctx->fail(Status::err(WEDLM_ERR_STATE, "context has no model"));
  if (ctx->comm) return ctx->fail(Status::err(WEDLM_ERR_STATE, "context already has a communicator"));
  if (ctx->session)
    return ctx->fail(Status::err(WEDLM_ERR_STATE, "a decode session is active"));
  if (!unique_id || nranks < 1 || rank < 0 || rank >= nranks || timeout_ms <= 0)
    return ctx->fail(Status::err(WEDLM_ERR_INVALID_ARG, "bad unique id / rank / nranks / timeout"));
  const wedlm::NcclApi& a = wedlm::nccl();
  if (!a.ok) return ctx->fail(Status::err(WEDLM_ERR_UNSUPPORTED, a.why));
  cudaError_t e = cudaSetDevice(ctx->device);
  if (e != cudaSuccess) return ctx->fail(Status::err(WEDLM_ERR_CUDA, cudaGetErrorString(e)));

  auto* c = new wedlm::Comm();
  c->rank = rank;
  c->nranks = nranks;
  c->timeout_ms = timeout_ms;
  ncclUniqueId id;
  std::memcpy(&id, unique_id, sizeof(id));
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  ncclResult_t r = a.CommInitRankConfig(&c->comm, nranks, id, rank, &cfg);
  Status s = Status::ok();
  if (r != ncclSuccess && r != ncclInProgress) {
    s = wedlm::nccl_err(r, "ncclCommInitRankConfig");
    if (c->comm) a.CommAbort(c->comm);
    delete c;
    return ctx->fail(s);
  }
  s = wedlm::wait_ready(c, "ncclCommInitRankConfig");
  if (!s.good()) {
    delete c;
    return ctx->fail(s);
  }

  // Exchange (shard begin, shard end, V, hidden) and check that the shards tile [0, V).
  const wedlm::ModelState* m = ctx->model;
  cudaStream_t st = m->stream;
  const int mine[4] = {m->vlo, m->vhi, m->V, m->H};
  e = cudaMalloc(&c->dbuf, sizeof(int) * 4 * (nranks + 1));
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(c->dbuf, mine, sizeof(mine), cudaMemcpyHostToDevice, st);
  if (e != cudaSuccess) {
    s = wedlm::comm_fail(c, Status::err(WEDLM_ERR_CUDA, cudaGetErrorString(e)));
  } else {
    wedlm::GatherPiece p;
    p.send = c->dbuf;
    p.recv = c->dbuf + 4;
    p.count = 4;
    p.dtype = wedlm::kCommInt32;
    s = wedlm::comm_all_gather(c, &p, 1, st);
    if (s.good()) s = wedlm::comm_sync(c, st);
  }
  std::vector<int> all(4 * nranks);
  if (s.good()) {
    e = cudaMemcpy(all.data(), c->dbuf + 4, sizeof(int) * 4 * nranks, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) s = Status::err(WEDLM_ERR_CUDA, cudaGetErrorString(e));
  }
  if (s.good()) {
    c->lo.resize(nranks);
    c->hi.resize(nranks);
    int expect = 0;
    for (int q = 0; q < nranks && s.good(); ++q) {
      c->lo[q] = all[4 * q];
      c->hi[q] = all[4 * q + 1];
      if (all[4 * q + 2] != m->V || all[4 * q + 3] != m->H)
        s = Status::err(WEDLM_ERR_INVALID_ARG, "the ranks' models differ in vocabulary or hidden size");
      else if (c->lo[q] != expect || c->hi[q] <= c->lo[q])
        s = Status::err(WEDLM_ERR_INVALID_ARG,
                        "the ranks' vocab shards do not tile [0, V) in rank order");
      expect = c->hi[q];
    }
    if (s.good() && expect != m->V)
      s = Status::err(WEDLM_ERR_INVALID_ARG, "the ranks' vocab shards do not tile [0, V) in rank order");
  }
  if (!s.good()) {
    ctx->comm = c;
    wedlm::comm_free(ctx);
    return ctx->fail(s);
  }
  ctx->comm = c;
  return WEDLM_OK;
}

int wedlm_comm_destroy(wedlm_ctx* ctx) {
  if (!ctx) return WEDLM_ERR_INVALID_ARG;
  if (ctx->session)
    return ctx->fail(Status::err(WEDLM_ERR_STATE, "a decode session is active"));
  cudaSetDevice(ctx->device);
  wedlm::comm_free(ctx);
  return WEDLM_OK;
}

}  // extern "C"
