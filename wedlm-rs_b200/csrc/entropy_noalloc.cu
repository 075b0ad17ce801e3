// Allocation-free form of the fused entropy-select entry point.
//
// wedlm_entropy_select keeps its scratch (per-split partial statistics, per-row
// entropies, per-sequence arrival counters) in context-owned device buffers that grow
// on demand, and growing them synchronises the device and calls cudaMalloc.  This
// entry point runs the same kernels with that scratch placed in a fixed file-scope
// __device__ array instead, so a call never allocates device memory, never frees it
// and makes no device-wide synchronisation.  The array's address is looked up once per
// device with cudaGetSymbolAddress.
#include <atomic>

#include "context.h"
#include "entropy_select.cuh"

using wedlm::Status;

namespace {

// Limits of the static scratch (each call is checked against them).
constexpr int kNoAllocMaxRows = 4096;        // mask rows per call
constexpr int kNoAllocMaxSeqs = 1024;        // sequences per call
constexpr int kNoAllocMaxRowSplits = 8192;   // rows x vocabulary splits per call
constexpr int kMaxDevices = 64;

// Layout (bytes): partials [kNoAllocMaxRowSplits][4] f32 | row_H [kNoAllocMaxRows] f32 |
// row_count [kNoAllocMaxRows] u32 | seq_count [kNoAllocMaxSeqs] u32.  Total 167,936 bytes.
constexpr size_t kPartialsOff = 0;
constexpr size_t kRowHOff = kPartialsOff + sizeof(float) * 4 * kNoAllocMaxRowSplits;
constexpr size_t kRowCountOff = kRowHOff + sizeof(float) * kNoAllocMaxRows;
constexpr size_t kSeqCountOff = kRowCountOff + sizeof(unsigned) * kNoAllocMaxRows;
constexpr size_t kScratchBytes = kSeqCountOff + sizeof(unsigned) * kNoAllocMaxSeqs;
static_assert(kRowHOff % 256 == 0 && kRowCountOff % 256 == 0 && kSeqCountOff % 256 == 0,
              "scratch sections stay aligned");
static_assert(kScratchBytes == 167936, "documented size");

// Static storage is zero when the module is loaded.  The row_count and seq_count sections
// must be zero before every launch: each launch's last CTA of a row (of a sequence) puts
// that counter back to zero, so the invariant holds from one call to the next.  The other
// sections are written before they are read within a launch.
static __device__ __align__(256) unsigned char g_entropy_scratch[kScratchBytes];

std::atomic<unsigned char*> g_scratch_addr[kMaxDevices];

// Device address of g_entropy_scratch on `device` (the current device), looked up once.
Status scratch_address(int device, unsigned char** out) {
  if (device < 0 || device >= kMaxDevices)
    return Status::err(WEDLM_ERR_INVALID_ARG, "device ordinal outside the static scratch table");
  unsigned char* p = g_scratch_addr[device].load(std::memory_order_acquire);
  if (!p) {
    void* addr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&addr, g_entropy_scratch);
    if (e != cudaSuccess)
      return Status::err(WEDLM_ERR_CUDA,
                         std::string("cudaGetSymbolAddress(entropy scratch): ") +
                             cudaGetErrorString(e));
    p = static_cast<unsigned char*>(addr);
    g_scratch_addr[device].store(p, std::memory_order_release);
  }
  *out = p;
  return Status::ok();
}

}  // namespace

extern "C" int wedlm_entropy_select_noalloc(wedlm_ctx* ctx, const void* logits, int dtype,
                                            int rows, int V, int ld, float temperature,
                                            float tau, float lambda, int nseq,
                                            const int32_t* seq_rows, const int32_t* mask_pos,
                                            const int32_t* caps, float* H, int32_t* argmax,
                                            float* maxprob, int32_t* selected,
                                            int32_t* n_selected, void* stream) {
  if (!ctx) return WEDLM_ERR_INVALID_ARG;
  cudaError_t e = cudaSetDevice(ctx->device);
  if (e != cudaSuccess) return ctx->fail(Status::err(WEDLM_ERR_CUDA, cudaGetErrorString(e)));
  if (rows < 0 || V <= 0 || nseq < 1)
    return ctx->fail(Status::err(WEDLM_ERR_INVALID_ARG, "bad rows / V / nseq"));
  if (rows > kNoAllocMaxRows)
    return ctx->fail(Status::err(WEDLM_ERR_INVALID_ARG,
                                 "rows exceeds the static entropy scratch limit of 4096"));
  if (nseq > kNoAllocMaxSeqs)
    return ctx->fail(Status::err(WEDLM_ERR_INVALID_ARG,
                                 "nseq exceeds the static entropy scratch limit of 1024"));
  const wedlm::EntropyPlan p = wedlm::plan_entropy(rows, V, dtype, ctx->num_sms);
  if ((long)rows * p.splits > kNoAllocMaxRowSplits)
    return ctx->fail(Status::err(WEDLM_ERR_INVALID_ARG,
                                 "rows x vocabulary splits exceeds the static entropy scratch "
                                 "limit of 8192"));
  unsigned char* base = nullptr;
  Status s = scratch_address(ctx->device, &base);
  if (!s.good()) return ctx->fail(s);

  wedlm::EntropyScratch W;
  W.partials = reinterpret_cast<float*>(base + kPartialsOff);
  W.partial_capacity = 4L * kNoAllocMaxRowSplits;
  W.row_H = reinterpret_cast<float*>(base + kRowHOff);
  W.row_capacity = kNoAllocMaxRows;
  W.row_count = reinterpret_cast<unsigned*>(base + kRowCountOff);
  W.seq_count = reinterpret_cast<unsigned*>(base + kSeqCountOff);
  W.seq_capacity = kNoAllocMaxSeqs;

  wedlm::EntropyArgs A;
  A.logits = logits;
  A.dtype = dtype;
  A.rows = rows;
  A.V = V;
  A.ld = ld;
  A.temperature = temperature;
  A.tau = tau;
  A.lambda = lambda;
  A.nseq = nseq;
  A.seq_rows = seq_rows;
  A.mask_pos = mask_pos;
  A.caps = caps;
  A.H = H;
  A.argmax = argmax;
  A.maxprob = maxprob;
  A.selected = selected;
  A.n_selected = n_selected;
  s = wedlm::run_entropy_select(A, W, ctx->num_sms, (cudaStream_t)stream);
  return s.good() ? WEDLM_OK : ctx->fail(s);
}
