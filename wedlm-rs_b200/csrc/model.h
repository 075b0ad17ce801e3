// Model state: weights, paged KV cache, activation buffers and the forward pass.
#pragma once

#include <string>
#include <vector>

#include "context.h"
#include "gemm.h"
#include "layer_ops.h"

namespace wedlm {

struct LayerWeights {
  void* wqkv = nullptr;   // [q_dim + 2 kv_dim, H]: q_proj rows, then k_proj, then v_proj
  void* wo = nullptr;     // [H, q_dim]
  void* wgate = nullptr;  // [I, H]
  void* wup = nullptr;    // [I, H]
  void* wdown = nullptr;  // [H, I]
  float* ln1 = nullptr;   // input_layernorm [H]
  float* ln2 = nullptr;   // post_attention_layernorm [H]
  float* qn = nullptr;    // q_norm [d]
  float* kn = nullptr;    // k_norm [d]
};

// One sequence's slice of a forward: `rows` window tokens written at cache slot `slot`
// starting at its committed length; logits for window rows [logit_begin, rows).
struct SeqSlice {
  int slot = 0;
  int rows = 0;
  int logit_begin = 0;
};

// Layout of the per-forward metadata (ints, device): R rows of B sequences.
struct MetaLayout {
  int tok, pos, rank, rslot, dst, rb, lsrc;  // [R] each: token, position, mask rank, cache
                                              // slot, cache row, sequence, logit-row source
  int s0, sr, sl, ss;                         // [B] each: first row, attention rows (window
                                              // length), committed cache length, cache slot
  int total;                                  // the fields above
  int act, total_dev;                         // [R] device loop only: 1 = a window row,
                                              // 0 = a padding row
  MetaLayout(int R, int B)
      : tok(0), pos(R), rank(2 * R), rslot(3 * R), dst(4 * R), rb(5 * R), lsrc(6 * R), s0(7 * R),
        sr(7 * R + B), sl(7 * R + 2 * B), ss(7 * R + 3 * B), total(7 * R + 4 * B),
        act(7 * R + 4 * B), total_dev(8 * R + 4 * B) {}
};

// A forward whose metadata a device kernel wrote into the model's metadata buffer (the
// device-resident decode loop): B sequences of W rows each (row b * W + j), every row
// projected; the logit rows (lsrc) are the step's mask rows followed by padding rows.
// The attention plan is built on the device (plan_attention_tc_device) into attn_ws.
struct DeviceForward {
  int B = 0, W = 0;
  const int* len_bound = nullptr;  // host [B]: upper bounds of the cache lengths (profiler)
  float* attn_ws = nullptr;
  long attn_ws_floats = 0;
  int max_work = 0, max_comb = 0;
  int* counts = nullptr;           // device int[2]
};

struct ModelState {
  wedlm_config cfg{};
  int dt = WEDLM_BF16, esz = 2;
  int H = 0, I = 0, V = 0, nh = 0, nkv = 0, d = 0, group = 1, nlayers = 0;
  int qdim = 0, kvdim = 0, qkvdim = 0;
  int vlo = 0, vhi = 0, vshard = 0;
  float eps = 1e-6f;

  uint8_t* arena = nullptr;  // every weight in one allocation
  size_t arena_bytes = 0;
  void* embed = nullptr;
  void* lm_head = nullptr;
  float* final_norm = nullptr;
  std::vector<LayerWeights> layers;
  float* cos = nullptr;  // [max_pos, d/2] (rounded to the model dtype, rope.rs:94-95)
  float* sin = nullptr;

  // paged KV cache: K [L][pages][nkv][page][d], V [L][pages][nkv][d][page]
  int page_size = 64, pages_per_seq = 0, num_pages = 0, max_seqs = 0, max_ctx = 0;
  void* kcache = nullptr;
  void* vcache = nullptr;
  int* page_table = nullptr;
  std::vector<int> cache_len;     // committed length per slot
  std::vector<int> pending_rows;  // rows written by the last forward, per slot

  // activations, capacity max_rows token rows
  int max_rows = 0;
  void *h = nullptr, *xn = nullptr, *qkv = nullptr, *q = nullptr, *attn = nullptr,
       *act = nullptr, *xl = nullptr;
  // per-forward metadata (device) and its pinned host staging
  int* d_meta = nullptr;
  int* h_meta = nullptr;
  size_t meta_ints = 0;
  float* slots = nullptr;  // split-K partial sets of the layer GEMMs (bf16)
  long slot_floats = 0;
  unsigned* sync = nullptr;  // grid-wide dependency counters of the fused layer tails
  int sync_count = 0;        // [layers][8]
  float* attn_ws = nullptr;
  long attn_ws_floats = 0;
  void* h_attn_staging = nullptr;
  size_t attn_staging_bytes = 0;
  cudaStream_t stream = nullptr;  // internal stream (NULL-stream calls use it)
};

Status model_create(wedlm_ctx* ctx, const wedlm_config& cfg, int max_seqs, int max_ctx);
// Checkpoint names of every tensor the model needs (safetensors / Hugging Face naming).
std::vector<std::string> model_weight_names(const ModelState* m);
void model_destroy(wedlm_ctx* ctx);

// Forward of a batch of windows.  tokens / positions / rank are host arrays over all
// rows (sequence-major).  Writes the window K/V at each slot's committed length (not
// committed) and, when logits != NULL, the logits of every sequence's rows
// [logit_begin, rows) densely to logits ([n, vshard], dtype logits_dtype).
// When hidden_out != NULL the LM head is not run: the final-normed hidden rows of the
// logit rows are written densely to hidden_out ([n, H], model dtype) instead.
Status model_forward(wedlm_ctx* ctx, const std::vector<SeqSlice>& seqs, const int* tokens,
                     const int* positions, const int* rank, void* logits, int logits_dtype,
                     int* n_logit_rows, cudaStream_t st, void* hidden_out = nullptr);

// The forward of a DeviceForward step: logits [B * W, vshard] (rows in lsrc order).  Every
// launch's shape is fixed by (B, W): the step can be captured in a CUDA graph once the
// scratch buffers have grown to it.
Status model_forward_device(wedlm_ctx* ctx, const DeviceForward& df, void* logits,
                            int logits_dtype, cudaStream_t st);

// The LM head alone (this context's vocabulary shard) over M final-normed hidden rows
// x ([M, ldx], model dtype, device): logits [M, vshard] of dtype logits_dtype.
Status model_lm_head(wedlm_ctx* ctx, const void* x, long ldx, int M, void* logits,
                     int logits_dtype, cudaStream_t st);

}  // namespace wedlm
