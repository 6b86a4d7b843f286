// C ABI of the GQA decode path (declared in include/gqa.h).
//
// The host side replaces the reference's clSetKernelArg/clEnqueueNDRangeKernel
// plumbing in gpu_decoder_layer_step (qwen_server.c:344-455) with argument
// validation, a split-KV plan and cudaLaunchKernelEx launches.  Errors are
// returned as gqa_status codes with a thread-local message; nothing exits.
#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <vector>

#include <cuda_bf16.h>

#include <nvtx3/nvToolsExt.h>

#include "gqa.h"
#include "gqa_common.cuh"
#include "gqa_merge.cuh"

namespace gqa {
size_t decode_smem_bytes();
cudaError_t prepare_decode_kernels();
cudaError_t launch_decode_split(const DecodeParams& p, int n_seq, bool fused, cudaStream_t st,
                                bool pdl, int variant);
int decode_variant_count();
int decode_variant_quant(int variant);
int decode_variant_grid_quant(int variant);
int phase_trace_read(unsigned long long* host, int max_records, bool reset);
int decode_grid_ctas_per_sm(int variant);
cudaError_t launch_combine(const CombineParams& c, int n_seq, cudaStream_t st, bool pdl);
cudaError_t launch_combine_wide(const CombineParams& c, int n_seq, cudaStream_t st, bool pdl);
cudaError_t launch_rope_append(float* qkv, long long qkv_stride, float* const* k_ptrs,
                               float* const* v_ptrs, float* k_base, float* v_base,
                               long long seq_stride, Lengths len, int t_max, int n_q, int n_kv,
                               const float* inv_freq, int* status, int n_seq, cudaStream_t st,
                               bool pdl);
cudaError_t launch_advance_pos(int* pos, int wrap_lo, int wrap_hi, cudaStream_t st, bool pdl);
cudaError_t launch_advance_lens(int* lens, int n, cudaStream_t st, bool pdl);
cudaError_t launch_fill_normal(float* dst, long long n, uint64_t key, long long offset,
                               int n_sm, cudaStream_t st);
cudaError_t prepare_prefill_kernels();
cudaError_t launch_prefill_rope_table(const float* inv_freq, float2* cs, int n_pos,
                                      cudaStream_t st);
cudaError_t launch_prefill(const float* qkv, long long seq_stride, int n_seq, int S, int n_q,
                           int n_kv, const float2* rope_cs, __nv_bfloat16* qimg,
                           __nv_bfloat16* kimg, __nv_bfloat16* vimg, float* const* k_caches,
                           float* const* v_caches, int t_max, float* out, int* status,
                           int* sched, int n_sm, cudaStream_t st);
int block_d_model(int model);
int block_d_ffn(int model);
int block_max_d_ffn();
cudaError_t prepare_block_kernels();
cudaError_t launch_gateup_gemv(int model, const void* w_gate, const void* w_up,
                               const float* gamma, const float* state, float* h, int* status,
                               cudaStream_t st, bool pdl);
cudaError_t launch_down_gemv(int model, const void* w_down, const float* h, float* state,
                             int* status, cudaStream_t st, bool pdl);
cudaError_t launch_qkv_gemv(int model, const void* w, const float* bias, const float* gamma,
                            const float* state, float* qkv, int M, int* status, cudaStream_t st,
                            bool pdl);
cudaError_t launch_wo_gemv(int model, const void* w, const float* attn, float* state, int M,
                           int* status, cudaStream_t st, bool pdl);
size_t exchange_inbox_bytes(int world, int n_rows);
cudaError_t launch_exchange_combine(const CombineParams& local, uint2* const* inbox,
                                    unsigned* epoch, int rank, int world, float* out, int* status,
                                    cudaStream_t st, bool pdl);
bool generic_shape_built(int head_dim, int group);
int generic_max_splits();
int generic_plan_splits(int n_kv, int plan_len, int n_sm);
cudaError_t launch_generic_attention(const float* qkv, float* out, float* k_cache, float* v_cache,
                                     Lengths len, int t_max, int n_q, int n_kv, int head_dim,
                                     int n_splits, int plan_len, const float* inv_freq,
                                     float* part_o, float* part_ml, int* status, cudaStream_t st,
                                     bool pdl_first, bool pdl, bool lengths_stable);
size_t lm_head_packed_bytes(long long n_rows);
size_t lm_head_q8_packed_bytes(long long n_rows);
cudaError_t launch_q8_pack(const void* src, int n_rows, void* dst, cudaStream_t st);
int lm_head_grid(int n_sm);
size_t lm_head_best_bytes(int grid);
cudaError_t launch_q6k_pack(const void* src, int n_rows, void* dst, cudaStream_t st);
cudaError_t prepare_head_kernels();
cudaError_t launch_lm_head(bool q8, const void* planes, int n_rows, const float* gamma,
                           const float* state, float* logits, int* token, void* best,
                           unsigned* done, int* status, int grid, cudaStream_t st, bool pdl);
cudaError_t launch_embed_q4(const void* table, int n_rows, int d_model, const int* token,
                            float* state, int* status, cudaStream_t st, bool pdl);
}  // namespace gqa

using namespace gqa;

constexpr int kMaxExchangeWorld = 32;  // = kExMaxWorld of the exchange kernel

// Peer-memory exchange group of one GPU (gqa_exchange_*).  The inbox is one
// allocation exported through CUDA IPC.
struct gqa_exchange {
  gqa_ctx* ctx = nullptr;  // compared, never dereferenced after creation
  int device = 0;
  int rank = 0, world = 1, n_rows = 0;
  void* base = nullptr;                    // local inbox
  cudaIpcMemHandle_t own{};                // handle of base
  void* peer[kMaxExchangeWorld] = {};      // mapped peer allocations (self: base)
  uint2** d_inbox = nullptr;               // device [world]
  unsigned* epoch = nullptr;               // device [n_rows] (exchange kernel's steps)
  unsigned* slice_epoch = nullptr;         // device [n_rows * kXSlices] (fused path's steps)
  bool opened = false;
};

struct gqa_ctx {
  int device = 0;
  int n_sm = 148;
  gqa_config cfg{};
  float h_inv_freq[kHalf];
  float* inv_freq = nullptr;  // device [64]
  int* status = nullptr;      // device
  float* part_o = nullptr;    // split scratch
  float* part_ml = nullptr;
  long long cap_slots = 0;    // (q row x split) slots the scratch holds
  int pdl = 0;
  int target_ctas = 0;
  int batch_chunk = 0;  // tokens per split in batched decode (0 = automatic)
  int batch_advance = 0;  // GQA_OPT_BATCH_ADVANCE: batched steps advance seq_lens
  int live_graphs = 0;  // graphs hold scratch pointers: no reallocation while > 0
  // Decode kernel shapes (csrc/gqa_decode.cu variant table).  Measured on
  // B200: one sequence (few long CTAs, latency-bound) runs best with 8 warps
  // x 8-row stages (variant 3); batches and long caches (many CTAs,
  // bandwidth-bound) with 8 warps x 4-row stages (variant 0).
  int variant = -1;     // -1: per path as above; otherwise forced (tuning knob)
  int layers_pdl = 1;   // programmatic dependent launch inside the layer loop
  // Cluster reduction for single-sequence launches.  Off by default: on B200
  // it measured slower than the separate combine kernel (cluster start skew
  // and ~1 us per dependent global round trip for the arrival counter and
  // the final merge).
  int cluster = 0;
  int* counters = nullptr;  // [kCounterSlots] arrival / item counters, kept at zero
  // Grid-merged single-sequence decode (one launch per layer call: the split
  // kernel's CTAs merge each other's epoch-tagged partials).  On by default;
  // off falls back to split kernel + combine kernel.
  int grid_merge = 1;
  int grid_ctas_per_sm = 0;                   // resident CTAs of the grid instance per SM
  int grid_ctas_per_sm_long = 0;              // the same for the long-range shape (variant 3)
  unsigned* grid_epoch = nullptr;             // [kGridEpochWords] per-KV-head launch epochs
  unsigned long long* grid_words = nullptr;   // tagged partials [n_q][kGridMaxParts][row]
  float* blk_qkv = nullptr;   // attention block workspace: qkv of the token
  float* blk_attn = nullptr;  // attention block workspace: attention output
  float* blk_h = nullptr;     // FFN workspace: silu(gate) * up
  bool generic = false;       // a shape the tuned kernels are not built for (gqa_generic.cu)
  void* head_best = nullptr;  // LM head: per-CTA greedy picks
  int head_grid = 0;          // LM head CTAs
  __nv_bfloat16* prefill_img = nullptr;  // bf16 tile images for the prefill
  size_t prefill_cap = 0;                // elements
  float2* rope_cs = nullptr;             // prefill RoPE table [rope_cap][64] (cos, sin)
  int rope_cap = 0;                      // positions in the table
};

struct gqa_graph {
  gqa_ctx* ctx = nullptr;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  const float* d_qkv = nullptr;
  float* d_out = nullptr;
  size_t qkv_bytes = 0;
  size_t out_bytes = 0;
};

namespace {

thread_local char g_err[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

#define GQA_CUDA(call)                                                                  \
  do {                                                                                  \
    cudaError_t e_ = (call);                                                            \
    if (e_ != cudaSuccess)                                                              \
      return fail(GQA_ERR_CUDA, "%s failed: %s", #call, cudaGetErrorString(e_));      \
  } while (0)

// An NVTX range named after the API call, for the call's host-side extent
// (what a profiler or a tracing tool shows around the call's launches).
struct NvtxRange {
  explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
  ~NvtxRange() { nvtxRangePop(); }
  NvtxRange(const NvtxRange&) = delete;
  NvtxRange& operator=(const NvtxRange&) = delete;
};
#define GQA_RANGE(name) NvtxRange gqa_range_(name)

// Makes the context's device current for the duration of an API call.
struct DeviceGuard {
  int prev = -1;
  cudaError_t err = cudaSuccess;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev != dev) err = cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

constexpr int kCluster = 8;             // CTAs per cluster in the cluster reduction
constexpr int kMaxCounters = 1 << 16;   // (sequence, KV head) arrival counters
// Two counters past the decode range: the prefill's dynamic item counter and
// its CTA-done counter (both zero between launches).
constexpr int kPrefillSchedSlot = kMaxCounters;
// The LM head's CTA arrival counter (zero between launches).
constexpr int kHeadDoneSlot = kMaxCounters + 2;
constexpr int kCounterSlots = kMaxCounters + 3;

int ceil_div(long long a, long long b) { return (int)((a + b - 1) / b); }


bool is_capturing(cudaStream_t st) {
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(st, &cs) != cudaSuccess) return false;
  return cs != cudaStreamCaptureStatusNone;
}

// Grows the split scratch to hold `slots` (row, split) partials.
int ensure_scratch(gqa_ctx* c, long long slots, cudaStream_t st) {
  if (slots <= c->cap_slots) return GQA_OK;
  if (c->live_graphs > 0)
    return fail(GQA_ERR_NO_MEMORY,
                "split scratch too small (%lld slots needed, %lld held) and %d captured "
                "graph(s) still use it; call gqa_reserve() before creating graphs",
                slots, c->cap_slots, c->live_graphs);
  if (is_capturing(st))
    return fail(GQA_ERR_NO_MEMORY,
                "split scratch too small (%lld slots needed, %lld held) while the stream is "
                "being captured; call gqa_reserve() before capturing",
                slots, c->cap_slots);
  if (c->part_o) cudaFree(c->part_o);
  if (c->part_ml) cudaFree(c->part_ml);
  c->part_o = nullptr;
  c->part_ml = nullptr;
  c->cap_slots = 0;
  if (cudaMalloc(&c->part_o, sizeof(float) * kHeadDim * (size_t)slots) != cudaSuccess ||
      cudaMalloc(&c->part_ml, sizeof(float) * 2 * (size_t)slots) != cudaSuccess) {
    cudaGetLastError();
    return fail(GQA_ERR_NO_MEMORY, "cudaMalloc of %lld split slots failed", slots);
  }
  c->cap_slots = slots;
  return GQA_OK;
}

// Number of splits for a decode over `len` rows of `rows_kv` (sequence, KV
// head) pairs: enough CTAs to cover the device once, never a split shorter
// than 32 rows.
int single_variant(const gqa_ctx* c) { return c->variant >= 0 ? c->variant : 3; }
int batch_variant(const gqa_ctx* c) { return c->variant >= 0 ? c->variant : 0; }

int plan_splits_single(const gqa_ctx* c, int rows_kv, int len) {
  const int target = c->target_ctas > 0 ? c->target_ctas : c->n_sm;
  int want = ceil_div(target, rows_kv);
  const int most = ceil_div(len, decode_variant_quant(single_variant(c)));
  if (want > most) want = most;
  if (want > kMergeMaxParts) want = kMergeMaxParts;  // the merge's weight table
  return want < 1 ? 1 : want;
}

// The grid-merged kernel shape: the forced variant if it has a grid instance,
// else variant 0 (8 warps x 4-row stages; two CTAs fit on an SM, so the next
// layer's CTAs can become resident beside the running ones).
int grid_variant(const gqa_ctx* c) { return c->variant >= 0 ? c->variant : 0; }

// The grid-merged shape for `len` rows over n_splits splits: the forced variant,
// or 8 warps x 8-row stages (variant 3, one CTA per SM) once a warp has more
// than 16 rows to stream, else variant 0.  Measured: long1 (443 rows per CTA)
// 15.7 us per step with variant 3 against 18.9 with variant 0; resident28 (56
// rows per CTA) 163 us per step with variant 0 against 178 with variant 3.
int grid_variant_for(const gqa_ctx* c, long long len, int n_splits) {
  if (c->variant >= 0) return c->variant;
  const long long rows_per_warp = (len + (long long)n_splits * 8 - 1) / ((long long)n_splits * 8);
  return rows_per_warp > 16 && c->grid_ctas_per_sm_long >= 1 ? 3 : 0;
}

// Splits of a grid-merged single-sequence decode over `len` rows, or 0 when
// the grid merge cannot be used: at least 6 splits, at most kGridMaxParts,
// and every CTA of the launch resident at once (its mergers wait on the other
// CTAs): one CTA per SM.  (The next launch's CTAs are released only once all
// of this launch's are running, so they can never take a slot this launch
// still needs.  Two CTAs per SM of one launch measured slower: the second
// wave waits for the previous launch's CTAs to leave, and the merge waits
// for it.)
int plan_splits_grid(const gqa_ctx* c, int rows_kv, int len) {
  if (!c->grid_merge || c->generic || c->grid_ctas_per_sm < 1 || !c->grid_words ||
      rows_kv > kGridEpochWords)
    return 0;
  const int quant = decode_variant_grid_quant(grid_variant(c));
  const int per_sm = c->grid_ctas_per_sm >= 1 ? 1 : 0;
  const int cap = c->n_sm * per_sm;
  const int target = c->target_ctas > 0 && c->target_ctas < cap ? c->target_ctas : cap;
  int want = target / rows_kv;
  const int most = ceil_div(len, quant);
  if (want > most) want = most;
  if (want > kGridMaxParts) want = kGridMaxParts;
  return want >= 6 ? want : 0;
}

// Rows per split of a batched decode, by how many waves of CTAs the batch
// yields (a sequence's rows estimated at half the longest's): 1024 while that
// still gives two waves, else 512 while it gives 1.5, else 256 (a small batch
// needs the CTAs).  Measured, 64 sequences of U[256, 8192] rows plus a
// 256-step window dealt to 1/2/4/8 GPUs (one GPU's share, us per step):
// 1024 rows 99.8 / 52.3 / 47.3 / 45.5, 512 rows 105.9 / 55.0 / 30.1 / 27.8,
// 256 rows 112.7 / 60.9 / 33.8 / 20.0.
int batch_chunk(const gqa_ctx* c, int n_seq, int max_len) {
  const int q = decode_variant_quant(batch_variant(c));
  int want = c->batch_chunk;
  if (want <= 0) {
    const auto ctas = [&](int rows) {
      return (long long)n_seq * c->cfg.n_heads_kv * ceil_div(max_len, 2 * rows);
    };
    const long long sms = c->n_sm;
    want = ctas(1024) >= 2 * sms ? 1024 : 2 * ctas(512) >= 3 * sms ? 512 : 256;
  }
  const int least = ceil_div(max_len, kMergeMaxParts);  // at most kMergeMaxParts splits
  if (want < least) want = least;
  return ((want + q - 1) / q) * q;
}

DecodeParams base_params(gqa_ctx* c) {
  DecodeParams p{};
  p.t_max = c->cfg.t_max;
  p.n_kv = c->cfg.n_heads_kv;
  p.inv_freq = c->inv_freq;
  p.q_scale = (1.0f / sqrtf((float)kHeadDim)) * 1.4426950408889634f;
  p.status = c->status;
  p.part_o = c->part_o;
  p.part_ml = c->part_ml;
  p.min_chunk = decode_variant_quant(single_variant(c));
  p.lengths_stable = 1;
  return p;
}

CombineParams combine_from_scratch(const gqa_ctx* c, int n_splits) {
  CombineParams cp{};
  cp.m = c->part_ml;
  cp.l = c->part_ml + 1;
  cp.o = c->part_o;
  cp.ml_part_stride = 2;
  cp.ml_row_stride = 2LL * n_splits;
  cp.o_part_stride = kHeadDim;
  cp.o_row_stride = (long long)kHeadDim * n_splits;
  cp.n_parts = n_splits;
  cp.rows_per_seq = c->cfg.n_heads_q;
  return cp;
}

int check_kv(const gqa_ctx* c, const gqa_layer_kv* kv) {
  if (!kv || !kv->k_cache || !kv->v_cache) return fail(GQA_ERR_INVALID_ARG, "null KV cache");
  if (!aligned16(kv->k_cache) || !aligned16(kv->v_cache))
    return fail(GQA_ERR_INVALID_ARG, "KV cache pointers must be 16-byte aligned");
  (void)c;
  return GQA_OK;
}

// One sequence: split kernel (+ combine when split), result to `out`.  When
// the grid merge applies (and `grid_ok`), one launch does both.  The
// attention blocks pass grid_ok = false: between the projections the split
// kernel + combine measured faster (block28 332 vs 427 us per token, token28
// 802 vs 895 us).
int run_single(gqa_ctx* c, cudaStream_t st, const gqa_layer_kv* kv, const float* qkv,
               Lengths len, int plan_len, bool fused, float* out, bool pdl_first,
               bool lengths_stable, bool grid_ok = true) {
  const int n_kv = c->cfg.n_heads_kv;
  const int grid_splits =
      (grid_ok && fused && out != nullptr) ? plan_splits_grid(c, n_kv, plan_len) : 0;
  if (grid_splits > 0) {
    DecodeParams p = base_params(c);
    p.k_base = kv->k_cache;
    p.v_base = kv->v_cache;
    p.qkv = qkv;
    p.len = len;
    p.lengths_stable = lengths_stable ? 1 : 0;
    p.n_splits = grid_splits;
    const int gv = grid_variant_for(c, plan_len, grid_splits);
    p.min_chunk = decode_variant_grid_quant(gv);
    p.out = out;
    p.grid_epoch = c->grid_epoch;
    p.grid_words = c->grid_words;
    GQA_CUDA(launch_decode_split(p, 1, true, st, pdl_first, gv));
    return GQA_OK;
  }
  int n_splits = plan_splits_single(c, n_kv, plan_len);
  // Enough splits for whole clusters: reduce in-kernel (no combine launch).
  const bool use_cluster = fused && c->cluster && n_splits >= kCluster && n_kv <= kMaxCounters;
  if (use_cluster) n_splits = ((n_splits + kCluster - 1) / kCluster) * kCluster;
  if (n_splits > 1) {
    int rc = ensure_scratch(c, (long long)c->cfg.n_heads_q * n_splits, st);
    if (rc != GQA_OK) return rc;
  }
  DecodeParams p = base_params(c);
  p.k_base = kv->k_cache;
  p.v_base = kv->v_cache;
  p.qkv = qkv;
  p.len = len;
  p.lengths_stable = lengths_stable ? 1 : 0;
  p.n_splits = n_splits;
  p.out = out;
  p.cluster = use_cluster ? kCluster : 0;
  p.counters = c->counters;
  GQA_CUDA(launch_decode_split(p, 1, fused, st, pdl_first, single_variant(c)));
  if (n_splits > 1 && !use_cluster) {
    CombineParams cp = combine_from_scratch(c, n_splits);
    cp.out = out;
    GQA_CUDA(launch_combine_wide(cp, 1, st, c->layers_pdl != 0));
  }
  return GQA_OK;
}

// The decode step on the shape-generic kernels (gqa_generic.cu): split
// partials (RoPE and the append fused), then the merge.
// lengths_stable: pos / seq_len are not produced by the preceding kernel (see
// split_generic_kernel).
int run_generic(gqa_ctx* c, cudaStream_t st, const gqa_layer_kv* kv, const float* qkv,
                Lengths len, int plan_len, float* out, bool pdl_first, bool lengths_stable) {
  const int nq = c->cfg.n_heads_q, nkv = c->cfg.n_heads_kv;
  const int n_splits = generic_plan_splits(nkv, plan_len, c->n_sm);
  int rc = ensure_scratch(c, (long long)nq * n_splits, st);
  if (rc != GQA_OK) return rc;
  GQA_CUDA(launch_generic_attention(qkv, out, kv->k_cache, kv->v_cache, len, c->cfg.t_max, nq,
                                    nkv, c->cfg.head_dim, n_splits, plan_len, c->inv_freq,
                                    c->part_o, c->part_ml, c->status, st, pdl_first,
                                    c->layers_pdl != 0, lengths_stable));
  return GQA_OK;
}

// Entry points built only for the tuned shape (head_dim 128, group 6).
int tuned_only(const gqa_ctx* c, const char* what) {
  if (c->generic)
    return fail(GQA_ERR_UNSUPPORTED, "%s: built for head_dim 128 with 6 q heads per KV head "
                "only (this context: head_dim %d, %d per KV head)", what, c->cfg.head_dim,
                c->cfg.n_heads_q / c->cfg.n_heads_kv);
  return GQA_OK;
}

int layers_impl(gqa_ctx* c, cudaStream_t st, int n_layers, const gqa_layer_kv* kv,
                const float* qkv, long long qkv_stride, float* out, long long out_stride,
                int* d_pos, int advance, int wrap_lo, int wrap_hi) {
  if (n_layers < 1 || !kv || !qkv || !out || !d_pos)
    return fail(GQA_ERR_INVALID_ARG, "gqa_decode_layers: null argument or n_layers < 1");
  const int nq = c->cfg.n_heads_q, nkv = c->cfg.n_heads_kv, hd = c->cfg.head_dim;
  if (qkv_stride < (long long)(nq + 2 * nkv) * hd || out_stride < (long long)nq * hd)
    return fail(GQA_ERR_INVALID_ARG, "layer strides smaller than one layer's qkv / output");
  if ((qkv_stride & 3) || (out_stride & 3) || !aligned16(qkv) || !aligned16(out))
    return fail(GQA_ERR_INVALID_ARG, "qkv/out and their layer strides must be 16-byte aligned");
  for (int l = 0; l < n_layers; ++l) {
    int rc = check_kv(c, &kv[l]);
    if (rc != GQA_OK) return rc;
  }
  Lengths len{};
  len.pos_dev = d_pos;
  for (int l = 0; l < n_layers; ++l) {
    // Layer 0 is launched without programmatic overlap, so whatever advanced
    // *d_pos before it has finished and it may read pos (and stream its
    // cache rows) at once.  Later layers follow a kernel of the previous
    // layer, which never writes pos or this layer's cache.
    const bool pdl = l > 0 && c->layers_pdl != 0;
    int rc = c->generic
                 ? run_generic(c, st, &kv[l], qkv + l * qkv_stride, len, c->cfg.t_max,
                               out + l * out_stride, pdl, /*lengths_stable=*/true)
                 : run_single(c, st, &kv[l], qkv + l * qkv_stride, len, c->cfg.t_max, true,
                              out + l * out_stride, pdl, /*lengths_stable=*/true);
    if (rc != GQA_OK) return rc;
  }
  if (advance) GQA_CUDA(launch_advance_pos(d_pos, wrap_lo, wrap_hi, st, true));
  return GQA_OK;
}

// The decoder sizes of the context's shape: 0 for Qwen2.5-1.5B (head_dim 128,
// 12 / 2 heads: d_model 1536, d_ffn 8960), 1 for Qwen2.5-0.5B (head_dim 64,
// 14 / 2 heads: d_model 896, d_ffn 4864), -1 for a shape whose projections
// are not built.
int block_model(const gqa_ctx* c) {
  const int dm = c->cfg.n_heads_q * c->cfg.head_dim;
  if (!c->generic && dm == block_d_model(0)) return 0;
  if (c->generic && c->cfg.head_dim == 64 && c->cfg.n_heads_kv == 2 && dm == block_d_model(1))
    return 1;
  return -1;
}

int need_block_model(const gqa_ctx* c, const char* what) {
  if (block_model(c) < 0)
    return fail(GQA_ERR_UNSUPPORTED, "%s built for the Qwen2.5-1.5B (128-dim heads, 12 / 2, "
                "d_model 1536) and Qwen2.5-0.5B (64-dim heads, 14 / 2, d_model 896) shapes only "
                "(this context: head_dim %d, %d / %d heads)", what, c->cfg.head_dim,
                c->cfg.n_heads_q, c->cfg.n_heads_kv);
  return GQA_OK;
}

// One attention block: QKV projection (with RMSNorm) -> split-KV attention
// (RoPE + append fused) and merge -> Wo projection into the state.
int check_block_weights(const gqa_ctx* c, const gqa_block_weights* w) {
  if (!w || !w->w_qkv || !w->b_qkv || !w->w_o || !w->gamma)
    return fail(GQA_ERR_INVALID_ARG, "null block weight pointer");
  if (need_block_model(c, "attention block") != GQA_OK) return GQA_ERR_UNSUPPORTED;
  if (!aligned16(w->w_qkv) || !aligned16(w->w_o) || !aligned16(w->b_qkv) || !aligned16(w->gamma))
    return fail(GQA_ERR_INVALID_ARG, "block weights must be 16-byte aligned");
  return GQA_OK;
}

// The split kernel's immediate predecessor is the QKV projection, which writes
// neither pos nor a cache, and every kernel of the library releases its
// dependents only after its own dependency wait: by the time the split kernel
// starts, the kernel that advanced a device-side pos (two launches back at the
// nearest) has finished, so the split may read the lengths and stream its cache
// rows before its wait, in every layer.
int block_impl(gqa_ctx* c, cudaStream_t st, const gqa_block_weights* w, const gqa_layer_kv* kv,
               float* state, Lengths len, int plan_len, bool pdl_first) {
  const bool lengths_stable = true;
  const int nq = c->cfg.n_heads_q, nkv = c->cfg.n_heads_kv, hd = c->cfg.head_dim;
  const int model = block_model(c);
  GQA_CUDA(launch_qkv_gemv(model, w->w_qkv, w->b_qkv, w->gamma, state, c->blk_qkv,
                           (nq + 2 * nkv) * hd, c->status, st, pdl_first));
  int rc = c->generic ? run_generic(c, st, kv, c->blk_qkv, len, plan_len, c->blk_attn, true,
                                    lengths_stable)
                      : run_single(c, st, kv, c->blk_qkv, len, plan_len, true, c->blk_attn, true,
                                   lengths_stable, /*grid_ok=*/false);
  if (rc != GQA_OK) return rc;
  GQA_CUDA(launch_wo_gemv(model, w->w_o, c->blk_attn, state, nq * hd, c->status, st, true));
  return GQA_OK;
}

int check_ffn_weights(const gqa_ctx* c, const gqa_ffn_weights* w) {
  if (!w || !w->w_gate || !w->w_up || !w->w_down || !w->gamma)
    return fail(GQA_ERR_INVALID_ARG, "null FFN weight pointer");
  if (need_block_model(c, "FFN block") != GQA_OK) return GQA_ERR_UNSUPPORTED;
  if (!aligned16(w->w_gate) || !aligned16(w->w_up) || !aligned16(w->w_down) ||
      !aligned16(w->gamma))
    return fail(GQA_ERR_INVALID_ARG, "FFN weights must be 16-byte aligned");
  return GQA_OK;
}

// q8: the Q8_0 head (built for d_model 896), else the Q6_K head (d_model 1536).
int check_head(const gqa_ctx* c, bool q8, const void* packed, int n_rows, const float* gamma) {
  if (block_model(c) != (q8 ? 1 : 0))
    return fail(GQA_ERR_UNSUPPORTED, "the %s LM head is built for d_model %d only (this context: "
                "%d)", q8 ? "Q8_0" : "Q6_K", block_d_model(q8 ? 1 : 0),
                c->cfg.n_heads_q * c->cfg.head_dim);
  if (!packed || !gamma || n_rows < 1)
    return fail(GQA_ERR_INVALID_ARG, "LM head: null weights or n_rows %d", n_rows);
  if (!aligned16(packed) || !aligned16(gamma))
    return fail(GQA_ERR_INVALID_ARG, "LM head weights must be 16-byte aligned");
  return GQA_OK;
}
int ffn_impl(gqa_ctx* c, cudaStream_t st, const gqa_ffn_weights* w, float* state, bool pdl_first) {
  const int model = block_model(c);
  GQA_CUDA(launch_gateup_gemv(model, w->w_gate, w->w_up, w->gamma, state, c->blk_h, c->status,
                              st, pdl_first));
  GQA_CUDA(launch_down_gemv(model, w->w_down, c->blk_h, state, c->status, st, true));
  return GQA_OK;
}

// Runs the split kernel of one KV shard (rows [shard_begin, shard_begin +
// shard_rows) of the sequence, global position pos) and describes its
// partials in *cp for a merge (cp->n_parts = 0 when the shard attends no row).
int shard_partials(gqa_ctx* c, cudaStream_t st, const gqa_layer_kv* kv, const float* qkv, int pos,
                   int shard_begin, int shard_rows, CombineParams* cp) {
  int rc = check_kv(c, kv);
  if (rc != GQA_OK) return rc;
  if (!qkv || !aligned16(qkv)) return fail(GQA_ERR_INVALID_ARG, "null or unaligned qkv");
  if (pos < 0 || shard_begin < 0 || shard_rows < 0 || shard_rows > c->cfg.t_max)
    return fail(GQA_ERR_INVALID_ARG, "pos %d / shard [%d, +%d) invalid (t_max %d)", pos,
                shard_begin, shard_rows, c->cfg.t_max);
  const int nq = c->cfg.n_heads_q;
  // Rows of this shard that the new token attends: global [shard_begin, pos].
  long long attended = (long long)pos + 1 - shard_begin;
  if (attended > shard_rows) attended = shard_rows;
  if (attended < 0) attended = 0;
  const bool owns = pos >= shard_begin && pos < shard_begin + shard_rows;
  *cp = CombineParams{};
  int n_splits = 0;
  if (attended > 0) {
    n_splits = plan_splits_single(c, c->cfg.n_heads_kv, (int)attended);
    rc = ensure_scratch(c, (long long)nq * n_splits, st);
    if (rc != GQA_OK) return rc;
    DecodeParams p = base_params(c);
    p.k_base = kv->k_cache;
    p.v_base = kv->v_cache;
    p.qkv = qkv;
    p.rope_override = 1;
    p.rope_pos = pos;
    p.skip_append = owns ? 0 : 1;
    p.len.pos_imm = owns ? pos - shard_begin : 0;
    p.len.seqlen_imm = (int)attended;
    p.t_end = (int)attended;
    p.n_splits = n_splits;
    p.out = nullptr;  // partials only
    GQA_CUDA(launch_decode_split(p, 1, true, st, c->pdl != 0, single_variant(c)));
    *cp = combine_from_scratch(c, n_splits);
  } else {
    cp->rows_per_seq = nq;
  }
  cp->n_parts = n_splits;
  return GQA_OK;
}

}  // namespace

namespace gqa {
// Records an error message for gqa_last_error_string() from other units.
int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

// The context's decoder sizes (block_model above), for the model loader.
int ctx_block_model(const gqa_ctx* c) { return block_model(c); }
}  // namespace gqa

extern "C" {

const char* gqa_last_error_string(void) { return g_err; }

const char* gqa_version(void) { return "gqa-b200 0.1 (sm_100a)"; }

int gqa_create(const gqa_config* cfg, int device, gqa_ctx** out) {
  if (!cfg || !out) return fail(GQA_ERR_INVALID_ARG, "gqa_create: null argument");
  *out = nullptr;
  if (cfg->n_heads_kv < 1 || cfg->n_heads_q % cfg->n_heads_kv)
    return fail(GQA_ERR_INVALID_ARG, "n_heads_q must be a multiple of n_heads_kv (got %d / %d)",
                cfg->n_heads_q, cfg->n_heads_kv);
  const int group = cfg->n_heads_q / cfg->n_heads_kv;
  const bool tuned = cfg->head_dim == kHeadDim && group == 6;
  if (!tuned && !generic_shape_built(cfg->head_dim, group))
    return fail(GQA_ERR_UNSUPPORTED,
                "shape not built: head_dim %d with %d q heads per KV head (built: 128 / 6, "
                "64 / 7)", cfg->head_dim, group);
  if (cfg->t_max < 1 || !(cfg->rope_theta > 0.f))
    return fail(GQA_ERR_INVALID_ARG, "t_max must be >= 1 and rope_theta > 0");
  if ((long long)cfg->n_heads_kv * cfg->t_max * kHeadDim > (1LL << 40))
    return fail(GQA_ERR_INVALID_ARG, "cache too large");
  int n_dev = 0;
  GQA_CUDA(cudaGetDeviceCount(&n_dev));
  if (device < 0 || device >= n_dev) return fail(GQA_ERR_INVALID_ARG, "no device %d", device);
  DeviceGuard g(device);
  if (g.err != cudaSuccess) return fail(GQA_ERR_CUDA, "cudaSetDevice: %s", cudaGetErrorString(g.err));
  int major = 0, minor = 0;
  GQA_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device));
  GQA_CUDA(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device));
  if (major != 10 || minor != 0)
    return fail(GQA_ERR_UNSUPPORTED, "built for sm_100a only; device is sm_%d%d", major, minor);

  gqa_ctx* c = new gqa_ctx();
  c->device = device;
  c->cfg = *cfg;
  cudaDeviceGetAttribute(&c->n_sm, cudaDevAttrMultiProcessorCount, device);
  // attention_gqa_benchmark.c:143: powf(ROPE_BASE, -2.0f * (float)tid / (float)HEAD_DIM),
  // evaluated once here with the host libm so the device multiplies the very
  // same fp32 inverse frequency by pos.
  c->generic = !tuned;
  for (int i = 0; i < kHalf; ++i)
    c->h_inv_freq[i] =
        i < cfg->head_dim / 2 ? powf(cfg->rope_theta, -2.0f * (float)i / (float)cfg->head_dim)
                              : 0.f;
  cudaError_t e = prepare_decode_kernels();
  if (e == cudaSuccess) e = prepare_prefill_kernels();
  if (e == cudaSuccess) e = cudaMalloc(&c->inv_freq, sizeof(float) * kHalf);
  if (e == cudaSuccess) e = cudaMalloc(&c->status, sizeof(int));
  if (e == cudaSuccess)
    e = cudaMalloc(&c->blk_qkv, sizeof(float) * (cfg->n_heads_q + 2 * cfg->n_heads_kv) * kHeadDim);
  if (e == cudaSuccess) e = cudaMalloc(&c->blk_attn, sizeof(float) * cfg->n_heads_q * kHeadDim);
  if (e == cudaSuccess) e = cudaMalloc(&c->blk_h, sizeof(float) * block_max_d_ffn());
  if (e == cudaSuccess) e = prepare_block_kernels();
  if (e == cudaSuccess) e = prepare_head_kernels();
  if (e == cudaSuccess) e = cudaMalloc(&c->counters, sizeof(int) * kCounterSlots);
  if (e == cudaSuccess) e = cudaMemset(c->counters, 0, sizeof(int) * kCounterSlots);
  // Epoch-tagged grid-merge partials: zeroed here and written by nothing else,
  // so no stale word ever carries a current epoch.
  const size_t grid_words_bytes =
      sizeof(unsigned long long) * (size_t)cfg->n_heads_q * kGridMaxParts * kGridRowWords;
  if (e == cudaSuccess) e = cudaMalloc(&c->grid_epoch, kGridEpochWords * sizeof(unsigned));
  if (e == cudaSuccess) e = cudaMemset(c->grid_epoch, 0, kGridEpochWords * sizeof(unsigned));
  if (e == cudaSuccess && tuned) e = cudaMalloc(&c->grid_words, grid_words_bytes);
  if (e == cudaSuccess && tuned) e = cudaMemset(c->grid_words, 0, grid_words_bytes);
  if (e == cudaSuccess) c->grid_ctas_per_sm = decode_grid_ctas_per_sm(grid_variant(c));
  if (e == cudaSuccess) c->grid_ctas_per_sm_long = decode_grid_ctas_per_sm(3);
  if (e == cudaSuccess) {
    c->head_grid = lm_head_grid(c->n_sm);
    e = cudaMalloc(&c->head_best, lm_head_best_bytes(c->head_grid));
  }
  if (e == cudaSuccess)
    e = cudaMemcpy(c->inv_freq, c->h_inv_freq, sizeof(float) * kHalf, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemset(c->status, 0, sizeof(int));
  if (e != cudaSuccess) {
    gqa_destroy(c);
    return fail(GQA_ERR_CUDA, "context set-up failed: %s", cudaGetErrorString(e));
  }
  *out = c;
  return GQA_OK;
}

int gqa_destroy(gqa_ctx* c) {
  if (!c) return GQA_OK;
  DeviceGuard g(c->device);
  if (c->inv_freq) cudaFree(c->inv_freq);
  if (c->status) cudaFree(c->status);
  if (c->counters) cudaFree(c->counters);
  if (c->grid_epoch) cudaFree(c->grid_epoch);
  if (c->grid_words) cudaFree(c->grid_words);
  if (c->blk_qkv) cudaFree(c->blk_qkv);
  if (c->blk_attn) cudaFree(c->blk_attn);
  if (c->blk_h) cudaFree(c->blk_h);
  if (c->head_best) cudaFree(c->head_best);
  if (c->prefill_img) cudaFree(c->prefill_img);
  if (c->rope_cs) cudaFree(c->rope_cs);
  if (c->part_o) cudaFree(c->part_o);
  if (c->part_ml) cudaFree(c->part_ml);
  delete c;
  return GQA_OK;
}

int gqa_set_option(gqa_ctx* c, int option, long long value) {
  if (!c) return fail(GQA_ERR_INVALID_ARG, "null context");
  switch (option) {
    case GQA_OPT_PDL: c->pdl = value ? 1 : 0; return GQA_OK;
    case GQA_OPT_TARGET_CTAS:
      if (value < 0 || value > (1 << 20)) return fail(GQA_ERR_INVALID_ARG, "target CTAs out of range");
      c->target_ctas = (int)value;
      return GQA_OK;
    case 3: /* GQA_OPT_BATCH_CHUNK (internal tuning knob) */
      if (value < 0 || value > (1 << 20)) return fail(GQA_ERR_INVALID_ARG, "chunk out of range");
      c->batch_chunk = (int)value;
      return GQA_OK;
    case 5: /* GQA_OPT_LAYERS_PDL (internal tuning knob) */
      c->layers_pdl = value ? 1 : 0;
      return GQA_OK;
    case 6: /* GQA_OPT_CLUSTER (internal tuning knob) */
      c->cluster = value ? 1 : 0;
      return GQA_OK;
    case GQA_OPT_BATCH_ADVANCE:
      c->batch_advance = value ? 1 : 0;
      return GQA_OK;
    case 7: /* GQA_OPT_GRID_MERGE (internal tuning knob) */
      c->grid_merge = value ? 1 : 0;
      return GQA_OK;
    case 4: /* GQA_OPT_KERNEL_VARIANT (internal tuning knob) */
      if (value < -1 || value >= decode_variant_count())
        return fail(GQA_ERR_INVALID_ARG, "kernel variant out of range (-1 = automatic)");
      c->variant = (int)value;
      c->grid_ctas_per_sm = decode_grid_ctas_per_sm(grid_variant(c));
      return GQA_OK;
    default: return fail(GQA_ERR_INVALID_ARG, "unknown option %d", option);
  }
}

int gqa_reserve(gqa_ctx* c, int n_seq, int max_len) {
  if (!c || n_seq < 1 || max_len < 1 || max_len > c->cfg.t_max)
    return fail(GQA_ERR_INVALID_ARG, "gqa_reserve: bad arguments");
  DeviceGuard g(c->device);
  if (c->generic)
    return ensure_scratch(c, (long long)n_seq * c->cfg.n_heads_q *
                                 generic_plan_splits(c->cfg.n_heads_kv, max_len, c->n_sm),
                          nullptr);
  int single = ((plan_splits_single(c, c->cfg.n_heads_kv, max_len) + kCluster - 1) /
                kCluster) * kCluster;
  const int grid = plan_splits_grid(c, c->cfg.n_heads_kv, max_len);
  if (grid > single) single = grid;
  const int batched = ceil_div(max_len, batch_chunk(c, 1, max_len));  // the most splits
  const int splits = single > batched ? single : batched;
  return ensure_scratch(c, (long long)n_seq * c->cfg.n_heads_q * splits, nullptr);
}

int gqa_device_status(gqa_ctx* c, int* status, int clear) {
  if (!c || !status) return fail(GQA_ERR_INVALID_ARG, "null argument");
  DeviceGuard g(c->device);
  GQA_CUDA(cudaDeviceSynchronize());
  GQA_CUDA(cudaMemcpy(status, c->status, sizeof(int), cudaMemcpyDeviceToHost));
  if (clear) GQA_CUDA(cudaMemset(c->status, 0, sizeof(int)));
  return GQA_OK;
}

int gqa_kv_alloc(gqa_ctx* c, int n_layers, gqa_layer_kv* out) {
  if (!c || !out || n_layers < 1) return fail(GQA_ERR_INVALID_ARG, "gqa_kv_alloc: bad arguments");
  DeviceGuard g(c->device);
  const size_t bytes =
      sizeof(float) * (size_t)c->cfg.n_heads_kv * c->cfg.t_max * c->cfg.head_dim;
  for (int l = 0; l < n_layers; ++l) out[l].k_cache = out[l].v_cache = nullptr;
  for (int l = 0; l < n_layers; ++l) {
    if (cudaMalloc(&out[l].k_cache, bytes) != cudaSuccess ||
        cudaMalloc(&out[l].v_cache, bytes) != cudaSuccess ||
        cudaMemset(out[l].k_cache, 0, bytes) != cudaSuccess ||
        cudaMemset(out[l].v_cache, 0, bytes) != cudaSuccess) {
      cudaGetLastError();
      gqa_kv_free(c, n_layers, out);
      return fail(GQA_ERR_NO_MEMORY, "KV cache allocation failed at layer %d", l);
    }
  }
  return GQA_OK;
}

int gqa_kv_free(gqa_ctx* c, int n_layers, gqa_layer_kv* kv) {
  if (!c || !kv || n_layers < 0) return fail(GQA_ERR_INVALID_ARG, "gqa_kv_free: bad arguments");
  DeviceGuard g(c->device);
  for (int l = 0; l < n_layers; ++l) {
    if (kv[l].k_cache) cudaFree(kv[l].k_cache);
    if (kv[l].v_cache) cudaFree(kv[l].v_cache);
    kv[l].k_cache = kv[l].v_cache = nullptr;
  }
  return GQA_OK;
}

int gqa_layer_attention_out(gqa_ctx* c, gqa_stream_t stream, const gqa_layer_kv* kv,
                            const float* qkv, int pos, int seq_len, float* out) {
  GQA_RANGE("gqa_layer_attention_out");
  if (!c) return fail(GQA_ERR_INVALID_ARG, "null context");
  int rc = check_kv(c, kv);
  if (rc != GQA_OK) return rc;
  if (!qkv || !out || !aligned16(qkv) || !aligned16(out))
    return fail(GQA_ERR_INVALID_ARG, "qkv/out must be non-null and 16-byte aligned");
  if (pos < 0 || pos >= c->cfg.t_max || seq_len < 1 || seq_len > c->cfg.t_max)
    return fail(GQA_ERR_INVALID_ARG, "pos %d / seq_len %d outside [0, t_max=%d)", pos, seq_len,
                c->cfg.t_max);
  DeviceGuard g(c->device);
  Lengths len{};
  len.pos_imm = pos;
  len.seqlen_imm = seq_len;
  if (c->generic) return run_generic(c, (cudaStream_t)stream, kv, qkv, len, seq_len, out,
                                     c->pdl != 0, true);
  return run_single(c, (cudaStream_t)stream, kv, qkv, len, seq_len, true, out, c->pdl != 0,
                    true);
}

int gqa_layer_attention(gqa_ctx* c, gqa_stream_t stream, const gqa_layer_kv* kv, float* qkv,
                        int pos, int seq_len) {
  return gqa_layer_attention_out(c, stream, kv, qkv, pos, seq_len, qkv);
}

int gqa_decode_layers(gqa_ctx* c, gqa_stream_t stream, int n_layers, const gqa_layer_kv* kv,
                      const float* qkv, long long qkv_layer_stride, float* out,
                      long long out_layer_stride, int* d_pos, int advance, int wrap_lo,
                      int wrap_hi) {
  GQA_RANGE("gqa_decode_layers");
  if (!c) return fail(GQA_ERR_INVALID_ARG, "null context");
  DeviceGuard g(c->device);
  return layers_impl(c, (cudaStream_t)stream, n_layers, kv, qkv, qkv_layer_stride, out,
                     out_layer_stride, d_pos, advance, wrap_lo, wrap_hi);
}

int gqa_graph_create_layers(gqa_ctx* c, int n_layers, const gqa_layer_kv* kv, const float* qkv,
                            long long qkv_layer_stride, float* out, long long out_layer_stride,
                            int* d_pos, int advance, int wrap_lo, int wrap_hi,
                            gqa_graph** out_graph) {
  GQA_RANGE("gqa_graph_create_layers");
  if (!c || !out_graph) return fail(GQA_ERR_INVALID_ARG, "null argument");
  *out_graph = nullptr;
  DeviceGuard g(c->device);
  int rc = gqa_reserve(c, 1, c->cfg.t_max);
  if (rc != GQA_OK) return rc;
  cudaStream_t st;
  GQA_CUDA(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
  cudaGraph_t graph = nullptr;
  cudaError_t e = cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal);
  if (e != cudaSuccess) {
    cudaStreamDestroy(st);
    return fail(GQA_ERR_CUDA, "cudaStreamBeginCapture: %s", cudaGetErrorString(e));
  }
  rc = layers_impl(c, st, n_layers, kv, qkv, qkv_layer_stride, out, out_layer_stride, d_pos,
                   advance, wrap_lo, wrap_hi);
  e = cudaStreamEndCapture(st, &graph);
  cudaStreamDestroy(st);
  if (rc != GQA_OK) {
    if (graph) cudaGraphDestroy(graph);
    return rc;
  }
  if (e != cudaSuccess) return fail(GQA_ERR_CUDA, "cudaStreamEndCapture: %s", cudaGetErrorString(e));
  cudaGraphExec_t exec = nullptr;
  e = cudaGraphInstantiate(&exec, graph, 0);
  if (e != cudaSuccess) {
    cudaGraphDestroy(graph);
    return fail(GQA_ERR_CUDA, "cudaGraphInstantiate: %s", cudaGetErrorString(e));
  }
  gqa_graph* gr = new gqa_graph();
  c->live_graphs++;
  gr->ctx = c;
  gr->graph = graph;
  gr->exec = exec;
  gr->d_qkv = qkv;
  gr->d_out = out;
  gr->qkv_bytes = sizeof(float) * (size_t)qkv_layer_stride * n_layers;
  gr->out_bytes = sizeof(float) * (size_t)out_layer_stride * n_layers;
  *out_graph = gr;
  return GQA_OK;
}

int gqa_graph_launch(gqa_graph* gr, gqa_stream_t stream) {
  GQA_RANGE("gqa_graph_launch");
  if (!gr) return fail(GQA_ERR_INVALID_ARG, "null graph");
  DeviceGuard g(gr->ctx->device);
  GQA_CUDA(cudaGraphLaunch(gr->exec, (cudaStream_t)stream));
  return GQA_OK;
}

int gqa_graph_step_host(gqa_graph* gr, gqa_stream_t stream, const float* h_qkv, float* h_out) {
  GQA_RANGE("gqa_graph_step_host");
  if (!gr || !h_qkv || !h_out) return fail(GQA_ERR_INVALID_ARG, "null argument");
  DeviceGuard g(gr->ctx->device);
  cudaStream_t st = (cudaStream_t)stream;
  GQA_CUDA(cudaMemcpyAsync((void*)gr->d_qkv, h_qkv, gr->qkv_bytes, cudaMemcpyHostToDevice, st));
  GQA_CUDA(cudaGraphLaunch(gr->exec, st));
  GQA_CUDA(cudaMemcpyAsync(h_out, gr->d_out, gr->out_bytes, cudaMemcpyDeviceToHost, st));
  return GQA_OK;
}

int gqa_graph_destroy(gqa_graph* gr) {
  if (!gr) return GQA_OK;
  DeviceGuard g(gr->ctx->device);
  if (gr->exec) cudaGraphExecDestroy(gr->exec);
  if (gr->graph) cudaGraphDestroy(gr->graph);
  gr->ctx->live_graphs--;
  delete gr;
  return GQA_OK;
}

int gqa_rope_kv_append(gqa_ctx* c, gqa_stream_t stream, const gqa_layer_kv* kv, float* q,
                       const float* k, const float* v, int pos) {
  GQA_RANGE("gqa_rope_kv_append");
  if (!c) return fail(GQA_ERR_INVALID_ARG, "null context");
  if (tuned_only(c, "gqa_rope_kv_append") != GQA_OK) return GQA_ERR_UNSUPPORTED;
  int rc = check_kv(c, kv);
  if (rc != GQA_OK) return rc;
  if (!q || !k || !v) return fail(GQA_ERR_INVALID_ARG, "null q/k/v");
  if (pos < 0 || pos >= c->cfg.t_max)
    return fail(GQA_ERR_INVALID_ARG, "pos %d outside [0, %d)", pos, c->cfg.t_max);
  const int nq = c->cfg.n_heads_q, nkv = c->cfg.n_heads_kv;
  // The kernel addresses k and v relative to q (one qkv row); stage separate
  // buffers through that layout only when they already are one row.
  if (k != q + (long long)nq * kHeadDim || v != k + (long long)nkv * kHeadDim)
    return fail(GQA_ERR_INVALID_ARG,
                "q, k, v must be consecutive slices of one qkv row (k = q + n_heads_q*128, "
                "v = k + n_heads_kv*128)");
  DeviceGuard g(c->device);
  Lengths len{};
  len.pos_imm = pos;
  len.seqlen_imm = pos + 1;
  GQA_CUDA(launch_rope_append(q, 0, nullptr, nullptr, kv->k_cache, kv->v_cache, 0, len,
                              c->cfg.t_max, nq, nkv, c->inv_freq, c->status, 1,
                              (cudaStream_t)stream, c->pdl != 0));
  return GQA_OK;
}

int gqa_decode(gqa_ctx* c, gqa_stream_t stream, const gqa_layer_kv* kv, const float* q_rot,
               int seq_len, float* out) {
  GQA_RANGE("gqa_decode");
  if (!c) return fail(GQA_ERR_INVALID_ARG, "null context");
  if (tuned_only(c, "gqa_decode") != GQA_OK) return GQA_ERR_UNSUPPORTED;
  int rc = check_kv(c, kv);
  if (rc != GQA_OK) return rc;
  if (!q_rot || !out || !aligned16(q_rot) || !aligned16(out))
    return fail(GQA_ERR_INVALID_ARG, "q/out must be non-null and 16-byte aligned");
  if (seq_len < 1 || seq_len > c->cfg.t_max)
    return fail(GQA_ERR_INVALID_ARG, "seq_len %d outside [1, %d]", seq_len, c->cfg.t_max);
  DeviceGuard g(c->device);
  Lengths len{};
  len.pos_imm = seq_len - 1;
  len.seqlen_imm = seq_len;
  return run_single(c, (cudaStream_t)stream, kv, q_rot, len, seq_len, false, out, c->pdl != 0,
                    true);
}

int gqa_decode_batched(gqa_ctx* c, gqa_stream_t stream, int n_seq, float* const* k_caches,
                       float* const* v_caches, const float* qkv, long long qkv_stride,
                       const int* seq_lens, int max_len, float* out, long long out_stride) {
  GQA_RANGE("gqa_decode_batched");
  if (!c) return fail(GQA_ERR_INVALID_ARG, "null context");
  if (tuned_only(c, "gqa_decode_batched") != GQA_OK) return GQA_ERR_UNSUPPORTED;
  if (n_seq < 1 || n_seq > 65535 || !k_caches || !v_caches || !qkv || !seq_lens || !out)
    return fail(GQA_ERR_INVALID_ARG, "gqa_decode_batched: null argument or n_seq out of range");
  if (max_len < 1 || max_len > c->cfg.t_max)
    return fail(GQA_ERR_INVALID_ARG, "max_len %d outside [1, %d]", max_len, c->cfg.t_max);
  const int nq = c->cfg.n_heads_q, nkv = c->cfg.n_heads_kv;
  if (qkv_stride < (long long)(nq + 2 * nkv) * kHeadDim || out_stride < (long long)nq * kHeadDim)
    return fail(GQA_ERR_INVALID_ARG, "qkv/out strides smaller than one sequence's row");
  if ((qkv_stride & 3) || (out_stride & 3) || !aligned16(qkv) || !aligned16(out))
    return fail(GQA_ERR_INVALID_ARG, "qkv/out and their strides must be 16-byte aligned");
  if (out != qkv && out < qkv + qkv_stride * n_seq && qkv < out + out_stride * n_seq)
    return fail(GQA_ERR_INVALID_ARG, "out overlaps qkv without being equal to it");
  DeviceGuard g(c->device);
  cudaStream_t st = (cudaStream_t)stream;
  const int chunk = batch_chunk(c, n_seq, max_len);
  const int n_splits = ceil_div(max_len, chunk);
  if (n_splits > 65535) return fail(GQA_ERR_INVALID_ARG, "too many splits");
  if (n_splits > 1) {
    int rc = ensure_scratch(c, (long long)n_seq * nq * n_splits, st);
    if (rc != GQA_OK) return rc;
  }
  // In-place output: the split kernels read q of their own sequence before
  // the combine overwrites it (separate launches), so out == qkv is safe.
  DecodeParams p = base_params(c);
  p.k_ptrs = k_caches;
  p.v_ptrs = v_caches;
  p.qkv = qkv;
  p.qkv_stride = qkv_stride;
  p.len.seq_lens = seq_lens;
  p.lengths_stable = 0;
  p.n_splits = n_splits;
  p.min_chunk = chunk;
  p.out = out;
  p.out_stride = out_stride;
  GQA_CUDA(launch_decode_split(p, n_seq, true, st, c->pdl != 0, batch_variant(c)));
  // With GQA_OPT_BATCH_ADVANCE the step's last kernel advances the lengths
  // (the caller's next step), after every read of them.
  int* advance = c->batch_advance ? const_cast<int*>(seq_lens) : nullptr;
  if (n_splits > 1) {
    CombineParams cp = combine_from_scratch(c, n_splits);
    cp.out = out;
    cp.out_stride = out_stride;
    cp.advance_lens = advance;
    GQA_CUDA(launch_combine(cp, n_seq, st, true));
  } else if (advance) {
    GQA_CUDA(launch_advance_lens(advance, n_seq, st, true));
  }
  return GQA_OK;
}

int gqa_decode_batched_host(gqa_ctx* c, gqa_stream_t stream, int n_seq, float* const* k_caches,
                            float* const* v_caches, const float* h_qkv, float* d_qkv,
                            long long qkv_stride, const int* seq_lens, int max_len, float* d_out,
                            long long out_stride, float* h_out) {
  GQA_RANGE("gqa_decode_batched_host");
  if (!c) return fail(GQA_ERR_INVALID_ARG, "null context");
  if (!h_qkv || !h_out || !d_qkv || !d_out)
    return fail(GQA_ERR_INVALID_ARG, "gqa_decode_batched_host: null buffer");
  if (n_seq < 1 || n_seq > 65535 || qkv_stride < 1)
    return fail(GQA_ERR_INVALID_ARG, "gqa_decode_batched_host: n_seq or qkv_stride out of range");
  DeviceGuard g(c->device);
  cudaStream_t st = (cudaStream_t)stream;
  GQA_CUDA(cudaMemcpyAsync(d_qkv, h_qkv, sizeof(float) * (size_t)qkv_stride * n_seq,
                           cudaMemcpyHostToDevice, st));
  const int rc = gqa_decode_batched(c, stream, n_seq, k_caches, v_caches, d_qkv, qkv_stride,
                                    seq_lens, max_len, d_out, out_stride);
  if (rc != GQA_OK) return rc;
  const size_t row = sizeof(float) * (size_t)c->cfg.n_heads_q * kHeadDim;
  const size_t pitch = sizeof(float) * (size_t)out_stride;
  if (pitch == row)  // packed rows: one plain copy
    GQA_CUDA(cudaMemcpyAsync(h_out, d_out, row * (size_t)n_seq, cudaMemcpyDeviceToHost, st));
  else
    GQA_CUDA(cudaMemcpy2DAsync(h_out, row, d_out, pitch, row, (size_t)n_seq,
                               cudaMemcpyDeviceToHost, st));
  return GQA_OK;
}

int gqa_decode_split_partial(gqa_ctx* c, gqa_stream_t stream, const gqa_layer_kv* kv,
                             const float* q_rot, int t_begin, int t_end, float* m, float* l,
                             float* o) {
  GQA_RANGE("gqa_decode_split_partial");
  if (!c) return fail(GQA_ERR_INVALID_ARG, "null context");
  if (tuned_only(c, "gqa_decode_split_partial") != GQA_OK) return GQA_ERR_UNSUPPORTED;
  int rc = check_kv(c, kv);
  if (rc != GQA_OK) return rc;
  if (!q_rot || !m || !l || !o || !aligned16(q_rot))
    return fail(GQA_ERR_INVALID_ARG, "null argument or unaligned q");
  if (t_begin < 0 || t_end < t_begin || t_end > c->cfg.t_max)
    return fail(GQA_ERR_INVALID_ARG, "range [%d, %d) outside [0, %d]", t_begin, t_end,
                c->cfg.t_max);
  DeviceGuard g(c->device);
  cudaStream_t st = (cudaStream_t)stream;
  const int nq = c->cfg.n_heads_q;
  CombineParams cp{};
  int n_splits = 0;
  if (t_end > t_begin) {
    n_splits = plan_splits_single(c, c->cfg.n_heads_kv, t_end - t_begin);
    rc = ensure_scratch(c, (long long)nq * n_splits, st);
    if (rc != GQA_OK) return rc;
    DecodeParams p = base_params(c);
    p.k_base = kv->k_cache;
    p.v_base = kv->v_cache;
    p.qkv = q_rot;
    p.len.pos_imm = t_end - 1;
    p.len.seqlen_imm = t_end;
    p.t_begin = t_begin;
    p.t_end = t_end;
    p.n_splits = n_splits;
    p.out = nullptr;  // always write partials
    GQA_CUDA(launch_decode_split(p, 1, false, st, c->pdl != 0, single_variant(c)));
    cp = combine_from_scratch(c, n_splits);
  } else {
    cp.rows_per_seq = nq;
  }
  cp.n_parts = n_splits;
  cp.out = o;
  cp.out_m = m;
  cp.out_l = l;
  GQA_CUDA(launch_combine(cp, 1, st, true));
  return GQA_OK;
}

int gqa_decode_kv_shard(gqa_ctx* c, gqa_stream_t stream, const gqa_layer_kv* kv,
                        const float* qkv, int pos, int shard_begin, int shard_rows, float* m,
                        float* l, float* o) {
  GQA_RANGE("gqa_decode_kv_shard");
  if (!c) return fail(GQA_ERR_INVALID_ARG, "null context");
  if (tuned_only(c, "gqa_decode_kv_shard") != GQA_OK) return GQA_ERR_UNSUPPORTED;
  if (!m || !l || !o) return fail(GQA_ERR_INVALID_ARG, "null argument");
  DeviceGuard g(c->device);
  cudaStream_t st = (cudaStream_t)stream;
  CombineParams cp{};
  int rc = shard_partials(c, st, kv, qkv, pos, shard_begin, shard_rows, &cp);
  if (rc != GQA_OK) return rc;
  cp.out = o;
  cp.out_m = m;
  cp.out_l = l;
  GQA_CUDA(launch_combine(cp, 1, st, true));
  return GQA_OK;
}

int gqa_attention_block(gqa_ctx* c, gqa_stream_t stream, const gqa_block_weights* w,
                        const gqa_layer_kv* kv, float* state, int pos, int seq_len) {
  GQA_RANGE("gqa_attention_block");
  if (!c) return fail(GQA_ERR_INVALID_ARG, "null context");
  int rc = check_block_weights(c, w);
  if (rc != GQA_OK) return rc;
  rc = check_kv(c, kv);
  if (rc != GQA_OK) return rc;
  if (!state || !aligned16(state)) return fail(GQA_ERR_INVALID_ARG, "null or unaligned state");
  if (pos < 0 || pos >= c->cfg.t_max || seq_len < 1 || seq_len > c->cfg.t_max)
    return fail(GQA_ERR_INVALID_ARG, "pos %d / seq_len %d out of range (t_max %d)", pos, seq_len,
                c->cfg.t_max);
  DeviceGuard g(c->device);
  Lengths len{};
  len.pos_imm = pos;
  len.seqlen_imm = seq_len;
  return block_impl(c, (cudaStream_t)stream, w, kv, state, len, seq_len, c->pdl != 0);
}

int gqa_attention_block_layers(gqa_ctx* c, gqa_stream_t stream, int n_layers,
                               const gqa_block_weights* w, const gqa_layer_kv* kv, float* state,
                               int* d_pos, int advance, int wrap_lo, int wrap_hi) {
  GQA_RANGE("gqa_attention_block_layers");
  if (!c) return fail(GQA_ERR_INVALID_ARG, "null context");
  if (n_layers < 1 || !w || !kv || !d_pos || !state || !aligned16(state))
    return fail(GQA_ERR_INVALID_ARG, "gqa_attention_block_layers: bad arguments");
  for (int l = 0; l < n_layers; ++l) {
    int rc = check_block_weights(c, &w[l]);
    if (rc == GQA_OK) rc = check_kv(c, &kv[l]);
    if (rc != GQA_OK) return rc;
  }
  DeviceGuard g(c->device);
  cudaStream_t st = (cudaStream_t)stream;
  Lengths len{};
  len.pos_dev = d_pos;
  for (int l = 0; l < n_layers; ++l) {
    // Layer 0's QKV projection may follow the kernel that advanced *d_pos;
    // the split kernel after it reads pos early (see block_impl).
    int rc = block_impl(c, st, &w[l], &kv[l], state, len, c->cfg.t_max, c->layers_pdl != 0);
    if (rc != GQA_OK) return rc;
  }
  if (advance) GQA_CUDA(launch_advance_pos(d_pos, wrap_lo, wrap_hi, st, true));
  return GQA_OK;
}

int gqa_ffn_block(gqa_ctx* c, gqa_stream_t stream, const gqa_ffn_weights* w, float* state) {
  GQA_RANGE("gqa_ffn_block");
  if (!c) return fail(GQA_ERR_INVALID_ARG, "null context");
  int rc = check_ffn_weights(c, w);
  if (rc != GQA_OK) return rc;
  if (!state || !aligned16(state)) return fail(GQA_ERR_INVALID_ARG, "null or unaligned state");
  DeviceGuard g(c->device);
  return ffn_impl(c, (cudaStream_t)stream, w, state, c->pdl != 0);
}

int gqa_decoder_layers(gqa_ctx* c, gqa_stream_t stream, int n_layers, const gqa_block_weights* attn,
                       const gqa_ffn_weights* ffn, const gqa_layer_kv* kv, float* state,
                       int* d_pos, int advance, int wrap_lo, int wrap_hi) {
  GQA_RANGE("gqa_decoder_layers");
  if (!c) return fail(GQA_ERR_INVALID_ARG, "null context");
  if (n_layers < 1 || !attn || !ffn || !kv || !d_pos || !state || !aligned16(state))
    return fail(GQA_ERR_INVALID_ARG, "gqa_decoder_layers: bad arguments");
  for (int l = 0; l < n_layers; ++l) {
    int rc = check_block_weights(c, &attn[l]);
    if (rc == GQA_OK) rc = check_ffn_weights(c, &ffn[l]);
    if (rc == GQA_OK) rc = check_kv(c, &kv[l]);
    if (rc != GQA_OK) return rc;
  }
  DeviceGuard g(c->device);
  cudaStream_t st = (cudaStream_t)stream;
  Lengths len{};
  len.pos_dev = d_pos;
  for (int l = 0; l < n_layers; ++l) {
    // (the split kernels read pos early: see block_impl)
    int rc = block_impl(c, st, &attn[l], &kv[l], state, len, c->cfg.t_max, c->layers_pdl != 0);
    if (rc == GQA_OK) rc = ffn_impl(c, st, &ffn[l], state, true);
    if (rc != GQA_OK) return rc;
  }
  if (advance) GQA_CUDA(launch_advance_pos(d_pos, wrap_lo, wrap_hi, st, true));
  return GQA_OK;
}

long long gqa_lm_head_packed_bytes(int n_rows) {
  return n_rows < 1 ? 0 : (long long)lm_head_packed_bytes(n_rows);
}

int gqa_lm_head_pack(gqa_ctx* c, gqa_stream_t stream, const void* q6k, int n_rows, void* packed) {
  if (!c) return fail(GQA_ERR_INVALID_ARG, "null context");
  if (!q6k || !packed || n_rows < 1)
    return fail(GQA_ERR_INVALID_ARG, "gqa_lm_head_pack: null buffer or n_rows %d", n_rows);
  if (!aligned16(packed)) return fail(GQA_ERR_INVALID_ARG, "packed head must be 16-byte aligned");
  DeviceGuard g(c->device);
  GQA_CUDA(launch_q6k_pack(q6k, n_rows, packed, (cudaStream_t)stream));
  return GQA_OK;
}

int gqa_lm_head(gqa_ctx* c, gqa_stream_t stream, const void* packed, int n_rows,
                const float* gamma, const float* state, float* logits, int* token) {
  GQA_RANGE("gqa_lm_head");
  if (!c) return fail(GQA_ERR_INVALID_ARG, "null context");
  int rc = check_head(c, false, packed, n_rows, gamma);
  if (rc != GQA_OK) return rc;
  if (!state || !aligned16(state)) return fail(GQA_ERR_INVALID_ARG, "null or unaligned state");
  if (!logits && !token) return fail(GQA_ERR_INVALID_ARG, "gqa_lm_head: no output requested");
  DeviceGuard g(c->device);
  GQA_CUDA(launch_lm_head(false, packed, n_rows, gamma, state, logits, token, c->head_best,
                          reinterpret_cast<unsigned*>(c->counters + kHeadDoneSlot), c->status,
                          c->head_grid, (cudaStream_t)stream, c->pdl != 0));
  return GQA_OK;
}

long long gqa_lm_head_q8_0_packed_bytes(int n_rows) {
  return n_rows < 1 ? 0 : (long long)lm_head_q8_packed_bytes(n_rows);
}

int gqa_lm_head_q8_0_pack(gqa_ctx* c, gqa_stream_t stream, const void* q8, int n_rows,
                          void* packed) {
  if (!c) return fail(GQA_ERR_INVALID_ARG, "null context");
  if (!q8 || !packed || n_rows < 1)
    return fail(GQA_ERR_INVALID_ARG, "gqa_lm_head_q8_0_pack: null buffer or n_rows %d", n_rows);
  if (!aligned16(packed)) return fail(GQA_ERR_INVALID_ARG, "packed head must be 16-byte aligned");
  DeviceGuard g(c->device);
  GQA_CUDA(launch_q8_pack(q8, n_rows, packed, (cudaStream_t)stream));
  return GQA_OK;
}

int gqa_lm_head_q8_0(gqa_ctx* c, gqa_stream_t stream, const void* packed, int n_rows,
                     const float* gamma, const float* state, float* logits, int* token) {
  GQA_RANGE("gqa_lm_head_q8_0");
  if (!c) return fail(GQA_ERR_INVALID_ARG, "null context");
  int rc = check_head(c, true, packed, n_rows, gamma);
  if (rc != GQA_OK) return rc;
  if (!state || !aligned16(state)) return fail(GQA_ERR_INVALID_ARG, "null or unaligned state");
  if (!logits && !token) return fail(GQA_ERR_INVALID_ARG, "gqa_lm_head_q8_0: no output requested");
  DeviceGuard g(c->device);
  GQA_CUDA(launch_lm_head(true, packed, n_rows, gamma, state, logits, token, c->head_best,
                          reinterpret_cast<unsigned*>(c->counters + kHeadDoneSlot), c->status,
                          c->head_grid, (cudaStream_t)stream, c->pdl != 0));
  return GQA_OK;
}

int gqa_token_embedding(gqa_ctx* c, gqa_stream_t stream, const void* table, int n_rows,
                        const int* d_token, float* state) {
  GQA_RANGE("gqa_token_embedding");
  if (!c) return fail(GQA_ERR_INVALID_ARG, "null context");
  if (need_block_model(c, "gqa_token_embedding") != GQA_OK) return GQA_ERR_UNSUPPORTED;
  if (!table || !d_token || !state || n_rows < 1)
    return fail(GQA_ERR_INVALID_ARG, "gqa_token_embedding: null argument or n_rows %d", n_rows);
  DeviceGuard g(c->device);
  GQA_CUDA(launch_embed_q4(table, n_rows, block_d_model(block_model(c)), d_token, state,
                           c->status, (cudaStream_t)stream, c->pdl != 0));
  return GQA_OK;
}

int gqa_decode_token(gqa_ctx* c, gqa_stream_t stream, const gqa_model* m, float* state,
                     int* d_token, int* d_pos, float* logits, int wrap_lo, int wrap_hi) {
  GQA_RANGE("gqa_decode_token");
  if (!c) return fail(GQA_ERR_INVALID_ARG, "null context");
  if (!m || m->n_layers < 1 || !m->attn || !m->ffn || !m->kv || !m->token_embd || !d_token ||
      !d_pos || !state || !aligned16(state))
    return fail(GQA_ERR_INVALID_ARG, "gqa_decode_token: bad arguments");
  if (m->lm_head_type != GQA_HEAD_Q6_K && m->lm_head_type != GQA_HEAD_Q8_0)
    return fail(GQA_ERR_INVALID_ARG, "gqa_decode_token: lm_head_type %d", m->lm_head_type);
  const bool q8 = m->lm_head_type == GQA_HEAD_Q8_0;
  int rc = check_head(c, q8, m->lm_head, m->vocab, m->gamma_output);
  if (rc != GQA_OK) return rc;
  for (int l = 0; l < m->n_layers; ++l) {
    rc = check_block_weights(c, &m->attn[l]);
    if (rc == GQA_OK) rc = check_ffn_weights(c, &m->ffn[l]);
    if (rc == GQA_OK) rc = check_kv(c, &m->kv[l]);
    if (rc != GQA_OK) return rc;
  }
  DeviceGuard g(c->device);
  cudaStream_t st = (cudaStream_t)stream;
  const bool pdl = c->layers_pdl != 0;
  GQA_CUDA(launch_embed_q4(m->token_embd, m->vocab, block_d_model(block_model(c)), d_token, state,
                           c->status, st, pdl));
  Lengths len{};
  len.pos_dev = d_pos;
  for (int l = 0; l < m->n_layers; ++l) {
    // (the split kernels read pos early: see block_impl)
    rc = block_impl(c, st, &m->attn[l], &m->kv[l], state, len, c->cfg.t_max, pdl);
    if (rc == GQA_OK) rc = ffn_impl(c, st, &m->ffn[l], state, pdl);
    if (rc != GQA_OK) return rc;
  }
  GQA_CUDA(launch_lm_head(q8, m->lm_head, m->vocab, m->gamma_output, state, logits, d_token,
                          c->head_best, reinterpret_cast<unsigned*>(c->counters + kHeadDoneSlot),
                          c->status, c->head_grid, st, pdl));
  GQA_CUDA(launch_advance_pos(d_pos, wrap_lo, wrap_hi, st, pdl));
  return GQA_OK;
}

int gqa_exchange_create(gqa_ctx* c, int rank, int world, gqa_exchange** out, void* ipc_handle) {
  if (!c || !out || !ipc_handle) return fail(GQA_ERR_INVALID_ARG, "null argument");
  if (tuned_only(c, "gqa_exchange_create") != GQA_OK) return GQA_ERR_UNSUPPORTED;
  *out = nullptr;
  if (world < 1 || world > kMaxExchangeWorld || rank < 0 || rank >= world)
    return fail(GQA_ERR_INVALID_ARG, "rank %d / world %d invalid (world <= %d)", rank, world,
                kMaxExchangeWorld);
  DeviceGuard g(c->device);
  gqa_exchange* x = new gqa_exchange();
  x->ctx = c;
  x->device = c->device;
  x->rank = rank;
  x->world = world;
  x->n_rows = c->cfg.n_heads_q;
  // One inbox serves either form of the merge: the exchange kernel's slots or
  // the fused split kernel's per-slice slots (kXSlotWords words each).
  const size_t fused_bytes =
      sizeof(unsigned long long) * 2ull * world * x->n_rows * kXSlices * kXSlotWords;
  const size_t bytes = std::max(exchange_inbox_bytes(world, x->n_rows), fused_bytes);
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaMalloc(&x->base, bytes);
  if (e == cudaSuccess) e = cudaMemset(x->base, 0, bytes);
  if (e == cudaSuccess) e = cudaMalloc(&x->epoch, sizeof(unsigned) * x->n_rows);
  if (e == cudaSuccess) e = cudaMemset(x->epoch, 0, sizeof(unsigned) * x->n_rows);
  if (e == cudaSuccess) e = cudaMalloc(&x->slice_epoch, sizeof(unsigned) * x->n_rows * kXSlices);
  if (e == cudaSuccess)
    e = cudaMemset(x->slice_epoch, 0, sizeof(unsigned) * x->n_rows * kXSlices);
  if (e == cudaSuccess) e = cudaMalloc(&x->d_inbox, sizeof(uint2*) * world);
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, x->base);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    gqa_exchange_destroy(x);
    return fail(GQA_ERR_CUDA, "gqa_exchange_create: %s", cudaGetErrorString(e));
  }
  memcpy(ipc_handle, &h, sizeof(h));
  x->own = h;
  *out = x;
  return GQA_OK;
}

int gqa_exchange_open(gqa_exchange* x, const void* handles) {
  if (!x || !handles) return fail(GQA_ERR_INVALID_ARG, "null argument");
  if (x->opened) return fail(GQA_ERR_INVALID_ARG, "exchange already opened");
  DeviceGuard g(x->device);
  uint2* inbox[kMaxExchangeWorld];
  for (int r = 0; r < x->world; ++r) {
    cudaIpcMemHandle_t h;
    memcpy(&h, static_cast<const char*>(handles) + (size_t)r * GQA_IPC_HANDLE_BYTES, sizeof(h));
    if (r == x->rank || memcmp(&h, &x->own, sizeof(h)) == 0) {
      // This process's own inbox (a handle cannot be opened by its exporter).
      x->peer[r] = x->base;
    } else {
      cudaError_t e = cudaIpcOpenMemHandle(&x->peer[r], h, cudaIpcMemLazyEnablePeerAccess);
      if (e != cudaSuccess) {
        x->peer[r] = nullptr;
        cudaGetLastError();
        return fail(GQA_ERR_CUDA, "opening the inbox of rank %d: %s", r, cudaGetErrorString(e));
      }
    }
    inbox[r] = static_cast<uint2*>(x->peer[r]);
  }
  GQA_CUDA(cudaMemcpy(x->d_inbox, inbox, sizeof(uint2*) * x->world, cudaMemcpyHostToDevice));
  x->opened = true;
  return GQA_OK;
}

}  // extern "C"

namespace {
// One GPU's share of a KV-range-split step as ONE launch: the grid-merged split
// kernel over this shard's rows (RoPE at the global position, the new row
// appended only by the shard that holds it), whose merging CTAs merge their
// slice locally, exchange it with every GPU over peer memory and write the
// output.  Every rank runs it, also a shard that attends no row (it publishes
// empty partials), so all ranks take the same steps.
int shard_exchange_fused(gqa_ctx* c, gqa_exchange* x, cudaStream_t st, const gqa_layer_kv* kv,
                         const float* qkv, int pos, int shard_begin, int shard_rows, float* out) {
  int rc = check_kv(c, kv);
  if (rc != GQA_OK) return rc;
  if (!qkv || !aligned16(qkv)) return fail(GQA_ERR_INVALID_ARG, "null or unaligned qkv");
  if (pos < 0 || shard_begin < 0 || shard_rows < 0 || shard_rows > c->cfg.t_max)
    return fail(GQA_ERR_INVALID_ARG, "pos %d / shard [%d, +%d) invalid (t_max %d)", pos,
                shard_begin, shard_rows, c->cfg.t_max);
  const int n_kv = c->cfg.n_heads_kv;
  long long attended = (long long)pos + 1 - shard_begin;  // global rows [shard_begin, pos]
  if (attended > shard_rows) attended = shard_rows;
  if (attended < 0) attended = 0;
  const bool owns = pos >= shard_begin && pos < shard_begin + shard_rows;
  const int quant = decode_variant_grid_quant(grid_variant(c));
  const int target = c->target_ctas > 0 && c->target_ctas < c->n_sm ? c->target_ctas : c->n_sm;
  int n_splits = target / n_kv;
  const int most = ceil_div(attended, quant);
  if (n_splits > most) n_splits = most;
  if (n_splits > kGridMaxParts) n_splits = kGridMaxParts;
  if (n_splits < 1) n_splits = 1;
  DecodeParams p = base_params(c);
  p.k_base = kv->k_cache;
  p.v_base = kv->v_cache;
  p.qkv = qkv;
  p.rope_override = 1;
  p.rope_pos = pos;
  p.skip_append = owns ? 0 : 1;
  p.len.pos_imm = owns ? pos - shard_begin : 0;
  p.len.seqlen_imm = (int)attended;
  p.t_end = (int)attended;
  p.lengths_stable = 1;
  p.n_splits = n_splits;
  const int gv = grid_variant_for(c, attended, n_splits);
  p.min_chunk = decode_variant_grid_quant(gv);
  p.out = out;
  p.grid_epoch = c->grid_epoch;
  p.grid_words = c->grid_words;
  p.allow_empty = 1;
  p.x_inbox = reinterpret_cast<unsigned long long* const*>(x->d_inbox);
  p.x_epoch = x->slice_epoch;
  p.x_rank = x->rank;
  p.x_world = x->world;
  GQA_CUDA(launch_decode_split(p, 1, true, st, c->pdl != 0, gv));
  return GQA_OK;
}
}  // namespace

extern "C" {

int gqa_decode_kv_shard_exchange(gqa_ctx* c, gqa_exchange* x, gqa_stream_t stream,
                                 const gqa_layer_kv* kv, const float* qkv, int pos,
                                 int shard_begin, int shard_rows, float* out) {
  GQA_RANGE("gqa_decode_kv_shard_exchange");
  if (!c || !x || !out) return fail(GQA_ERR_INVALID_ARG, "null argument");
  if (tuned_only(c, "gqa_decode_kv_shard_exchange") != GQA_OK) return GQA_ERR_UNSUPPORTED;
  if (x->ctx != c || !x->opened)
    return fail(GQA_ERR_INVALID_ARG, "exchange belongs to another context or is not opened");
  if (!aligned16(out)) return fail(GQA_ERR_INVALID_ARG, "out must be 16-byte aligned");
  DeviceGuard g(c->device);
  cudaStream_t st = (cudaStream_t)stream;
  if (c->grid_merge && c->grid_ctas_per_sm >= 1 && c->grid_words && x->world <= kXMaxWorld)
    return shard_exchange_fused(c, x, st, kv, qkv, pos, shard_begin, shard_rows, out);
  CombineParams cp{};
  int rc = shard_partials(c, st, kv, qkv, pos, shard_begin, shard_rows, &cp);
  if (rc != GQA_OK) return rc;
  GQA_CUDA(launch_exchange_combine(cp, x->d_inbox, x->epoch, x->rank, x->world, out, c->status,
                                   st, true));
  return GQA_OK;
}

int gqa_exchange_destroy(gqa_exchange* x) {
  if (!x) return GQA_OK;
  DeviceGuard g(x->device);
  for (int r = 0; r < x->world; ++r)
    if (x->peer[r] && x->peer[r] != x->base) cudaIpcCloseMemHandle(x->peer[r]);
  if (x->d_inbox) cudaFree(x->d_inbox);
  if (x->epoch) cudaFree(x->epoch);
  if (x->slice_epoch) cudaFree(x->slice_epoch);
  if (x->base) cudaFree(x->base);
  delete x;
  return GQA_OK;
}

int gqa_lse_combine(gqa_ctx* c, gqa_stream_t stream, int n_parts, int n_rows, const float* m,
                    const float* l, const float* o, float* out) {
  GQA_RANGE("gqa_lse_combine");
  if (!c) return fail(GQA_ERR_INVALID_ARG, "null context");
  if (tuned_only(c, "gqa_lse_combine") != GQA_OK) return GQA_ERR_UNSUPPORTED;
  if (n_parts < 0 || n_parts > 4096 || n_rows < 1 || n_rows > 65535 || !m || !l || !o || !out)
    return fail(GQA_ERR_INVALID_ARG, "gqa_lse_combine: bad arguments");
  DeviceGuard g(c->device);
  CombineParams cp{};
  cp.m = m;
  cp.l = l;
  cp.o = o;
  cp.ml_part_stride = n_rows;
  cp.ml_row_stride = 1;
  cp.o_part_stride = (long long)n_rows * kHeadDim;
  cp.o_row_stride = kHeadDim;
  cp.n_parts = n_parts;
  cp.rows_per_seq = n_rows;
  cp.out = out;
  GQA_CUDA(launch_combine(cp, 1, (cudaStream_t)stream, c->pdl != 0));
  return GQA_OK;
}

int gqa_lse_combine_packed(gqa_ctx* c, gqa_stream_t stream, int n_parts, int n_rows,
                           const float* packed, long long part_stride, float* out) {
  GQA_RANGE("gqa_lse_combine_packed");
  if (!c) return fail(GQA_ERR_INVALID_ARG, "null context");
  if (tuned_only(c, "gqa_lse_combine_packed") != GQA_OK) return GQA_ERR_UNSUPPORTED;
  if (n_parts < 0 || n_parts > 4096 || n_rows < 1 || n_rows > 65535 || !packed || !out ||
      part_stride < (long long)n_rows * (2 + kHeadDim))
    return fail(GQA_ERR_INVALID_ARG, "gqa_lse_combine_packed: bad arguments");
  DeviceGuard g(c->device);
  CombineParams cp{};
  cp.m = packed;
  cp.l = packed + n_rows;
  cp.o = packed + 2 * n_rows;
  cp.ml_part_stride = part_stride;
  cp.ml_row_stride = 1;
  cp.o_part_stride = part_stride;
  cp.o_row_stride = kHeadDim;
  cp.n_parts = n_parts;
  cp.rows_per_seq = n_rows;
  cp.out = out;
  GQA_CUDA(launch_combine(cp, 1, (cudaStream_t)stream, c->pdl != 0));
  return GQA_OK;
}

int gqa_prefill_bf16(gqa_ctx* c, gqa_stream_t stream, int n_seq, int seq_len, const float* qkv,
                     float* out, float* const* k_caches, float* const* v_caches) {
  GQA_RANGE("gqa_prefill_bf16");
  if (!c) return fail(GQA_ERR_INVALID_ARG, "null context");
  if (tuned_only(c, "gqa_prefill_bf16") != GQA_OK) return GQA_ERR_UNSUPPORTED;
  if (n_seq < 1 || n_seq > 65535 || !qkv || !out)
    return fail(GQA_ERR_INVALID_ARG, "gqa_prefill_bf16: null argument or n_seq out of range");
  if (seq_len < 128 || seq_len % 128 != 0 || seq_len > 65535 * 128)
    return fail(GQA_ERR_UNSUPPORTED, "gqa_prefill_bf16: seq_len %d must be a positive multiple of 128",
                seq_len);
  if ((k_caches == nullptr) != (v_caches == nullptr))
    return fail(GQA_ERR_INVALID_ARG, "give both cache arrays or neither");
  if (k_caches && seq_len > c->cfg.t_max)
    return fail(GQA_ERR_INVALID_ARG, "seq_len %d exceeds the cache capacity t_max %d", seq_len,
                c->cfg.t_max);
  if (!aligned16(qkv) || !aligned16(out))
    return fail(GQA_ERR_INVALID_ARG, "qkv/out must be 16-byte aligned");
  DeviceGuard g(c->device);
  cudaStream_t st = (cudaStream_t)stream;
  const int nq = c->cfg.n_heads_q, nkv = c->cfg.n_heads_kv;
  const size_t per = (size_t)n_seq * seq_len * kHeadDim;
  const size_t need = per * (size_t)(nq + 2 * nkv);
  if (need > c->prefill_cap) {
    if (is_capturing(st) || c->live_graphs > 0)
      return fail(GQA_ERR_NO_MEMORY, "prefill scratch must grow outside capture / live graphs");
    if (c->prefill_img) cudaFree(c->prefill_img);
    c->prefill_img = nullptr;
    c->prefill_cap = 0;
    if (cudaMalloc(&c->prefill_img, need * sizeof(__nv_bfloat16)) != cudaSuccess) {
      cudaGetLastError();
      return fail(GQA_ERR_NO_MEMORY, "cudaMalloc of %zu bytes of prefill scratch failed",
                  need * sizeof(__nv_bfloat16));
    }
    c->prefill_cap = need;
  }
  if (seq_len > c->rope_cap) {
    // The table covers max(seq_len, t_max) positions and is filled once, on
    // the caller's stream, when it is (re)allocated.
    if (is_capturing(st) || c->live_graphs > 0)
      return fail(GQA_ERR_NO_MEMORY, "prefill RoPE table must grow outside capture / live graphs");
    const int cap = seq_len > c->cfg.t_max ? seq_len : c->cfg.t_max;
    if (c->rope_cs) cudaFree(c->rope_cs);
    c->rope_cs = nullptr;
    c->rope_cap = 0;
    if (cudaMalloc(&c->rope_cs, sizeof(float2) * (size_t)cap * (kHeadDim / 2)) != cudaSuccess) {
      cudaGetLastError();
      return fail(GQA_ERR_NO_MEMORY, "cudaMalloc of the prefill RoPE table failed");
    }
    GQA_CUDA(launch_prefill_rope_table(c->inv_freq, c->rope_cs, cap, st));
    c->rope_cap = cap;
  }
  __nv_bfloat16* qimg = c->prefill_img;
  __nv_bfloat16* kimg = qimg + per * nq;
  __nv_bfloat16* vimg = kimg + per * nkv;
  GQA_CUDA(launch_prefill(qkv, (long long)seq_len * (nq + 2 * nkv) * kHeadDim, n_seq, seq_len, nq,
                          nkv, c->rope_cs, qimg, kimg, vimg, k_caches, v_caches, c->cfg.t_max,
                          out, c->status, c->counters + kPrefillSchedSlot, c->n_sm, st));
  return GQA_OK;
}

int gqa_fill_normal(gqa_ctx* c, gqa_stream_t stream, float* dst, long long n,
                    unsigned long long seed, unsigned long long stream_id, long long offset) {
  if (!c || !dst || n < 0 || offset < 0) return fail(GQA_ERR_INVALID_ARG, "bad arguments");
  if (n == 0) return GQA_OK;
  DeviceGuard g(c->device);
  // Stream key: splitmix64 finaliser of seed ^ (stream_id * odd constant);
  // identical to seeded.stream_key() on the host.
  uint64_t z = (uint64_t)seed ^ ((uint64_t)stream_id * 0xD1B54A32D192ED03ULL);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
  z = z ^ (z >> 31);
  GQA_CUDA(launch_fill_normal(dst, n, z, offset, c->n_sm, (cudaStream_t)stream));
  return GQA_OK;
}

int gqa_phase_trace_read(unsigned long long* records, int max_records, int reset,
                         int* n_records) {
  if (!n_records || max_records < 0 || (max_records > 0 && !records))
    return fail(GQA_ERR_INVALID_ARG, "gqa_phase_trace_read: bad arguments");
  *n_records = 0;
  const int n = phase_trace_read(records, max_records, reset != 0);
  if (n == -1)
    return fail(GQA_ERR_UNSUPPORTED, "this library was built without the phase trace "
                "(build with -DGQA_PHASE_TRACE)");
  if (n < 0) return fail(GQA_ERR_CUDA, "gqa_phase_trace_read: copy failed");
  *n_records = n;
  return GQA_OK;
}

int gqa_inv_freq(const gqa_ctx* c, float* out) {
  if (!c || !out) return fail(GQA_ERR_INVALID_ARG, "null argument");
  memcpy(out, c->h_inv_freq, sizeof(c->h_inv_freq));
  return GQA_OK;
}

}  // extern "C"
