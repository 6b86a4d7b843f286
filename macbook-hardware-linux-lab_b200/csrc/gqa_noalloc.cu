// Attention layer call that allocates nothing (gqa_layer_attention_static).
//
// Some callers cannot allocate device memory at the point where they run the
// layer call: code running inside a host callback or a custom allocator's
// critical section, plugins whose host framework owns every device allocation
// (or forbids them after start-up), and graph-capture setups where any
// allocation would be an error.  Such callers can still run the full fused
// decode through this entry point: its split-KV scratch is a file-scope
// static device array, part of the library's own image, so no context,
// cudaMalloc, cudaFree or allocating library routine is involved.
//
// Limits and sharing.  The array holds kStaticSlots (q head x split) partials:
// 4096 slots of 130 floats (about 2.03 MiB) plus a 64-float RoPE table and a
// status word, and every GPU that loads the library keeps it until the process
// exits.  A call whose split plan needs more slots than that is rejected.
// Each device has its own copy of the array, and all calls on one device
// share it; it keeps the last call's contents.  Calls on one device that can
// overlap on the GPU (issued to different streams without ordering between
// them) race on it, so the caller must order them (one stream, or events).
// The partials need no clearing: every partial a call reads was written
// earlier in the same call.  The status word is cleared at set-up and read
// (and cleared) with gqa_static_status.
#include <cmath>
#include <cstdio>
#include <mutex>

#include "gqa.h"
#include "gqa_common.cuh"

namespace gqa {
cudaError_t prepare_decode_kernels();
cudaError_t launch_decode_split(const DecodeParams& p, int n_seq, bool fused, cudaStream_t st,
                                bool pdl, int variant);
cudaError_t launch_combine(const CombineParams& c, int n_seq, cudaStream_t st, bool pdl);
int decode_variant_quant(int variant);
int set_error(int code, const char* fmt, ...);
}  // namespace gqa

using namespace gqa;

namespace {

constexpr int kStaticSlots = 4096;
constexpr size_t kOffPartO = 0;
constexpr size_t kOffPartMl = kOffPartO + (size_t)kStaticSlots * kHeadDim;
constexpr size_t kOffInvFreq = kOffPartMl + (size_t)kStaticSlots * 2;
constexpr size_t kOffStatus = kOffInvFreq + kHalf;
constexpr size_t kStaticFloats = kOffStatus + 64;  // status word, padded

// The scratch itself.  In host code this name is only a stand-in for the
// symbol: its device address comes from cudaGetSymbolAddress, per device.
static __device__ __align__(256) float g_noalloc_scratch[kStaticFloats];

constexpr int kMaxDevices = 64;
struct StaticDevice {
  bool ready = false;
  float* base = nullptr;  // device address of g_noalloc_scratch on this device
  int n_sm = 0;
  float theta = NAN;      // rope_theta whose table is loaded
};
StaticDevice g_dev[kMaxDevices];
std::mutex g_mu;

// First call on a device (with that device current): look up the array's
// device address, prepare the kernels and clear the status word (synchronous
// copies, so this first call must come before any stream capture).  Whenever
// rope_theta differs from the one last written, the new inverse-frequency
// table is written with an asynchronous copy on the caller's stream, so it is
// ordered like the calls themselves: calls ordered on one stream (or by
// events) each see their own table.  Calls that may overlap on the GPU race on
// the table as on the rest of the array.
int setup_device(int dev, float theta, cudaStream_t st, StaticDevice** out) {
  std::lock_guard<std::mutex> lock(g_mu);
  StaticDevice& s = g_dev[dev];
  if (!s.ready) {
    cudaError_t e = cudaGetSymbolAddress(reinterpret_cast<void**>(&s.base), g_noalloc_scratch);
    if (e != cudaSuccess)
      return set_error(GQA_ERR_CUDA, "cudaGetSymbolAddress(static scratch) failed: %s",
                       cudaGetErrorString(e));
    e = prepare_decode_kernels();
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&s.n_sm, cudaDevAttrMultiProcessorCount, dev);
    const float zero[1] = {0.f};
    if (e == cudaSuccess)
      e = cudaMemcpyToSymbol(g_noalloc_scratch, zero, sizeof(zero), sizeof(float) * kOffStatus,
                             cudaMemcpyHostToDevice);
    if (e != cudaSuccess)
      return set_error(GQA_ERR_CUDA, "static-scratch set-up failed: %s", cudaGetErrorString(e));
    s.ready = true;
  }
  if (!(s.theta == theta)) {
    float table[kHalf];
    // attention_gqa_benchmark.c:143 evaluated once on the host, as the
    // context path does.
    for (int i = 0; i < kHalf; ++i) table[i] = powf(theta, -2.0f * (float)i / (float)kHeadDim);
    cudaError_t e = cudaMemcpyToSymbolAsync(g_noalloc_scratch, table, sizeof(table),
                                            sizeof(float) * kOffInvFreq, cudaMemcpyHostToDevice,
                                            st);
    if (e != cudaSuccess)
      return set_error(GQA_ERR_CUDA, "writing the RoPE table failed: %s", cudaGetErrorString(e));
    s.theta = theta;
  }
  *out = &s;
  return GQA_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" int gqa_layer_attention_static(const gqa_config* cfg, gqa_stream_t stream,
                                          const gqa_layer_kv* kv, float* qkv, int pos,
                                          int seq_len) {
  if (!cfg || !kv || !kv->k_cache || !kv->v_cache || !qkv)
    return set_error(GQA_ERR_INVALID_ARG, "gqa_layer_attention_static: null argument");
  if (cfg->head_dim != kHeadDim || cfg->n_heads_kv < 1 || cfg->n_heads_q != 6 * cfg->n_heads_kv)
    return set_error(GQA_ERR_UNSUPPORTED,
                     "gqa_layer_attention_static: needs head_dim 128 and n_heads_q = 6 * n_heads_kv");
  if (cfg->t_max < 1 || !(cfg->rope_theta > 0.f))
    return set_error(GQA_ERR_INVALID_ARG, "gqa_layer_attention_static: bad t_max / rope_theta");
  if (pos < 0 || pos >= cfg->t_max || seq_len < 1 || seq_len > cfg->t_max)
    return set_error(GQA_ERR_INVALID_ARG, "pos %d / seq_len %d outside [0, t_max=%d)", pos,
                     seq_len, cfg->t_max);
  if (!aligned16(qkv) || !aligned16(kv->k_cache) || !aligned16(kv->v_cache))
    return set_error(GQA_ERR_INVALID_ARG, "qkv and the caches must be 16-byte aligned");
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return set_error(GQA_ERR_CUDA, "no usable current device");
  StaticDevice* s = nullptr;
  int rc = setup_device(dev, cfg->rope_theta, (cudaStream_t)stream, &s);
  if (rc != GQA_OK) return rc;

  // Same split plan as the context path: one CTA per SM over the KV heads,
  // never a split shorter than the kernel's row quantum.
  const int n_q = cfg->n_heads_q, n_kv = cfg->n_heads_kv;
  const int quant = decode_variant_quant(0);
  int n_splits = (s->n_sm + n_kv - 1) / n_kv;
  const int most = (seq_len + quant - 1) / quant;
  if (n_splits > most) n_splits = most;
  if (n_splits < 1) n_splits = 1;
  if ((long long)n_q * n_splits > kStaticSlots)
    return set_error(GQA_ERR_INVALID_ARG,
                     "gqa_layer_attention_static: %d q heads x %d splits need %lld scratch slots; "
                     "the static scratch holds %d",
                     n_q, n_splits, (long long)n_q * n_splits, kStaticSlots);

  cudaStream_t st = (cudaStream_t)stream;
  DecodeParams p{};
  p.k_base = kv->k_cache;
  p.v_base = kv->v_cache;
  p.t_max = cfg->t_max;
  p.n_kv = n_kv;
  p.qkv = qkv;
  p.len.pos_imm = pos;
  p.len.seqlen_imm = seq_len;
  p.lengths_stable = 1;
  p.n_splits = n_splits;
  p.min_chunk = quant;
  p.inv_freq = s->base + kOffInvFreq;
  p.q_scale = (1.0f / sqrtf((float)kHeadDim)) * 1.4426950408889634f;
  p.part_o = s->base + kOffPartO;
  p.part_ml = s->base + kOffPartMl;
  p.out = qkv;
  p.status = reinterpret_cast<int*>(s->base + kOffStatus);
  e = launch_decode_split(p, 1, true, st, false, 0);
  if (e == cudaSuccess && n_splits > 1) {
    CombineParams cp{};
    cp.m = p.part_ml;
    cp.l = p.part_ml + 1;
    cp.o = p.part_o;
    cp.ml_part_stride = 2;
    cp.ml_row_stride = 2LL * n_splits;
    cp.o_part_stride = kHeadDim;
    cp.o_row_stride = (long long)kHeadDim * n_splits;
    cp.n_parts = n_splits;
    cp.rows_per_seq = n_q;
    cp.out = qkv;
    e = launch_combine(cp, 1, st, true);
  }
  if (e != cudaSuccess)
    return set_error(GQA_ERR_CUDA, "gqa_layer_attention_static launch failed: %s",
                     cudaGetErrorString(e));
  return GQA_OK;
}

// Reads (and with `clear` zeroes) the status word of the allocation-free
// calls on `device`: the bits the kernels raise (bad length, wait timeout) in
// place of a return value.  It waits for all work on that device first.  A
// device that never ran such a call reads 0.
extern "C" int gqa_static_status(int device, int* status, int clear) {
  if (!status) return set_error(GQA_ERR_INVALID_ARG, "gqa_static_status: null status");
  *status = 0;
  if (device < 0 || device >= kMaxDevices)
    return set_error(GQA_ERR_INVALID_ARG, "gqa_static_status: no device %d", device);
  {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_dev[device].ready) return GQA_OK;
  }
  int prev = -1;
  cudaError_t e = cudaGetDevice(&prev);
  if (e == cudaSuccess && prev != device) e = cudaSetDevice(device);
  int word = 0;
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e == cudaSuccess)
    e = cudaMemcpyFromSymbol(&word, g_noalloc_scratch, sizeof(int), sizeof(float) * kOffStatus,
                             cudaMemcpyDeviceToHost);
  if (e == cudaSuccess && clear) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_noalloc_scratch, &zero, sizeof(int), sizeof(float) * kOffStatus,
                           cudaMemcpyHostToDevice);
  }
  if (prev >= 0 && prev != device) cudaSetDevice(prev);
  if (e != cudaSuccess)
    return set_error(GQA_ERR_CUDA, "gqa_static_status: %s", cudaGetErrorString(e));
  *status = word;
  return GQA_OK;
}
