// Cross-GPU log-sum-exp exchange for a KV-range-split decode step, fused with
// the merge it feeds.
//
// One long sequence's cache rows are cut into contiguous ranges, one per GPU.
// Each GPU runs the split kernel over its range (gqa_decode.cu), then this
// kernel, one CTA per q head:
//   1. merges this GPU's split partials into one (m, l, o) for the head
//      (merge_partials, as in combine_kernel);
//   2. stores that triple straight into the inbox of every GPU of the group
//      (peer memory mapped through CUDA IPC, stores over NVLink), each value
//      as one 64-bit word {value, step epoch};
//   3. polls (bounded) its own inbox until every source's words carry this
//      step's epoch, and merges the world triples into the head's output.
// Each word is written and read by one 64-bit scalar access, which is
// single-copy atomic, so a word whose epoch is current holds its value: no
// fence and no separate flag is needed.
// This is the reference's split-K segment reduce (kernel_attention_gqa.cl:
// 378-397) stretched over several GPUs, with the all-gather done by the
// merging kernel itself instead of a collective library call.
//
// Steps are told apart by a per-head epoch kept on the device (so graph
// replays advance it); inbox slots alternate by epoch parity.  A GPU cannot
// run two steps ahead of a peer: its step e+1 waits for the peer's step-e+1
// words, which the peer stores only after its step-e kernel (and every read
// of the slots it reuses) has finished.
#include "gqa_common.cuh"
#include "gqa_merge.cuh"

#include <math_constants.h>

namespace gqa {

constexpr int kExSlot = 130;        // 8-byte words per (source, head) slot: m, l, o[128]
constexpr int kExGroups = kMergeGroups;  // groups of 128 threads
constexpr long long kExWaitBudget = 2000000000LL;  // ~1 s of SM clocks
constexpr int kExMaxWorld = 32;
constexpr int kExPerGroup = kExMaxWorld / kExGroups;  // sources gathered by one group

struct ExchangeParams {
  CombineParams local;          // this GPU's split partials (n_parts may be 0)
  uint2* const* inbox;          // [world] -> that GPU's slots [2][world][n_rows][kExSlot]
  unsigned* epoch;              // [n_rows] steps done by this GPU, per head
  int rank, world;
  float* out;                   // [n_rows][128]
  int* status;
};

// One word {value (low half), epoch (high half)}, stored and loaded as a single
// 64-bit scalar at system scope.  A scalar access is single-copy atomic, so a
// reader that sees the epoch of a store sees its value too.  (A .v2.u32 pair
// would not do: the memory model treats a vector access as separate scalar
// accesses, so a reader could pair a new epoch with an old value.)
__device__ __forceinline__ void st_word(uint2* p, float v, unsigned e) {
  const unsigned long long w = ((unsigned long long)e << 32) | __float_as_uint(v);
  asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}

__device__ __forceinline__ uint2 ld_word(const uint2* p) {
  unsigned long long w;
  asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
  return make_uint2((unsigned)w, (unsigned)(w >> 32));
}

// Reloads word w from p until its epoch reaches e; false if that takes past
// the deadline.
__device__ __forceinline__ bool settle_word(const uint2* p, unsigned e, long long deadline,
                                            uint2& w) {
  while ((int)(w.y - e) < 0) {
    if (clock64() > deadline) return false;
    w = ld_word(p);
  }
  return true;
}

__global__ void __launch_bounds__(kHeadDim * kExGroups) exchange_combine_kernel(
    const ExchangeParams x) {
  __shared__ MergeSmem sm;
  __shared__ float s_o[kExGroups][kHeadDim];
  __shared__ float s_m[kExGroups], s_l[kExGroups];
  __shared__ float s_wm[kExMaxWorld], s_wl[kExMaxWorld];  // every source's m and l
  const CombineParams& c = x.local;
  const int h = blockIdx.x, n_rows = c.rows_per_seq;
  const int d = threadIdx.x % kHeadDim, g = threadIdx.x / kHeadDim;
  pdl_launch_dependents();
  pdl_wait();

  // ---- 1. merge this GPU's split partials (m in natural-log units) ----
  float Mt = -CUDART_INF_F, Lt = 0.f, Ot = 0.f;
  merge_partials(c, h, sm, Mt, Lt, Ot);

  const unsigned e = x.epoch[h] + 1u;  // only this CTA advances epoch[h]
  const int par = e & 1u;

  // ---- 2. publish (M, L, O) of this GPU to every GPU's inbox ----
  if (g == 0) {
    const long long slot = ((long long)(par * x.world + x.rank) * n_rows + h) * kExSlot;
    for (int dst = 0; dst < x.world; ++dst) {
      uint2* p = x.inbox[dst] + slot;
      st_word(p + 2 + d, Ot, e);
      if (d == 0) {
        st_word(p, Mt, e);
        st_word(p + 1, Lt, e);
      }
    }
  }

  // ---- 3./4. gather every source's words of this step and merge them ----
  // The o words of a thread's sources (spread over the 4 groups) are all
  // loaded before any is checked; meanwhile one thread per (source, m or l)
  // settles those words into shared memory.  Stale words are re-polled.
  const uint2* base = x.inbox[x.rank] + (long long)par * x.world * n_rows * kExSlot +
                      (long long)h * kExSlot;
  const long long src_stride = (long long)n_rows * kExSlot;
  uint2 wo[kExPerGroup];
#pragma unroll
  for (int k = 0; k < kExPerGroup; ++k) {
    const int src = g + k * kExGroups;
    if (src < x.world) wo[k] = ld_word(base + src * src_stride + 2 + d);
  }
  const long long deadline = clock64() + kExWaitBudget;
  bool ok = true;
  if (threadIdx.x < 2 * x.world) {
    const int src = threadIdx.x % x.world, which = threadIdx.x / x.world;  // 0: m, 1: l
    const uint2* p = base + src * src_stride + which;
    uint2 w = ld_word(p);
    ok = settle_word(p, e, deadline, w);
    (which ? s_wl : s_wm)[src] = __uint_as_float(w.x);
  }
  if (!__syncthreads_and(ok)) {
    if (threadIdx.x == 0) atomicOr(x.status, kStatusWaitTimeout);
    return;
  }
  float Mg = -CUDART_INF_F;
#pragma unroll
  for (int k = 0; k < kExPerGroup; ++k) {
    const int src = g + k * kExGroups;
    if (src < x.world && s_wl[src] > 0.f) Mg = fmaxf(Mg, s_wm[src]);
  }
  float Lg = 0.f, Og = 0.f;
#pragma unroll
  for (int k = 0; k < kExPerGroup; ++k) {
    const int src = g + k * kExGroups;
    if (src < x.world && ok) {
      ok = settle_word(base + src * src_stride + 2 + d, e, deadline, wo[k]);
      if (s_wl[src] > 0.f) {
        const float w = expf(s_wm[src] - Mg);
        Lg += w * s_wl[src];
        Og += w * __uint_as_float(wo[k].x);
      }
    }
  }
  __syncthreads();  // the publish step above has finished reading s_m / s_l / s_o
  s_o[g][d] = Og;
  if (d == 0) {
    s_m[g] = Mg;
    s_l[g] = Lg;
  }
  if (!__syncthreads_and(ok)) {
    // A peer did not arrive: report it, leave out and epoch untouched.
    if (threadIdx.x == 0) atomicOr(x.status, kStatusWaitTimeout);
    return;
  }
  if (g == 0) {
    float Mw = -CUDART_INF_F;
#pragma unroll
    for (int k = 0; k < kExGroups; ++k) Mw = fmaxf(Mw, s_m[k]);
    float Lw = 0.f, Ow = 0.f;
    if (Mw != -CUDART_INF_F) {
#pragma unroll
      for (int k = 0; k < kExGroups; ++k) {
        const float w = (s_m[k] == -CUDART_INF_F) ? 0.f : expf(s_m[k] - Mw);
        Lw += w * s_l[k];
        Ow += (w != 0.f) ? w * s_o[k][d] : 0.f;
      }
    }
    x.out[(long long)h * kHeadDim + d] = Lw > 0.f ? Ow / Lw : 0.f;
  }
  if (threadIdx.x == 0) x.epoch[h] = e;
}

size_t exchange_inbox_bytes(int world, int n_rows) {
  return sizeof(uint2) * 2ull * world * n_rows * kExSlot;
}

cudaError_t launch_exchange_combine(const CombineParams& local, uint2* const* inbox,
                                    unsigned* epoch, int rank, int world, float* out, int* status,
                                    cudaStream_t st, bool pdl) {
  ExchangeParams x{};
  x.local = local;
  x.inbox = inbox;
  x.epoch = epoch;
  x.rank = rank;
  x.world = world;
  x.out = out;
  x.status = status;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(local.rows_per_seq);
  cfg.blockDim = dim3(kHeadDim * kExGroups);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  void* args[] = {&x};
  return cudaLaunchKernelExC(&cfg, (const void*)exchange_combine_kernel, args);
}

}  // namespace gqa
