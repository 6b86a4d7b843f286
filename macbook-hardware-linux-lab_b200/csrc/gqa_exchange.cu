// Cross-GPU log-sum-exp exchange for a KV-range-split decode step, fused with
// the merge it feeds.
//
// One long sequence's cache rows are cut into contiguous ranges, one per GPU.
// Each GPU runs the split kernel over its range (gqa_decode.cu), then this
// kernel, one CTA per q head:
//   1. merges this GPU's split partials into one (m, l, o) for the head
//      (the same log-sum-exp merge as combine_kernel);
//   2. stores that triple straight into the inbox of every GPU of the group
//      (peer memory mapped through CUDA IPC, stores over NVLink), each value
//      as one 8-byte word {value, step epoch};
//   3. polls (bounded) its own inbox until every source's words carry this
//      step's epoch, and merges the world triples into the head's output.
// An aligned 8-byte store is never seen half-written, so a word whose epoch
// is current holds its value: no fence and no separate flag is needed.
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

#include <math_constants.h>

namespace gqa {

constexpr int kExSlot = 130;        // 8-byte words per (source, head) slot: m, l, o[128]
constexpr int kExGroups = 4;        // local merge: groups of 128 threads over the split parts
constexpr int kExBatch = 16;        // parts loaded per group before any is used
constexpr long long kExWaitBudget = 2000000000LL;  // ~1 s of SM clocks

struct ExchangeParams {
  CombineParams local;          // this GPU's split partials (n_parts may be 0)
  uint2* const* inbox;          // [world] -> that GPU's slots [2][world][n_rows][kExSlot]
  unsigned* epoch;              // [n_rows] steps done by this GPU, per head
  int rank, world;
  float* out;                   // [n_rows][128]
  int* status;
};

// One word {value, epoch}, stored and loaded whole at system scope.
__device__ __forceinline__ void st_word(uint2* p, float v, unsigned e) {
  asm volatile("st.relaxed.sys.global.v2.u32 [%0], {%1, %2};" ::"l"(p), "r"(__float_as_uint(v)),
               "r"(e) : "memory");
}

__device__ __forceinline__ uint2 ld_word(const uint2* p) {
  uint2 v;
  asm volatile("ld.relaxed.sys.global.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p)
               : "memory");
  return v;
}

// Value of word p once its epoch reaches e; false if that takes past deadline.
__device__ __forceinline__ bool wait_word(const uint2* p, unsigned e, long long deadline,
                                          float& v) {
  uint2 w = ld_word(p);
  while ((int)(w.y - e) < 0) {
    if (clock64() > deadline) return false;
    w = ld_word(p);
  }
  v = __uint_as_float(w.x);
  return true;
}

__global__ void __launch_bounds__(kHeadDim * kExGroups) exchange_combine_kernel(
    const ExchangeParams x) {
  __shared__ float s_o[kExGroups][kHeadDim];
  __shared__ float s_m[kExGroups], s_l[kExGroups];
  const CombineParams& c = x.local;
  const int h = blockIdx.x, n_rows = c.rows_per_seq;
  const int d = threadIdx.x % kHeadDim, g = threadIdx.x / kHeadDim;
  pdl_launch_dependents();
  pdl_wait();

  // ---- 1. merge this GPU's split partials (m in natural-log units) ----
  float M = -CUDART_INF_F, L = 0.f, O = 0.f;
  for (int i0 = g; i0 < c.n_parts; i0 += kExGroups * kExBatch) {
    float mv[kExBatch], lv[kExBatch], ov[kExBatch];
#pragma unroll
    for (int u = 0; u < kExBatch; ++u) {
      const int i = i0 + u * kExGroups;
      const bool in = i < c.n_parts;
      mv[u] = in ? __ldcg(c.m + i * c.ml_part_stride + h * c.ml_row_stride) : -CUDART_INF_F;
      lv[u] = in ? __ldcg(c.l + i * c.ml_part_stride + h * c.ml_row_stride) : 0.f;
      ov[u] = in ? __ldcg(c.o + i * c.o_part_stride + h * c.o_row_stride + d) : 0.f;
    }
    float bm = M;
#pragma unroll
    for (int u = 0; u < kExBatch; ++u)
      if (lv[u] > 0.f) bm = fmaxf(bm, mv[u]);
    if (bm == -CUDART_INF_F) continue;
    const float sc = (M == -CUDART_INF_F) ? 0.f : expf(M - bm);
    L *= sc;
    O *= sc;
#pragma unroll
    for (int u = 0; u < kExBatch; ++u) {
      const float w = lv[u] > 0.f ? expf(mv[u] - bm) : 0.f;
      L += w * lv[u];
      O += (w != 0.f) ? w * ov[u] : 0.f;
    }
    M = bm;
  }
  s_o[g][d] = O;
  if (d == 0) {
    s_m[g] = M;
    s_l[g] = L;
  }
  __syncthreads();

  const unsigned e = x.epoch[h] + 1u;  // only this CTA advances epoch[h]
  const int par = e & 1u;

  // ---- 2. publish (M, L, O) of this GPU to every GPU's inbox ----
  if (g == 0) {
    float Mt = -CUDART_INF_F;
#pragma unroll
    for (int k = 0; k < kExGroups; ++k) Mt = fmaxf(Mt, s_m[k]);
    float Lt = 0.f, Ot = 0.f;
    if (Mt != -CUDART_INF_F) {
#pragma unroll
      for (int k = 0; k < kExGroups; ++k) {
        const float w = (s_m[k] == -CUDART_INF_F) ? 0.f : expf(s_m[k] - Mt);
        Lt += w * s_l[k];
        Ot += (w != 0.f) ? w * s_o[k][d] : 0.f;
      }
    }
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

  // ---- 3./4. wait for every source's words of this step and merge them ----
  bool ok = true;
  float Ow = 0.f, Lw = 0.f;
  if (g == 0) {
    const uint2* base = x.inbox[x.rank] + (long long)par * x.world * n_rows * kExSlot +
                        (long long)h * kExSlot;
    const long long src_stride = (long long)n_rows * kExSlot;
    const long long deadline = clock64() + kExWaitBudget;
    float Mw = -CUDART_INF_F;
    for (int s = 0; s < x.world && ok; ++s) {
      float ms, ls;
      ok = wait_word(base + s * src_stride, e, deadline, ms) &&
           wait_word(base + s * src_stride + 1, e, deadline, ls);
      if (ok && ls > 0.f) Mw = fmaxf(Mw, ms);
    }
    for (int s = 0; s < x.world && ok; ++s) {
      float ms, ls, os;
      ok = wait_word(base + s * src_stride, e, deadline, ms) &&
           wait_word(base + s * src_stride + 1, e, deadline, ls) &&
           wait_word(base + s * src_stride + 2 + d, e, deadline, os);
      if (ok && ls > 0.f) {
        const float w = expf(ms - Mw);
        Lw += w * ls;
        Ow += w * os;
      }
    }
  }
  if (!__syncthreads_and(ok)) {
    // A peer did not arrive: report it, leave out and epoch untouched.
    if (threadIdx.x == 0) atomicOr(x.status, kStatusWaitTimeout);
    return;
  }
  if (g == 0) x.out[(long long)h * kHeadDim + d] = Lw > 0.f ? Ow / Lw : 0.f;
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
