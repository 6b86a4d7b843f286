// fp32 GQA decode attention for sm_100a.
//
// Replaces the reference's five decode launches (kernel_attention_gqa.cl:149-397:
// RoPE+append, scores, softmax, segmented PV, segment reduce) by
//   decode_split_kernel : RoPE of q and of the new k (optional), KV append,
//                         QK^T, online softmax and PV over one token range of
//                         one KV head for all 6 query heads of its group, so
//                         every K/V byte is read from HBM exactly once; in its
//                         grid-merged form (GRID) the same launch also merges
//                         the ranges' partials into the final output;
//   combine_kernel /
//   combine_wide_kernel : log-sum-exp merge of the per-range partials, where
//                         the split kernel leaves partials (batches, shards,
//                         the attention blocks).
//
// Memory path.  Each CTA owns a contiguous token range of one KV head; each of
// its NW warps owns a contiguous part of that range and streams it through a
// private ring of NS stages of ST rows in shared memory with cp.async.bulk
// (1-D TMA: one copy per K tile and one per V tile, evict-first L2 hint),
// issued before the dependency wait whenever the lengths are known.
// Consecutive cache rows are contiguous ([h][t][128] layout), so a tile is
// one linear copy; no tensor map and no multicast is needed.
//
// Compute path (per warp, per ST-token stage).  q is rotated and scaled once
// per CTA into shared memory; lane l holds dims 4l..4l+3 of the 6 q heads.
// QK^T gives ST x 6 partial dot products per lane; a butterfly reduce-scatter
// leaves each lane 3 complete scores.  Softmax runs in the log2 domain with a
// lazily updated running max (rescale only when a score exceeds the max by
// more than 2^8), p is staged through a small per-warp buffer and PV
// accumulates o[6][4] per lane.  Warps are merged in shared memory at the end.
#include "gqa_common.cuh"
#include "gqa_merge.cuh"

#include <math_constants.h>

#include <type_traits>

namespace gqa {

constexpr float kRescaleThresh = 8.0f;           // log2 units
constexpr long long kWaitBudget = 2000000000LL;  // ~1 s of SM clocks per wait
constexpr float kLn2 = 0.6931471805599453f;
constexpr int kG = 6;                            // q heads per KV head

// Kernel shape: NW streaming warps per CTA, each with a private ring of NS
// stages of ST cache rows (K and V).  Instantiated shapes are listed in
// decode_variant(); the host picks one per launch.
template <int NW, int ST, int NS>
struct DecodeSmem {
  float k[NW][NS][ST * kHeadDim];
  float v[NW][NS][ST * kHeadDim];
  float cs[kHalf][2];
  float q[kG][kHeadDim];  // raw (pre-RoPE) q of the group, staged once per CTA
  float p[NW][ST][12];    // p of each token's 6 heads, each value twice (f32x2 operands)
  float wm[NW][kG];
  float lp[NW][ST][8];  // per-warp l partials, one row per owner token
  float wa[NW][kG];   // per-warp merge weights
  float wla[NW][kG];  // weight * l per warp
  float hm[kG];       // CTA max per head (log2 units)
  float hl[kG];       // CTA sum per head (cluster reduction input)
  SliceSmem<kGridMaxParts> slice;  // grid merge
  float gm[kSliceThreads / 32];    // grid merge: each merging warp's maximum (log2 units)
  float gl[kSliceThreads / 32];    // and its sum of l
  uint64_t full[NW][NS];
  int err;
  int gok;                  // grid merge: every word of the slice arrived in time
  unsigned gep;             // grid merge: this launch's epoch
  // cross-GPU exchange of a merged slice (KV-range shards)
  float xo[kSliceDims];     // this GPU's un-normalised slice sums
  float xM;                 // this GPU's slice maximum (log2 units)
  float xm[kXMaxWorld], xl[kXMaxWorld];
  float xov[kXMaxWorld][kSliceDims];
  unsigned xe;              // the slice's step epoch
  unsigned trace_slot;      // phase-trace record of this CTA (traced builds)
};

// ---------------------------------------------------------------------------
// Phase trace (opt-in build with -DGQA_PHASE_TRACE; the stamps compile to
// nothing otherwise).  Thread 0 of every CTA of the split kernel records one
// record: {tag, SM id, globaltimer at start, clock64 at start, clock64 at each
// of kPhaseEvents phase ends}; tag = (q pointer << 2) | grid-merged.  Read
// with gqa_phase_trace_read; macbook-hardware-linux-lab_b200/phase_trace.py
// turns a run of the resident decode into a per-phase table.
// ---------------------------------------------------------------------------
#ifdef GQA_PHASE_TRACE
constexpr int kPhaseEvents = 6;   // wait, q staged, loop, partial stored, poll, merge
constexpr int kPhaseWords = 4 + kPhaseEvents;
constexpr int kPhaseRecords = 1 << 16;
static __device__ unsigned long long g_phase_rec[kPhaseRecords * kPhaseWords];
static __device__ unsigned g_phase_next;
__device__ __forceinline__ unsigned long long phase_gtime() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
#define GQA_PHASE_BEGIN(slot, tag)                                                  \
  do {                                                                              \
    if (threadIdx.x == 0) {                                                         \
      unsigned s_ = atomicAdd(&g_phase_next, 1u);                                   \
      if (s_ >= (unsigned)kPhaseRecords) s_ = kPhaseRecords - 1;                    \
      unsigned smid_;                                                               \
      asm volatile("mov.u32 %0, %%smid;" : "=r"(smid_));                            \
      unsigned long long* r_ = g_phase_rec + (long long)s_ * kPhaseWords;           \
      r_[0] = (tag);                                                                \
      r_[1] = smid_;                                                                \
      r_[2] = phase_gtime();                                                        \
      r_[3] = clock64();                                                            \
      for (int e_ = 0; e_ < kPhaseEvents; ++e_) r_[4 + e_] = 0;                     \
      (slot) = s_;                                                                  \
    }                                                                               \
  } while (0)
#define GQA_PHASE(slot, ev)                                                         \
  do {                                                                              \
    if (threadIdx.x == 0)                                                           \
      g_phase_rec[(long long)(slot) * kPhaseWords + 3 + (ev)] = clock64();          \
  } while (0)
#else
#define GQA_PHASE_BEGIN(slot, tag) \
  do {                             \
  } while (0)
#define GQA_PHASE(slot, ev) \
  do {                      \
  } while (0)
#endif

// 2^x by the hardware's approximate exponential (ex2.approx.ftz: relative error
// about 2^-22, 0 for -inf), for softmax weights.
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ int ceil_div_i(int a, int b) { return (a + b - 1) / b; }
__device__ __forceinline__ int round_up_i(int a, int b) { return ceil_div_i(a, b) * b; }

// Token range of split `split` when [t_begin, t_end) is cut into n_splits
// chunks of a multiple of `quant` tokens (at least min_chunk).  The host
// planner (gqa_api.cu) uses the same rule.
__device__ __forceinline__ int chunk_tokens(int len, int n_splits, int min_chunk, int quant) {
  int c = round_up_i(ceil_div_i(len, n_splits), quant);
  return c > min_chunk ? c : min_chunk;
}

__device__ __forceinline__ void resolve_lengths(const Lengths& L, int seq, int& pos,
                                                int& seq_len) {
  if (L.pos_dev) {
    pos = *L.pos_dev;
    seq_len = pos + 1;
  } else if (L.seq_lens) {
    seq_len = L.seq_lens[seq];
    pos = seq_len - 1;
  } else {
    pos = L.pos_imm;
    seq_len = L.seqlen_imm;
  }
}

// Reduce-scatter of ST*6 partial dot products (index t*6 + h) over the 32
// lanes.  H = log2(2*ST) halving rounds at lane offsets 16, 8, ... leave each
// lane 3 complete-over-the-upper-bits sums; the remaining offsets are summed
// directly.  Lane ends up owning token t = lane >> (6 - H) and heads
// h0..h0+2 with h0 = 3 * ((lane >> (5 - H)) & 1); the 2^(5-H) lanes that differ
// only in the lowest bits hold identical copies.
template <int N, int OFF>
__device__ __forceinline__ void bfly_halve(float* v, int lane) {
  const bool up = (lane & OFF) != 0;
#pragma unroll
  for (int i = 0; i < N / 2; ++i) {
    const float send = up ? v[i] : v[i + N / 2];
    const float keep = up ? v[i + N / 2] : v[i];
    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, OFF);
  }
}

template <int ST>
struct Bfly {
  static constexpr int H = ST == 8 ? 4 : ST == 4 ? 3 : ST == 2 ? 2 : -1;
  static_assert(H > 0, "ST must be 2, 4 or 8");
  static constexpr int kLowBits = 5 - H;  // duplicate-copy bits
  __device__ __forceinline__ static void run(float* v, int lane) {
    bfly_halve<ST * 6, 16>(v, lane);
    if constexpr (H >= 2) bfly_halve<ST * 3, 8>(v, lane);
    if constexpr (H >= 3) bfly_halve<ST * 3 / 2, 4>(v, lane);
    if constexpr (H >= 4) bfly_halve<ST * 3 / 4, 2>(v, lane);
#pragma unroll
    for (int off = 1 << (kLowBits - 1); off > 0; off >>= 1) {
#pragma unroll
      for (int i = 0; i < 3; ++i) v[i] += __shfl_xor_sync(0xffffffffu, v[i], off);
    }
  }
  // Select-free form: each exchange keeps positions [0, N/2) and sends
  // [N/2, N); correct when partials are stored in the lane-permuted order
  // described at the call site.
  template <int N, int OFF>
  __device__ __forceinline__ static void halve_permuted(float* v) {
#pragma unroll
    for (int i = 0; i < N / 2; ++i) v[i] += __shfl_xor_sync(0xffffffffu, v[i + N / 2], OFF);
  }
  // The same with the adds paired into f32x2 operations (half the add
  // instructions; the sums are the same, value for value).
  template <int N, int OFF>
  __device__ __forceinline__ static void halve_permuted2(float* v) {
    constexpr int K = N / 2;
#pragma unroll
    for (int i = 0; i + 1 < K; i += 2) {
      const float2 r = make_float2(__shfl_xor_sync(0xffffffffu, v[i + K], OFF),
                                   __shfl_xor_sync(0xffffffffu, v[i + 1 + K], OFF));
      const float2 s = __fadd2_rn(make_float2(v[i], v[i + 1]), r);
      v[i] = s.x;
      v[i + 1] = s.y;
    }
    if constexpr (K % 2) v[K - 1] += __shfl_xor_sync(0xffffffffu, v[2 * K - 1], OFF);
  }
  __device__ __forceinline__ static void run_permuted(float* v) {
    halve_permuted2<ST * 6, 16>(v);
    if constexpr (H >= 2) halve_permuted2<ST * 3, 8>(v);
    if constexpr (H >= 3) halve_permuted2<ST * 3 / 2, 4>(v);
    if constexpr (H >= 4) halve_permuted2<ST * 3 / 4, 2>(v);
#pragma unroll
    for (int off = 1 << (kLowBits - 1); off > 0; off >>= 1) {
      const float2 r = make_float2(__shfl_xor_sync(0xffffffffu, v[0], off),
                                   __shfl_xor_sync(0xffffffffu, v[1], off));
      const float2 s = __fadd2_rn(make_float2(v[0], v[1]), r);
      v[2] += __shfl_xor_sync(0xffffffffu, v[2], off);
      v[0] = s.x;
      v[1] = s.y;
    }
  }
  __device__ __forceinline__ static int token(int lane) { return lane >> (6 - H); }
  __device__ __forceinline__ static int head0(int lane) { return 3 * ((lane >> (5 - H)) & 1); }
  __device__ __forceinline__ static bool owner(int lane) {
    return (lane & ((1 << kLowBits) - 1)) == 0;
  }
};

// CTAs per SM the register budget is sized for: as many as the shared memory
// footprint (two K/V rings of NW x NS x ST rows) lets reside, but never so
// many that a thread gets fewer than 128 registers (the loop holds 24 q, 24 o
// and up to 48 partial-sum registers) and at most 3.
template <int NW, int ST, int NS>
struct MinBlocks {
  static constexpr int kRingBytes = 2 * NW * NS * ST * kRowBytes;
  static constexpr int kBySmem = (227 * 1024) / (kRingBytes + 8 * 1024);
  static constexpr int kByRegs = 16 / NW;  // 65536 / (NW * 32 * 128)
  static constexpr int kMin = kBySmem < kByRegs ? kBySmem : kByRegs;
  static constexpr int value = kMin < 1 ? 1 : (kMin > 3 ? 3 : kMin);
};

// Cluster reduction of the per-CTA partials of one (sequence, KV head):
// cluster CTA r merges outputs [r*96, r*96+96) of the 6x128 over the cluster's
// CTAs through distributed shared memory and writes them as the cluster's
// partial; the last CTA to finish (arrival counter) merges all clusters'
// partials into the output and resets the counter.  Every thread of every CTA
// of the cluster calls this (it holds two cluster barriers).
template <int NT>
__device__ __forceinline__ void cluster_epilogue(const DecodeParams& p, float (*co)[kHeadDim],
                                                 float* cm, float* cl, int seq, int hkv) {
  constexpr int G = kG;
  constexpr int kOut = G * kHeadDim;  // 768 outputs per (sequence, KV head)
  const int tid = threadIdx.x;
  const int CL = p.cluster;
  const uint32_t rank = cluster_ctarank();
  const int n_cl = gridDim.x / CL;
  const int cl_id = blockIdx.x / CL;
  const int n_q = p.n_kv * G;
  __shared__ int s_last;
  __syncthreads();
  cluster_sync();  // every CTA's (cm, cl, co) is in place
  const int per = kOut / CL;
  for (int t = tid; t < per; t += NT) {
    const int idx = (int)rank * per + t;
    const int h = idx / kHeadDim, d = idx % kHeadDim;
    float mv[8], lv[8], ov[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      if (c < CL) {
        mv[c] = ld_cluster_f32(cluster_map(&cm[h], c));
        lv[c] = ld_cluster_f32(cluster_map(&cl[h], c));
        ov[c] = ld_cluster_f32(cluster_map(&co[h][d], c));
      } else {
        mv[c] = -CUDART_INF_F;
        lv[c] = 0.f;
        ov[c] = 0.f;
      }
    }
    float M = -CUDART_INF_F;
#pragma unroll
    for (int c = 0; c < 8; ++c)
      if (lv[c] > 0.f) M = fmaxf(M, mv[c]);
    float L = 0.f, O = 0.f;
    if (M != -CUDART_INF_F) {
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const float w = lv[c] > 0.f ? exp2f(mv[c] - M) : 0.f;
        L += w * lv[c];
        O += (w != 0.f) ? w * ov[c] : 0.f;
      }
    }
    const long long r = ((long long)seq * n_q + hkv * G + h) * n_cl + cl_id;
    p.part_o[r * kHeadDim + d] = O;
    if (d == 0) {
      p.part_ml[r * 2 + 0] = M;  // log2 units: consumed only below
      p.part_ml[r * 2 + 1] = L;
    }
  }
  cluster_sync();  // remote reads done before any CTA of the cluster exits

  // Arrival count over all CTAs of this (sequence, KV head).
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    const int old = atomicAdd(&p.counters[seq * p.n_kv + hkv], 1);
    s_last = (old == (int)gridDim.x - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  // All of an output's cluster partials are loaded before any is used (one
  // L2 round trip per batch of kFinalBatch clusters).
  constexpr int kFinalBatch = 16;
  for (int idx = tid; idx < kOut; idx += NT) {
    const int h = idx / kHeadDim, d = idx % kHeadDim;
    const long long r0 = ((long long)seq * n_q + hkv * G + h) * n_cl;
    float M = -CUDART_INF_F, L = 0.f, O = 0.f;
    for (int c0 = 0; c0 < n_cl; c0 += kFinalBatch) {
      float mv[kFinalBatch], lv[kFinalBatch], ov[kFinalBatch];
#pragma unroll
      for (int u = 0; u < kFinalBatch; ++u) {
        const bool ok = c0 + u < n_cl;
        const long long r = r0 + c0 + u;
        mv[u] = ok ? __ldcg(p.part_ml + r * 2) : -CUDART_INF_F;
        lv[u] = ok ? __ldcg(p.part_ml + r * 2 + 1) : 0.f;
        ov[u] = ok ? __ldcg(p.part_o + r * kHeadDim + d) : 0.f;
      }
      float bm = M;
#pragma unroll
      for (int u = 0; u < kFinalBatch; ++u)
        if (lv[u] > 0.f) bm = fmaxf(bm, mv[u]);
      if (bm == -CUDART_INF_F) continue;
      const float sc = (M == -CUDART_INF_F) ? 0.f : exp2f(M - bm);
      L *= sc;
      O *= sc;
#pragma unroll
      for (int u = 0; u < kFinalBatch; ++u) {
        const float w = lv[u] > 0.f ? exp2f(mv[u] - bm) : 0.f;
        L += w * lv[u];
        O += (w != 0.f) ? w * ov[u] : 0.f;
      }
      M = bm;
    }
    p.out[(long long)seq * p.out_stride + (long long)(hkv * G + h) * kHeadDim + d] =
        L > 0.f ? O / L : 0.f;
  }
  if (tid == 0) p.counters[seq * p.n_kv + hkv] = 0;
}

// Cross-GPU step of a merged slice (KV-range shards): store this GPU's (M, L,
// O[16]) into every GPU's inbox as tagged words at system scope, poll this
// GPU's inbox until every source's words carry the slice's step epoch, and
// write the merged output.  Thread t publishes / polls word t % 18 of GPU
// t / 18.  False (status set) when a peer's words did not arrive in time.
template <int NW, int ST, int NS>
__device__ __forceinline__ bool exchange_slice(const DecodeParams& p, DecodeSmem<NW, ST, NS>& sm,
                                               int head, int slice, int slot_id) {
  constexpr int NT = NW * 32;
  constexpr int kWords = 2 + kSliceDims;  // M, L, O[16]
  const int tid = threadIdx.x;
  const int W = p.x_world, n_q = p.n_kv * kG;
  const unsigned E = sm.xe;
  const int par = (int)(E & 1u);
  auto slot = [&](int src) {
    return ((((long long)par * W + src) * n_q + head) * kXSlices + slice) * kXSlotWords;
  };
  for (int t = tid; t < W * kWords; t += NT) {
    const int r = t / kWords, w = t % kWords;
    const float v = w == 0 ? sm.xM : (w == 1 ? sm.slice.L : sm.xo[w - 2]);
    st_tagged_sys(p.x_inbox[r] + slot(p.x_rank) + w, v, E);
  }
  const unsigned long long* own = p.x_inbox[p.x_rank];
  bool ok = true;
  for (int t = tid; t < W * kWords; t += NT) {
    const int src = t / kWords, w = t % kWords;
    const unsigned long long* a = own + slot(src) + w;
    unsigned long long v = ld_tagged_sys(a);
    if (tag_of(v) != E) {
      const long long t0 = clock64();
      while (tag_of(v) != E) {
        if (clock64() - t0 > kWaitBudget) {
          ok = false;
          break;
        }
        v = ld_tagged_sys(a);
      }
    }
    const float f = value_of(v);
    if (w == 0)
      sm.xm[src] = f;
    else if (w == 1)
      sm.xl[src] = f;
    else
      sm.xov[src][w - 2] = f;
  }
  if (!__syncthreads_and(ok)) {
    // A peer did not arrive: report it, leave the output and the epoch as they are.
    if (tid == 0) atomicOr(p.status, kStatusWaitTimeout);
    return false;
  }
  if (tid < kSliceDims) {
    float Mg = -CUDART_INF_F;
    for (int src = 0; src < W; ++src)
      if (sm.xl[src] > 0.f) Mg = fmaxf(Mg, sm.xm[src]);
    float Lg = 0.f, Og = 0.f;
    for (int src = 0; src < W; ++src) {
      if (sm.xl[src] > 0.f) {
        const float w = exp2f(sm.xm[src] - Mg);
        Lg += w * sm.xl[src];
        Og += w * sm.xov[src][tid];
      }
    }
    p.out[(long long)head * kHeadDim + slice * kSliceDims + tid] = Lg > 0.f ? Og / Lg : 0.f;
  }
  if (tid == 0) st_relaxed_gpu(p.x_epoch + slot_id, E);
  return true;
}

// Grid merge of one single-sequence launch (GRID instance).  Every CTA has
// stored its partial for its split and its 6 q heads as tagged words (value,
// epoch) at grid_words [q head][split][kGridRowWords] (o[128], m in log2
// units, l).  The 48 slices (6 q heads x 8 slices of 16 dims) of a KV head are
// merged by that KV head's CTAs, CTA `split` taking slices split, split +
// n_splits, ...  A merging thread polls (bounded) the words it needs until
// all carry this launch's epoch -- there is no barrier and no fence: a word
// whose tag is current holds its value (each word is one 64-bit access).
// Warp w takes parts 16w .. 16w + 15, two lanes per part (8 dims each, with
// the part's m and l): the warp merges its parts against its own maximum by
// shuffles alone, and the 8 warps' (M, L, O[16]) meet once in shared memory.
// Once every warp has seen every split's (m, l), every CTA of the KV head has
// read the epoch, so the merging CTA may store it back for the next launch.
template <int NW, int ST, int NS>
__device__ __forceinline__ void grid_epilogue(const DecodeParams& p, DecodeSmem<NW, ST, NS>& sm,
                                              int hkv, int split, unsigned ep) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int kMergeWarps = kSliceThreads / 32;
  constexpr int kPartsPerWarp = kGridMaxParts / kMergeWarps;
  static_assert(kPartsPerWarp == 16, "two lanes per part");
  static_assert(kSliceDims == 16, "8 dims per lane");
  static_assert(NW * 32 >= kSliceThreads, "the grid merge maps 256 threads");
  // Threads beyond the first 256 only take part in the CTA barriers.
  const bool merger = tid < kSliceThreads;
  constexpr int kSlices = kHeadDim / kSliceDims;
  const int S = p.n_splits;
  const int part = warp * kPartsPerWarp + (lane >> 1);
  const int half = lane & 1;
  const bool has = merger && part < S;
  GQA_PHASE(sm.trace_slot, 4);  // partial stored
  for (int s = split; s < kG * kSlices; s += S) {
    const int head = hkv * kG + s / kSlices;
    const int d0 = (s % kSlices) * kSliceDims;
    const unsigned long long* row =
        p.grid_words + ((long long)head * S + (has ? part : 0)) * kGridRowWords;
    if (s != split) __syncthreads();  // the previous slice's shared memory is free
    if (tid == 0) sm.gok = 1;
    const int slot_id = head * kXSlices + s % kSlices;  // the slice's exchange slot
    if (tid == 0 && p.x_inbox != nullptr) sm.xe = ld_relaxed_gpu_u32(p.x_epoch + slot_id) + 1u;

    // w[0..7]: o of dims d0 + 8 half + 0..7; w[8], w[9]: m, l.
    unsigned long long w[10];
    bool ok = true;
    if (has) {
      const unsigned long long* src[5] = {row + d0 + 8 * half, row + d0 + 8 * half + 2,
                                          row + d0 + 8 * half + 4, row + d0 + 8 * half + 6,
                                          row + kHeadDim};
#pragma unroll
      for (int k = 0; k < 5; ++k) ld_tagged2(src[k], w[2 * k], w[2 * k + 1]);
      const long long t0 = clock64();
      for (;;) {
        bool fresh = true;
#pragma unroll
        for (int k = 0; k < 5; ++k) {
          if (tag_of(w[2 * k]) != ep || tag_of(w[2 * k + 1]) != ep) {
            fresh = false;
            ld_tagged2(src[k], w[2 * k], w[2 * k + 1]);
          }
        }
        if (fresh) break;
        if (clock64() - t0 > kWaitBudget) {
          ok = false;
          break;
        }
      }
    } else {
#pragma unroll
      for (int k = 0; k < 10; ++k) w[k] = 0ull;
    }
    if (!ok) sm.gok = 0;  // benign race: every writer stores 0

    if (merger) {  // whole warps
      const float l = has ? value_of(w[9]) : 0.f;
      const float m = l > 0.f ? value_of(w[8]) : -CUDART_INF_F;
      float M = m;  // the two lanes of a part hold the same m
#pragma unroll
      for (int off = 16; off > 1; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
      const float wt = m == -CUDART_INF_F ? 0.f : exp2f(m - M);
      float Lw = half == 0 ? wt * l : 0.f;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) Lw += __shfl_xor_sync(0xffffffffu, Lw, off);
      float o[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) o[k] = wt == 0.f ? 0.f : wt * value_of(w[k]);
      // Sum over the warp's parts (lane bits 4..1), dims scattered as they go:
      // lane keeps dim 8 half + 4 b4 + 2 b3 + b2 (b = lane bits).
      bfly_halve<8, 16>(o, lane);
      bfly_halve<4, 8>(o, lane);
      bfly_halve<2, 4>(o, lane);
      o[0] += __shfl_xor_sync(0xffffffffu, o[0], 2);
      if ((lane & 2) == 0) {
        const int dim = 8 * half + 4 * ((lane >> 4) & 1) + 2 * ((lane >> 3) & 1) + ((lane >> 2) & 1);
        sm.slice.red[warp][dim] = o[0];
      }
      if (lane == 0) {
        sm.gm[warp] = M;
        sm.gl[warp] = Lw;
      }
    }
    __syncthreads();
    if (s == split) GQA_PHASE(sm.trace_slot, 5);  // every warp's slice sums in shared memory
    if (!sm.gok) {
      if (tid == 0) atomicOr(p.status, kStatusWaitTimeout);
      return;
    }
    // Every split of this KV head has stored its (m, l): all of its CTAs have
    // read the epoch, which may now advance (every merging CTA stores the
    // same value).
    if (tid == 0) st_relaxed_gpu(p.grid_epoch + hkv, ep);
    if (tid < kSliceDims) {
      float Mg = -CUDART_INF_F;
#pragma unroll
      for (int k = 0; k < kMergeWarps; ++k) Mg = fmaxf(Mg, sm.gm[k]);
      float L = 0.f, O = 0.f;
#pragma unroll
      for (int k = 0; k < kMergeWarps; ++k) {
        const float mk = sm.gm[k];
        if (mk != -CUDART_INF_F) {
          const float f = exp2f(mk - Mg);
          L += f * sm.gl[k];
          O += f * sm.slice.red[k][tid];
        }
      }
      if (p.x_inbox == nullptr) {
        p.out[(long long)head * kHeadDim + d0 + tid] = L > 0.f ? O / L : 0.f;
      } else {
        sm.xo[tid] = O;
        if (tid == 0) {
          sm.slice.L = L;
          sm.xM = Mg;
        }
      }
      if (s == split) GQA_PHASE(sm.trace_slot, 6);  // merged slice stored
    }
    if (p.x_inbox != nullptr) {
      __syncthreads();  // the slice's sums, L and M are in shared memory
      if (!exchange_slice<NW, ST, NS>(p, sm, head, s % kSlices, slot_id)) return;
    }
  }
}

template <int NW, int ST, int NS, bool FUSED, bool CLUSTER = false, bool GRID = false>
__global__ void __launch_bounds__(NW * 32, MinBlocks<NW, ST, NS>::value)
    decode_split_kernel(const DecodeParams p) {
  constexpr int G = kG;
  constexpr int NT = NW * 32;
  static_assert(NT % kHeadDim == 0, "epilogue maps threads onto head dims");
  using B = Bfly<ST>;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  DecodeSmem<NW, ST, NS>& sm = *reinterpret_cast<DecodeSmem<NW, ST, NS>*>(smem_raw);
  GQA_PHASE_BEGIN(sm.trace_slot, ((unsigned long long)(uintptr_t)p.qkv << 2) | (GRID ? 1u : 0u));

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int split = blockIdx.x, hkv = blockIdx.y, seq = blockIdx.z;
  const int n_q = p.n_kv * G;

  // Only the fused kernel streams the cache before its dependency wait, and
  // only when the host marked the lengths as stable (not produced by the
  // preceding kernel, e.g. the device pos advanced at the end of a step).
  // The unfused kernel usually follows rope_append, which writes row pos.
  const bool early = FUSED && p.lengths_stable != 0;
  // A grid-merged launch lets the next kernel's CTAs become resident (and
  // start their own cache streaming) while it runs: they are launched only
  // once every CTA of this grid is running, so they can never keep one of
  // this grid's CTAs (and with it the merge barrier) waiting for an SM.
  if constexpr (GRID) pdl_launch_dependents();
  if (!early) pdl_wait();

  int pos, seq_len;
  resolve_lengths(p.len, seq, pos, seq_len);
  const int r_end = p.t_end > 0 ? p.t_end : seq_len;
  const bool has_row = FUSED && p.skip_append == 0;  // this launch holds the new token's row
  // An empty KV-range shard (allow_empty, no row attended) is not an error.
  const bool none = p.allow_empty != 0 && r_end == p.t_begin;
  const bool bad = (!none && seq_len < 1) || seq_len > p.t_max ||
                   (has_row && (pos < 0 || pos >= p.t_max)) || p.t_begin < 0 ||
                   r_end > p.t_max || (!none && p.t_begin >= r_end);
  if (bad) {
    if (early) pdl_wait();
    if (tid == 0) atomicOr(p.status, kStatusBadLength);
    return;
  }

  const int len = r_end - p.t_begin;
  const int chunk = chunk_tokens(len, p.n_splits, p.min_chunk, p.quant);
  const int c0 = p.t_begin + split * chunk;
  const int c1 = min(c0 + chunk, r_end);
  const long long prow = ((long long)seq * n_q + hkv * G) * p.n_splits + split;

  if (!CLUSTER && !GRID && c0 >= r_end) {
    // Empty split (short sequence in a batch planned for the longest one).
    // (In cluster and grid-merge modes empty CTAs run through with no rows:
    // they must still take part in the barriers and the merge.)
    if (early) pdl_wait();
    pdl_launch_dependents();
    if (tid < G) {
      p.part_ml[(prow + (long long)tid * p.n_splits) * 2 + 0] = -CUDART_INF_F;
      p.part_ml[(prow + (long long)tid * p.n_splits) * 2 + 1] = 0.f;
    }
    return;
  }

  const int ctoks = max(c1 - c0, 0);
  const int wchunk = round_up_i(ceil_div_i(ctoks, NW), ST);
  const int w0 = c0 + warp * wchunk;
  const int w1 = min(w0 + wchunk, c1);
  const int n_tok = max(w1 - w0, 0);
  const int n_it = ceil_div_i(n_tok, ST);

  float* kc;
  float* vc;
  if (p.k_ptrs) {
    kc = p.k_ptrs[seq];
    vc = p.v_ptrs[seq];
  } else {
    kc = p.k_base + (long long)seq * p.seq_stride;
    vc = p.v_base + (long long)seq * p.seq_stride;
  }
  kc += (long long)hkv * p.t_max * kHeadDim;
  vc += (long long)hkv * p.t_max * kHeadDim;

  if (tid == 0) sm.err = 0;
  if (lane == 0) {
#pragma unroll
    for (int s = 0; s < NS; ++s) mbar_init(&sm.full[warp][s], 1);
    fence_barrier_init();
  }
  __syncwarp();

  const uint64_t policy = l2_policy_evict_first();
  auto issue = [&](int stage, int it) {
    const int t = w0 + it * ST;
    const int nt = min(ST, w1 - t);
    const uint32_t bytes = (uint32_t)nt * kRowBytes;
    mbar_arrive_expect_tx(&sm.full[warp][stage], 2 * bytes);
    bulk_copy_g2s(sm.k[warp][stage], kc + (long long)t * kHeadDim, bytes, &sm.full[warp][stage],
                  policy);
    bulk_copy_g2s(sm.v[warp][stage], vc + (long long)t * kHeadDim, bytes, &sm.full[warp][stage],
                  policy);
  };
  // Cache rows before pos are not written by the preceding kernel: stream
  // them before waiting on it.
  if (lane == 0) {
    for (int s = 0; s < NS && s < n_it; ++s) issue(s, s);
  }
  if constexpr (GRID) {
    // This launch's q and new row, read right after the dependency wait, into
    // L2 (coherent there, so a later write by the preceding kernel still wins).
    if (tid == 32 && early) {
      const float* qin = p.qkv + (long long)seq * p.qkv_stride;
      bulk_prefetch_l2(qin + (long long)hkv * G * kHeadDim, G * kRowBytes);
      bulk_prefetch_l2(qin + (long long)(n_q + hkv) * kHeadDim, kRowBytes);
      bulk_prefetch_l2(qin + (long long)(n_q + p.n_kv + hkv) * kHeadDim, kRowBytes);
    }
  }

  // RoPE angle table (cos, sin per rotation pair).  When pos is known before
  // the dependency wait, it is built while the previous kernel finishes.
  auto rope_table = [&]() {
    if (tid < kHalf) {
      float sn, cs;
      const int angle_pos = p.rope_override ? p.rope_pos : pos;
      sincosf((float)angle_pos * __ldg(p.inv_freq + tid), &sn, &cs);
      sm.cs[tid][0] = cs;
      sm.cs[tid][1] = sn;
    }
  };
  if (FUSED && early) {
    rope_table();
    __syncthreads();  // angle table complete (before the wait, off the critical path)
  }
  if (early) pdl_wait();
  if constexpr (!GRID) pdl_launch_dependents();
  GQA_PHASE(sm.trace_slot, 1);  // dependency released
  if (FUSED && !early) {
    rope_table();
    __syncthreads();
  }

  // ---- q, rotated and scaled once per CTA ----------------------------------
  // Thread 16h + k (k < 16) loads dims 4k..4k+3 and their RoPE partners
  // 64+4k..64+4k+3 of head h, applies the reference's half rotation
  // (a' = a c - b s, b' = a s + b c for the pair (i, i + 64)) and the softmax
  // scale, and stores both to sm.q; each warp then reads its lanes' dims.
  const float* qin = p.qkv + (long long)seq * p.qkv_stride;
  if (tid < G * 16) {
    const int h = tid >> 4, k = tid & 15;
    const float4* qg = reinterpret_cast<const float4*>(qin + (long long)(hkv * G + h) * kHeadDim);
    const float4 x = __ldcg(qg + k), y = __ldcg(qg + 16 + k);
    float4 xa, ya;
    if (FUSED) {
      float c[4], s[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 t = *reinterpret_cast<const float2*>(sm.cs[4 * k + j]);
        c[j] = t.x;
        s[j] = t.y;
      }
      xa = make_float4((x.x * c[0] - y.x * s[0]) * p.q_scale, (x.y * c[1] - y.y * s[1]) * p.q_scale,
                       (x.z * c[2] - y.z * s[2]) * p.q_scale, (x.w * c[3] - y.w * s[3]) * p.q_scale);
      ya = make_float4((x.x * s[0] + y.x * c[0]) * p.q_scale, (x.y * s[1] + y.y * c[1]) * p.q_scale,
                       (x.z * s[2] + y.z * c[2]) * p.q_scale, (x.w * s[3] + y.w * c[3]) * p.q_scale);
    } else {
      xa = make_float4(x.x * p.q_scale, x.y * p.q_scale, x.z * p.q_scale, x.w * p.q_scale);
      ya = make_float4(y.x * p.q_scale, y.y * p.q_scale, y.z * p.q_scale, y.w * p.q_scale);
    }
    reinterpret_cast<float4*>(sm.q[h])[k] = xa;
    reinterpret_cast<float4*>(sm.q[h])[16 + k] = ya;
  }
  // This launch's epoch for the tagged partials (read after the wait: the
  // previous launch, which may have advanced it, has finished).
  if (GRID && tid == 0) sm.gep = ld_relaxed_gpu_u32(p.grid_epoch + hkv) + 1u;
  const bool pos_attended = pos >= p.t_begin && pos < r_end;
  const bool row_writer = has_row && (pos_attended ? (pos >= w0 && pos < w1)
                                                   : (split == 0 && warp == 0));
  float4 nk = make_float4(0.f, 0.f, 0.f, 0.f), nv = nk;
  if (row_writer) {
    // The new row: lane l holds dims 4l..4l+3; the RoPE partner dims (+-64)
    // are in lane l ^ 16's load.
    const float4* kh = reinterpret_cast<const float4*>(qin + (long long)(n_q + hkv) * kHeadDim);
    nk = __ldcg(kh + lane);
    const float4 nkp = __ldcg(kh + (lane ^ 16));
    nv = __ldcg(reinterpret_cast<const float4*>(qin + (long long)(n_q + p.n_kv + hkv) *
                                                kHeadDim) + lane);
    if (FUSED) {
      float c[4], sn[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 t = *reinterpret_cast<const float2*>(sm.cs[4 * (lane & 15) + j]);
        c[j] = t.x;
        sn[j] = t.y;
      }
      const bool lo = lane < 16;
      auto rot = [&](float x, float y, int j) {
        return lo ? (x * c[j] - y * sn[j]) : (y * sn[j] + x * c[j]);
      };
      nk = make_float4(rot(nk.x, nkp.x, 0), rot(nk.y, nkp.y, 1), rot(nk.z, nkp.z, 2),
                       rot(nk.w, nkp.w, 3));
      if (!pos_attended) {
        // Not read by this launch: store it right away.
        reinterpret_cast<float4*>(kc + (long long)pos * kHeadDim)[lane] = nk;
        reinterpret_cast<float4*>(vc + (long long)pos * kHeadDim)[lane] = nv;
      }
    }
  }

  // o[h] dims 4l..4l+1 in oa[h], 4l+2..4l+3 in ob[h]: f32x2 accumulators.
  float2 oa[G], ob[G];
  float m[G];
#pragma unroll
  for (int h = 0; h < G; ++h) {
    m[h] = -CUDART_INF_F;
    oa[h] = make_float2(0.f, 0.f);
    ob[h] = make_float2(0.f, 0.f);
  }
  const int tt = B::token(lane);     // token this lane's scores belong to
  const int hb = B::head0(lane);     // first of this lane's three heads
  const bool hi = hb != 0;
  const bool own = B::owner(lane);   // one lane per (token, head triple) writes p
  __syncthreads();  // rotated q staged
  GQA_PHASE(sm.trace_slot, 2);
  // Partials are stored in a lane-dependent order -- position (tp, hp) holds
  // token tp ^ tt and head hp with its triple swapped when `hi` -- so that
  // every butterfly exchange keeps the lower half and sends the upper half
  // with no select (Bfly::run_permuted).  The q registers are swapped once.
  float2 qa[G], qb[G];  // dims 4l..4l+1 and 4l+2..4l+3 of the (swapped) heads
#pragma unroll
  for (int h = 0; h < G; ++h) {
    const float4 t = reinterpret_cast<const float4*>(sm.q[hi ? (h + 3) % G : h])[lane];
    qa[h] = make_float2(t.x, t.y);
    qb[h] = make_float2(t.z, t.w);
  }
  float lown[3] = {0.f, 0.f, 0.f};  // this owner lane's share of l for its heads
  int consumed = 0;
  bool failed = false;

  for (int it = 0; it < n_it; ++it) {
    const int s = it % NS;
    const uint32_t par = (uint32_t)(it / NS) & 1u;
    bool ok = mbar_wait_bounded(&sm.full[warp][s], par, kWaitBudget);
    ok = __all_sync(0xffffffffu, ok);
    if (!ok) {
      failed = true;
      break;
    }
    consumed = it + 1;
    const int t0 = w0 + it * ST;
    const int nt = min(ST, w1 - t0);
    float* ks = sm.k[warp][s];
    float* vs = sm.v[warp][s];

    // The row at pos is the new token's: put it into the landed stage (the
    // stale copy the transfer brought in is overwritten) and into the cache.
    if (row_writer && pos >= t0 && pos < t0 + nt) {
      reinterpret_cast<float4*>(ks + (pos - t0) * kHeadDim)[lane] = nk;
      reinterpret_cast<float4*>(vs + (pos - t0) * kHeadDim)[lane] = nv;
      reinterpret_cast<float4*>(kc + (long long)pos * kHeadDim)[lane] = nk;
      reinterpret_cast<float4*>(vc + (long long)pos * kHeadDim)[lane] = nv;
      __syncwarp();
    }

    // ---- scores: ST tokens x 6 heads, reduced over the 32 lanes ----
    float part[ST * G];
    auto scores = [&](auto full) {
#pragma unroll
      for (int tp = 0; tp < ST; ++tp) {
        const int t = tp ^ tt;
        if (decltype(full)::value || t < nt) {
          const float4 kv = reinterpret_cast<const float4*>(ks + t * kHeadDim)[lane];
          const float2 k01 = make_float2(kv.x, kv.y), k23 = make_float2(kv.z, kv.w);
#pragma unroll
          for (int h = 0; h < G; ++h) {
            const float2 d = __ffma2_rn(qb[h], k23, __fmul2_rn(qa[h], k01));
            part[tp * G + h] = d.x + d.y;
          }
        } else {
#pragma unroll
          for (int h = 0; h < G; ++h) part[tp * G + h] = 0.f;
        }
      }
    };
    if (nt == ST) scores(std::true_type{}); else scores(std::false_type{});
    B::run_permuted(part);

    float sc[3];
    const bool valid = tt < nt;
#pragma unroll
    for (int i = 0; i < 3; ++i) sc[i] = valid ? part[i] : -CUDART_INF_F;

    // ---- online softmax with lazy max update ----
    if (it == 0) {
      // Seed the running max with token 0's scores (always a valid token):
      // six broadcasts instead of a full reduction.
      const int src_hi = 1 << (5 - B::H);  // first lane holding heads 3..5 of token 0
#pragma unroll
      for (int h = 0; h < G; ++h) m[h] = __shfl_sync(0xffffffffu, sc[h % 3], h < 3 ? 0 : src_hi);
    }
    float mo[3];
#pragma unroll
    for (int i = 0; i < 3; ++i) mo[i] = hi ? m[3 + i] : m[i];
    const bool exceed = sc[0] > mo[0] + kRescaleThresh || sc[1] > mo[1] + kRescaleThresh ||
                        sc[2] > mo[2] + kRescaleThresh;
    if (__any_sync(0xffffffffu, exceed)) {
      float mx[G];
#pragma unroll
      for (int h = 0; h < G; ++h) mx[h] = ((h / 3) == (hi ? 1 : 0)) ? sc[h % 3] : -CUDART_INF_F;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
#pragma unroll
        for (int h = 0; h < G; ++h) mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], off));
      }
#pragma unroll
      for (int h = 0; h < G; ++h) {
        const float mnew = fmaxf(m[h], mx[h]);
        const float alpha = (mnew == -CUDART_INF_F) ? 1.f : fast_exp2(m[h] - mnew);
        oa[h] = __fmul2_rn(oa[h], make_float2(alpha, alpha));
        ob[h] = __fmul2_rn(ob[h], make_float2(alpha, alpha));
        if ((h / 3) == (hi ? 1 : 0)) lown[h % 3] *= alpha;
        m[h] = mnew;
      }
#pragma unroll
      for (int i = 0; i < 3; ++i) mo[i] = hi ? m[3 + i] : m[i];
    }
    float pv[3];
#pragma unroll
    for (int i = 0; i < 3; ++i) pv[i] = fast_exp2(sc[i] - mo[i]);
    if (own) {
#pragma unroll
      for (int i = 0; i < 3; ++i) {
        lown[i] += pv[i];
        *reinterpret_cast<float2*>(&sm.p[warp][tt][2 * (hb + i)]) = make_float2(pv[i], pv[i]);
      }
    }
    __syncwarp();

    // ---- o += p . V ----
    auto pv_acc = [&](auto full) {
#pragma unroll
      for (int t = 0; t < ST; ++t) {
        if (decltype(full)::value || t < nt) {
          const float4 p01 = *reinterpret_cast<const float4*>(&sm.p[warp][t][0]);
          const float4 p23 = *reinterpret_cast<const float4*>(&sm.p[warp][t][4]);
          const float4 p45 = *reinterpret_cast<const float4*>(&sm.p[warp][t][8]);
          const float4 vv = reinterpret_cast<const float4*>(vs + t * kHeadDim)[lane];
          const float2 v01 = make_float2(vv.x, vv.y), v23 = make_float2(vv.z, vv.w);
          const float2 pr[6] = {make_float2(p01.x, p01.y), make_float2(p01.z, p01.w),
                                make_float2(p23.x, p23.y), make_float2(p23.z, p23.w),
                                make_float2(p45.x, p45.y), make_float2(p45.z, p45.w)};
#pragma unroll
          for (int h = 0; h < G; ++h) {
            oa[h] = __ffma2_rn(pr[h], v01, oa[h]);
            ob[h] = __ffma2_rn(pr[h], v23, ob[h]);
          }
        }
      }
    };
    if (nt == ST) pv_acc(std::true_type{}); else pv_acc(std::false_type{});
    __syncwarp();
    if (it + NS < n_it && lane == 0) {
      fence_proxy_async_smem();
      issue(s, it + NS);
    }
  }

  GQA_PHASE(sm.trace_slot, 3);  // this warp's loop done (thread 0: warp 0)
  if (failed) {
    // Drain whatever this warp still has in flight (bounded), then report.
    const int issued = min(n_it, consumed + NS);
    for (int it = consumed; it < issued; ++it)
      (void)mbar_wait_bounded(&sm.full[warp][it % NS], (uint32_t)(it / NS) & 1u,
                              kWaitBudget / 16);
    if (lane == 0) {
      atomicOr(p.status, kStatusWaitTimeout);
      atomicOr(&sm.err, 1);
    }
  }

  // ---- per-warp (m, l, o) -> shared memory ----
  if (own) {
#pragma unroll
    for (int i = 0; i < 3; ++i) sm.lp[warp][tt][hb + i] = lown[i];
  }
  if (lane == 0) {
#pragma unroll
    for (int h = 0; h < G; ++h) sm.wm[warp][h] = m[h];
  }
  // Each warp reuses stage 0 of its own K ring (all its copies have landed).
  static_assert(NS * ST * kHeadDim >= G * kHeadDim, "K ring too small for the epilogue");
  float* ow = &sm.k[warp][0][0];
#pragma unroll
  for (int h = 0; h < G; ++h)
    reinterpret_cast<float4*>(ow + h * kHeadDim)[lane] =
        make_float4(oa[h].x, oa[h].y, ob[h].x, ob[h].y);
  __syncthreads();
  if (!CLUSTER && !GRID && sm.err) return;

  // ---- merge the warps: weights once per (warp, head), then one pass ----
  if (tid < NW * G) {
    const int h = tid % G, w = tid / G;
    float M = -CUDART_INF_F;
#pragma unroll
    for (int k = 0; k < NW; ++k) M = fmaxf(M, sm.wm[k][h]);
    const float mw = sm.wm[w][h];
    const float a = (mw == -CUDART_INF_F) ? 0.f : exp2f(mw - M);
    float lw = 0.f;  // warp w's l for head h: the sum over its owner lanes, in token order
#pragma unroll
    for (int t = 0; t < ST; ++t) lw += sm.lp[w][t][h];
    sm.wa[w][h] = a;
    sm.wla[w][h] = a == 0.f ? 0.f : a * lw;
    if (w == 0) sm.hm[h] = M;
  }
  __syncthreads();
  constexpr int NGRP = NT / kHeadDim;             // thread groups
  constexpr int GPT = (G + NGRP - 1) / NGRP;      // heads per group
  const int d = tid % kHeadDim;
  const int hg = tid / kHeadDim;
#pragma unroll
  for (int hh = 0; hh < GPT; ++hh) {
    const int h = hg * GPT + hh;
    if (h >= G) break;
    float ov[NW];
#pragma unroll
    for (int w = 0; w < NW; ++w) ov[w] = (&sm.k[w][0][0])[h * kHeadDim + d];
    float O = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      const float a = sm.wa[w][h];
      O += (a != 0.f) ? a * ov[w] : 0.f;
    }
    float Lsum = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) Lsum += sm.wla[w][h];
    const float M = sm.hm[h];
    if constexpr (CLUSTER) {
      // Keep this CTA's partial in its own shared memory (the q staging area
      // is free by now) for the cluster reduction below.
      sm.q[h][d] = O;
      if (d == 0) sm.hl[h] = (sm.err || M == -CUDART_INF_F) ? 0.f : Lsum;
    } else if constexpr (GRID) {
      // Tagged words, m in log2 units: the grid merge below is the only
      // reader.  A CTA that failed publishes an empty partial (m = -inf,
      // l = 0), which the merge gives weight 0.
      unsigned long long* row =
          p.grid_words + ((long long)(hkv * G + h) * p.n_splits + split) * kGridRowWords;
      const unsigned ep = sm.gep;
      const bool empty = sm.err || M == -CUDART_INF_F;
      st_tagged(row + d, O, ep);
      if (d == 0) {
        st_tagged(row + kHeadDim, empty ? -CUDART_INF_F : M, ep);
        st_tagged(row + kHeadDim + 1, empty ? 0.f : Lsum, ep);
      }
    } else if (p.out != nullptr && p.n_splits == 1) {
      p.out[(long long)seq * p.out_stride + (long long)(hkv * G + h) * kHeadDim + d] =
          Lsum > 0.f ? O / Lsum : 0.f;
    } else {
      const long long r = prow + (long long)h * p.n_splits;
      p.part_o[r * kHeadDim + d] = O;
      if (d == 0) {
        p.part_ml[r * 2 + 0] = M * kLn2;  // natural-log units outside this kernel
        p.part_ml[r * 2 + 1] = Lsum;
      }
    }
  }
  if constexpr (CLUSTER) cluster_epilogue<NT>(p, sm.q, sm.hm, sm.hl, seq, hkv);
  if constexpr (GRID) grid_epilogue<NW, ST, NS>(p, sm, hkv, split, sm.gep);
}

// Log-sum-exp merge of n_parts partials per output row (merge_partials in
// gqa_merge.cuh): one CTA of kMergeGroups x 128 threads per row.
__global__ void __launch_bounds__(kHeadDim * kMergeGroups) combine_kernel(const CombineParams c) {
  __shared__ MergeSmem sm;
  const int h = blockIdx.x, seq = blockIdx.y;
  const int d = threadIdx.x % kHeadDim, g = threadIdx.x / kHeadDim;
  const long long r = (long long)seq * c.rows_per_seq + h;
  // The next kernel is released once this grid runs (after its wait), not
  // before: released earlier, its CTAs would sit in their own wait holding
  // SM space the split kernel still running ahead of this one needs (a
  // trace showed the next grid's tail stretched by ~5 us).  It waits for
  // this grid before it reads or writes anything this grid touches.
  pdl_wait();
  pdl_launch_dependents();
  // The split kernel has finished reading the lengths (the wait above).
  if (c.advance_lens != nullptr && h == 0 && threadIdx.x == 0) c.advance_lens[seq] += 1;
  float M, L, O;
  merge_partials(c, r, sm, M, L, O);
  if (g != 0) return;
  float* dst = c.out + (long long)seq * c.out_stride + (long long)h * kHeadDim;
  if (c.out_m) {
    dst[d] = O;
    if (d == 0) {
      c.out_m[r] = M;
      c.out_l[r] = L;
    }
  } else {
    dst[d] = L > 0.f ? O / L : 0.f;
  }
}

// Single-sequence combine over many CTAs: CTA (slice, q head, sequence)
// merges dims [16 slice, +16) of that head's output over its split partials
// (merge_slice16: coalesced loads, one L2 round trip).  Used where there are
// few output rows, so that the merge's loads spread over 8 x rows CTAs.
__global__ void __launch_bounds__(kSliceThreads) combine_wide_kernel(const CombineParams c) {
  __shared__ SliceSmem<kMergeMaxParts> sm;
  const int slice = blockIdx.x, h = blockIdx.y, seq = blockIdx.z;
  const long long r = (long long)seq * c.rows_per_seq + h;
  pdl_wait();  // released after the wait, as combine_kernel
  pdl_launch_dependents();
  const int d0 = slice * kSliceDims;
  merge_slice16<kMergeMaxParts>(c.o + r * c.o_row_stride + d0, c.o_part_stride,
                                c.m + r * c.ml_row_stride, c.l + r * c.ml_row_stride,
                                c.ml_part_stride, c.n_parts, 1.4426950408889634f, sm,
                                c.out + (long long)seq * c.out_stride + (long long)h * kHeadDim +
                                    d0);
}

// RoPE on every q head (in place) and every k head of one new token per
// sequence, with the rotated k and raw v written to cache row pos: the
// reference's kernel_rope_and_kv_append (kernel_attention_gqa.cl:149-194) for
// a batch of sequences.  One CTA per sequence, one thread per rotation pair.
__global__ void __launch_bounds__(kHalf) rope_append_kernel(
    float* qkv, long long qkv_stride, float* const* k_ptrs, float* const* v_ptrs, float* k_base,
    float* v_base, long long seq_stride, Lengths len, int t_max, int n_q, int n_kv,
    const float* inv_freq, int* status) {
  const int seq = blockIdx.x, i = threadIdx.x;
  pdl_wait();
  pdl_launch_dependents();
  int pos, seq_len;
  resolve_lengths(len, seq, pos, seq_len);
  if (pos < 0 || pos >= t_max) {
    if (i == 0) atomicOr(status, kStatusBadLength);
    return;
  }
  float* q = qkv + (long long)seq * qkv_stride;
  const float* k = q + (long long)n_q * kHeadDim;
  const float* v = k + (long long)n_kv * kHeadDim;
  float* kc = k_ptrs ? k_ptrs[seq] : k_base + (long long)seq * seq_stride;
  float* vc = v_ptrs ? v_ptrs[seq] : v_base + (long long)seq * seq_stride;
  float sn, cs;
  sincosf((float)pos * inv_freq[i], &sn, &cs);
  for (int h = 0; h < n_q; ++h) {
    float* qh = q + (long long)h * kHeadDim;
    const float q0 = qh[i], q1 = qh[i + kHalf];
    qh[i] = q0 * cs - q1 * sn;
    qh[i + kHalf] = q0 * sn + q1 * cs;
  }
  for (int h = 0; h < n_kv; ++h) {
    const float k0 = k[h * kHeadDim + i], k1 = k[h * kHeadDim + i + kHalf];
    const long long row = ((long long)h * t_max + pos) * kHeadDim;
    kc[row + i] = k0 * cs - k1 * sn;
    kc[row + i + kHalf] = k0 * sn + k1 * cs;
    vc[row + i] = v[h * kHeadDim + i];
    vc[row + i + kHalf] = v[h * kHeadDim + i + kHalf];
  }
}

// Advances every sequence's length by one after a batched step whose split
// kernel wrote the outputs itself (no combine launch to do it).
__global__ void advance_lens_kernel(int* lens, int n) {
  pdl_wait();
  pdl_launch_dependents();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    lens[i] += 1;
}

// Advances the device-side position after a replayed decode step, wrapping
// from wrap_hi back to wrap_lo (a fixed window of positions can then be
// replayed indefinitely).
__global__ void advance_pos_kernel(int* pos, int wrap_lo, int wrap_hi) {
  pdl_wait();
  int nxt = *pos + 1;
  if (wrap_hi > wrap_lo && nxt >= wrap_hi) nxt = wrap_lo;
  *pos = nxt;
}

// Seeded N(0,1) fill: element i is one half of the Box-Muller pair i/2 drawn
// from two counter-indexed splitmix64 outputs.  The same sequence is produced
// on the host by the package's seeded.py, so device-filled and host-filled
// tensors of the same (seed, stream) hold the same distribution; bit-equality
// with the host is not promised (double-precision log/cos may differ in the
// last ulp).
__device__ __forceinline__ uint64_t splitmix_mix(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
  return z ^ (z >> 31);
}

__global__ void fill_normal_kernel(float* dst, long long n, uint64_t key, long long offset) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const long long e = i + offset;
    const uint64_t j = (uint64_t)(e >> 1);
    const uint64_t r1 = splitmix_mix(key + (2 * j + 1) * 0x9E3779B97F4A7C15ULL);
    const uint64_t r2 = splitmix_mix(key + (2 * j + 2) * 0x9E3779B97F4A7C15ULL);
    const double u1 = ((double)(r1 >> 11) + 1.0) * (1.0 / 9007199254740992.0);
    const double u2 = (double)(r2 >> 11) * (1.0 / 9007199254740992.0);
    const double rad = sqrt(-2.0 * log(u1));
    const double ang = 6.283185307179586 * u2;
    dst[i] = (float)((e & 1) ? rad * sin(ang) : rad * cos(ang));
  }
}

// ---------------------------------------------------------------------------
// Host-side launchers (C++; the C ABI in gqa_api.cu validates and calls these)
// ---------------------------------------------------------------------------
// Instantiated kernel shapes (warps, rows per stage, stages).  Variant 0 is
// the default; the others exist for tuning and are selected per context.
struct Variant {
  const void* fused;
  const void* unfused;
  const void* fused_cluster;
  const void* fused_grid;  // grid-merged instance (null where not built)
  int threads;
  int quant;
  int grid_quant;          // row quantum of a grid-merged split
  size_t smem;
};

template <int NW, int ST, int NS, bool WITH_GRID = false>
static Variant make_variant() {
  Variant v;
  v.fused = (const void*)decode_split_kernel<NW, ST, NS, true>;
  v.unfused = (const void*)decode_split_kernel<NW, ST, NS, false>;
  v.fused_cluster = (const void*)decode_split_kernel<NW, ST, NS, true, true>;
  v.fused_grid = nullptr;
  if constexpr (WITH_GRID)
    v.fused_grid = (const void*)decode_split_kernel<NW, ST, NS, true, false, true>;
  v.threads = NW * 32;
  v.quant = NW * ST > 32 ? NW * ST : 32;
  v.grid_quant = ST;
  v.smem = sizeof(DecodeSmem<NW, ST, NS>);
  return v;
}

static const Variant& decode_variant(int i) {
  static const Variant table[] = {
      make_variant<8, 4, 3, true>(),  // 0: 256 threads, 12 KB ring per warp, 2 CTAs/SM
      make_variant<4, 8, 3>(),  // 1: 128 threads, 24 KB ring per warp, 2 CTAs/SM
      make_variant<4, 4, 4>(),  // 2: 128 threads, 16 KB ring per warp, 3 CTAs/SM
      make_variant<8, 8, 2, true>(),  // 3: 256 threads, 32 KB ring per warp, 1 CTA/SM
      make_variant<8, 2, 4>(),  // 4: 256 threads,  8 KB ring per warp, 2-3 CTAs/SM
      make_variant<16, 4, 2, true>(), // 5: 512 threads,  8 KB ring per warp, 1 CTA/SM
      make_variant<16, 2, 3>(), // 6: 512 threads,  6 KB ring per warp, 1 CTA/SM
  };
  constexpr int n = sizeof(table) / sizeof(table[0]);
  return table[(i >= 0 && i < n) ? i : 0];
}

// Copies up to max_records phase-trace records (kPhaseWords words each) to
// host memory; returns how many were recorded (-1: a build without the trace).
int phase_trace_read(unsigned long long* host, int max_records, bool reset) {
#ifdef GQA_PHASE_TRACE
  unsigned n = 0;
  if (cudaMemcpyFromSymbol(&n, g_phase_next, sizeof(n)) != cudaSuccess) return -2;
  if (n > (unsigned)kPhaseRecords) n = kPhaseRecords;
  const int copy = (int)n < max_records ? (int)n : max_records;
  if (host && copy > 0 &&
      cudaMemcpyFromSymbol(host, g_phase_rec, sizeof(unsigned long long) * kPhaseWords * copy) !=
          cudaSuccess)
    return -2;
  if (reset) {
    const unsigned zero = 0;
    if (cudaMemcpyToSymbol(g_phase_next, &zero, sizeof(zero)) != cudaSuccess) return -2;
  }
  return (int)n;
#else
  (void)host;
  (void)max_records;
  (void)reset;
  return -1;
#endif
}

int decode_variant_count() { return 7; }
int decode_variant_quant(int i) { return decode_variant(i).quant; }
int decode_variant_grid_quant(int i) { return decode_variant(i).grid_quant; }

// CTAs of the grid-merged instance of variant i that fit on one SM (0: not
// built).  The grid merge's barrier needs every CTA of a launch resident at
// once, so a launch may use at most n_sm x this many CTAs.
int decode_grid_ctas_per_sm(int i) {
  const Variant& v = decode_variant(i);
  if (!v.fused_grid) return 0;
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, v.fused_grid, v.threads, v.smem) !=
      cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

static cudaError_t launch_ex(const void* fn, dim3 grid, dim3 block, size_t smem,
                             cudaStream_t st, bool pdl, void** args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelExC(&cfg, fn, args);
}

cudaError_t prepare_decode_kernels() {
  for (int i = 0; i < decode_variant_count(); ++i) {
    const Variant& v = decode_variant(i);
    cudaError_t e = cudaFuncSetAttribute(v.fused, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)v.smem);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(v.unfused, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)v.smem);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(v.fused_cluster, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)v.smem);
    if (e == cudaSuccess && v.fused_grid)
      e = cudaFuncSetAttribute(v.fused_grid, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)v.smem);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

cudaError_t launch_decode_split(const DecodeParams& p, int n_seq, bool fused, cudaStream_t st,
                                bool pdl, int variant) {
  const Variant& v = decode_variant(variant);
  dim3 grid(p.n_splits, p.n_kv, n_seq);
  DecodeParams copy = p;
  copy.quant = v.quant;
  void* args[] = {&copy};
  if (p.grid_words != nullptr) {
    // Grid-merged single-sequence launch: the output is final when it ends.
    if (!fused || n_seq != 1 || !v.fused_grid || p.n_splits < 1 ||
        p.n_splits > kGridMaxParts || p.out == nullptr)
      return cudaErrorInvalidValue;
    copy.quant = v.grid_quant;
    return launch_ex(v.fused_grid, grid, dim3(v.threads), v.smem, st, pdl, args);
  }
  if (p.cluster > 1) {
    if (!fused || p.n_splits % p.cluster != 0 || p.cluster > 8) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(v.threads);
    cfg.dynamicSmemBytes = v.smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)p.cluster;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 2 : 1;
    return cudaLaunchKernelExC(&cfg, v.fused_cluster, args);
  }
  return launch_ex(fused ? v.fused : v.unfused, grid, dim3(v.threads), v.smem, st, pdl, args);
}

cudaError_t launch_combine(const CombineParams& c, int n_seq, cudaStream_t st, bool pdl) {
  dim3 grid(c.rows_per_seq, n_seq);
  CombineParams copy = c;
  void* args[] = {&copy};
  return launch_ex((const void*)combine_kernel, grid, dim3(kHeadDim * kMergeGroups), 0, st, pdl,
                   args);
}

cudaError_t launch_combine_wide(const CombineParams& c, int n_seq, cudaStream_t st, bool pdl) {
  if (c.out_m != nullptr || c.n_parts > kMergeMaxParts) return cudaErrorInvalidValue;
  dim3 grid(kHeadDim / kSliceDims, c.rows_per_seq, n_seq);
  CombineParams copy = c;
  void* args[] = {&copy};
  return launch_ex((const void*)combine_wide_kernel, grid, dim3(kSliceThreads), 0, st, pdl, args);
}

cudaError_t launch_rope_append(float* qkv, long long qkv_stride, float* const* k_ptrs,
                               float* const* v_ptrs, float* k_base, float* v_base,
                               long long seq_stride, Lengths len, int t_max, int n_q, int n_kv,
                               const float* inv_freq, int* status, int n_seq, cudaStream_t st,
                               bool pdl) {
  void* args[] = {&qkv, &qkv_stride, (void*)&k_ptrs, (void*)&v_ptrs, &k_base, &v_base,
                  &seq_stride, &len, &t_max, &n_q, &n_kv, (void*)&inv_freq, &status};
  return launch_ex((const void*)rope_append_kernel, dim3(n_seq), dim3(kHalf), 0, st, pdl, args);
}

cudaError_t launch_advance_lens(int* lens, int n, cudaStream_t st, bool pdl) {
  void* args[] = {&lens, &n};
  return launch_ex((const void*)advance_lens_kernel, dim3((n + 255) / 256), dim3(256), 0, st, pdl,
                   args);
}

cudaError_t launch_advance_pos(int* pos, int wrap_lo, int wrap_hi, cudaStream_t st, bool pdl) {
  void* args[] = {&pos, &wrap_lo, &wrap_hi};
  return launch_ex((const void*)advance_pos_kernel, dim3(1), dim3(1), 0, st, pdl, args);
}

cudaError_t launch_fill_normal(float* dst, long long n, uint64_t key, long long offset,
                               int n_sm, cudaStream_t st) {
  long long blocks = (n + 255) / 256;
  const long long cap = (long long)n_sm * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  fill_normal_kernel<<<(unsigned)blocks, 256, 0, st>>>(dst, n, key, offset);
  return cudaGetLastError();
}

}  // namespace gqa
