// The GQA decode step for model shapes other than the one the tuned kernels
// are built for (head_dim 128, 6 query heads per KV head, gqa_decode.cu):
// Qwen2.5-0.5B's head_dim 64 with 7 query heads per KV head
// (generate_stream_05b.c:19-31; its attention kernels,
// kernel_decoder_layer_05b.cl:142-380, are the 1.5B ones at these sizes).
// Same math as the reference: RoPE on pairs (i, i + D/2) with
// theta_i = pos * base^(-2i/D), the new K row (rotated) and V row appended at
// pos, s = (q . k) * (1 / sqrt(D)) over rows t < seq_len, a stable softmax and
// the PV product; here split over KV ranges and merged by log-sum-exp.
//
//   split_generic_kernel        one CTA per (split, KV head): its first tile's
//                               cache rows requested (cp.async) before the
//                               dependency wait when the step's position is
//                               not produced by the preceding kernel -- rows
//                               below pos are never written by it; RoPE of its
//                               KV head's q heads into shared memory (the
//                               caller's qkv stays as given), and on the CTA
//                               whose range holds pos the new K (rotated) and
//                               V rows into the caches -- the reference's
//                               kernel_rope_and_kv_append, one thread per pair;
//                               then its rows in tiles
//                               of 64 staged in shared memory by coalesced
//                               16-byte async copies; scores of the G heads per row
//                               (thread = row x head set, float4 reads rotated
//                               per row so a warp's 32 rows hit different banks),
//                               a per-tile max and exp, then PV with one thread
//                               per (head, dim) output; running (m, l, o) per head
//   merge_generic_kernel        one CTA per q head: the splits' (m, l, o) merged
//                               by log-sum-exp into the output row, all loads
//                               of a round in flight at once
#include "gqa_common.cuh"

#include <math_constants.h>

namespace gqa {

constexpr int kGenThreads = 256;
constexpr int kGenTile = 64;            // rows per shared-memory tile
constexpr int kGenMaxSplits = 1024;

template <int D, int G>
struct GenShape {
  static constexpr int kChunks = D / 4;                 // float4 per row
  static constexpr int kOut = G * D;                    // outputs per KV head
  static constexpr int kOutPerThread = (kOut + kGenThreads - 1) / kGenThreads;
  static constexpr int kHeadSets = kGenThreads / kGenTile;          // 4
  static constexpr int kHeadsPerThread = (G + kHeadSets - 1) / kHeadSets;
  static_assert(D % 4 == 0 && D <= 128, "head_dim");
  static_assert(kGenThreads % kGenTile == 0, "tile");
};

struct GenParams {
  const float* q;    // [n_q][D] new token, before RoPE
  const float* k;    // [n_kv][D] new token
  const float* v;
  float* k_cache;    // [n_kv][t_max][D]
  float* v_cache;
  Lengths len;
  int t_max, n_q, n_kv, n_splits, rows_per_split;
  int lengths_stable;     // pos / seq_len not written by the preceding kernel
  const float* inv_freq;  // [D / 2]
  float scale;            // 1 / sqrt(D)
  float* part_o;          // [n_q][n_splits][D]
  float* part_ml;         // [n_q][n_splits][2]
  float* out;             // [n_q][D]
  int* status;
};

// pos and seq_len of the step (from device memory when len.pos_dev is set,
// seq_len = pos + 1 then); false when they leave the cache.
__device__ __forceinline__ bool gen_lengths(const GenParams& p, int& pos, int& seq_len) {
  if (p.len.pos_dev) {
    pos = *p.len.pos_dev;
    seq_len = pos + 1;
  } else {
    pos = p.len.pos_imm;
    seq_len = p.len.seqlen_imm;
  }
  return pos >= 0 && pos < p.t_max && seq_len >= 1 && seq_len <= p.t_max;
}

template <int D, int G>
struct GenSmem {
  float q[G][D];            // rotated q of the KV head's G q heads
  float knew[D], vnew[D];   // the new row (owner CTA only)
  float k[kGenTile][D];
  float v[kGenTile][D];
  float s[G][kGenTile];     // scores, then weights e^(s - m)
  float m[G], corr[G];      // running max per head, rescale of this tile
  float l[G];               // running sum of the weights per head
};

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src)
               : "memory");
}

// Rows [tb, tb + nrow) of the KV head's K and V into the tile buffers, as
// 16-byte async copies (one commit group; cp.async.wait_all completes it).
template <int D, int G>
__device__ __forceinline__ void gen_issue_tile(GenSmem<D, G>& sm, const float* kc,
                                               const float* vc, int tb, int nrow, int tid) {
  using S = GenShape<D, G>;
  for (int i = tid; i < nrow * S::kChunks; i += kGenThreads) {
    const int r = i / S::kChunks, c = i % S::kChunks;
    cp_async16(&sm.k[r][4 * c], kc + (long long)(tb + r) * D + 4 * c);
    cp_async16(&sm.v[r][4 * c], vc + (long long)(tb + r) * D + 4 * c);
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
}

template <int D, int G>
__global__ void __launch_bounds__(kGenThreads) split_generic_kernel(const GenParams p) {
  using S = GenShape<D, G>;
  __shared__ __align__(16) GenSmem<D, G> sm;
  // With stable lengths the first tile is requested before the dependency
  // wait: the preceding kernel (the previous layer's merge, a projection, the
  // embedding) writes neither pos nor this layer's cache, and the split that
  // wrote row pos - 1 finished before it could start.  Row pos itself, which
  // this kernel appends, is replaced in shared memory below.
  const bool early = p.lengths_stable != 0;
  if (!early) pdl_wait();
  int pos, seq_len;
  if (!gen_lengths(p, pos, seq_len)) {
    if (early) pdl_wait();
    pdl_launch_dependents();
    if (blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0)
      atomicOr(p.status, kStatusBadLength);
    return;
  }
  constexpr int H = D / 2;
  const int split = blockIdx.x, hkv = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int t0 = split * p.rows_per_split;
  const int t1 = min(seq_len, t0 + p.rows_per_split);
  float* kc = p.k_cache + (long long)hkv * p.t_max * D;
  float* vc = p.v_cache + (long long)hkv * p.t_max * D;
  // The split whose range holds pos (the last one when pos lies past them
  // all) appends the new row; only it may attend that row.
  const bool owner = split == min(pos / p.rows_per_split, p.n_splits - 1);
  if (t0 < t1) gen_issue_tile(sm, kc, vc, t0, min(kGenTile, t1 - t0), tid);
  if (early) pdl_wait();
  pdl_launch_dependents();

  // ---- RoPE: theta_i = pos * inv_freq[i], pairs (i, i + D/2); each thread
  // takes its own angles, so these loads share a round trip with the first
  // tile's (the tile's barrier publishes sm.q) ----
  for (int i = tid; i < G * H; i += kGenThreads) {
    const int g = i / H, j = i % H;
    const float* qh = p.q + (long long)(hkv * G + g) * D;
    const float q0 = qh[j], q1 = qh[j + H];
    float sn, cs;
    sincosf((float)pos * p.inv_freq[j], &sn, &cs);
    sm.q[g][j] = q0 * cs - q1 * sn;
    sm.q[g][j + H] = q0 * sn + q1 * cs;
  }
  if (owner && tid < H) {
    const float k0 = p.k[hkv * D + tid], k1 = p.k[hkv * D + tid + H];
    float sn, cs;
    sincosf((float)pos * p.inv_freq[tid], &sn, &cs);
    const float kr0 = k0 * cs - k1 * sn, kr1 = k0 * sn + k1 * cs;
    const float v0 = p.v[hkv * D + tid], v1 = p.v[hkv * D + tid + H];
    kc[(long long)pos * D + tid] = kr0;
    kc[(long long)pos * D + tid + H] = kr1;
    vc[(long long)pos * D + tid] = v0;
    vc[(long long)pos * D + tid + H] = v1;
    sm.knew[tid] = kr0;
    sm.knew[tid + H] = kr1;
    sm.vnew[tid] = v0;
    sm.vnew[tid + H] = v1;
  }
  if (tid < G) {
    sm.m[tid] = -CUDART_INF_F;
    sm.l[tid] = 0.f;
  }
  float o[S::kOutPerThread];
#pragma unroll
  for (int k = 0; k < S::kOutPerThread; ++k) o[k] = 0.f;

  for (int tb = t0; tb < t1; tb += kGenTile) {
    const int nrow = min(kGenTile, t1 - tb);
    // ---- the tile's K and V rows (the first tile's were requested above;
    // the previous tile's buffers are free after the loop's last barrier) ----
    if (tb != t0) gen_issue_tile(sm, kc, vc, tb, nrow, tid);
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();
    if (owner && pos >= tb && pos < tb + nrow) {  // the row just appended, as written
      for (int i = tid; i < D; i += kGenThreads) {
        sm.k[pos - tb][i] = sm.knew[i];
        sm.v[pos - tb][i] = sm.vnew[i];
      }
      __syncthreads();
    }
    // ---- scores: thread (set, r) takes heads set, set + 4, ... of row r ----
    {
      const int r = tid % kGenTile, set = tid / kGenTile;
      float acc[S::kHeadsPerThread];
#pragma unroll
      for (int j = 0; j < S::kHeadsPerThread; ++j) acc[j] = 0.f;
      if (r < nrow) {
#pragma unroll 4
        for (int cc = 0; cc < S::kChunks; ++cc) {
          const int c = (cc + r) % S::kChunks;  // rotated: the warp's rows on different banks
          const float4 kv = reinterpret_cast<const float4*>(&sm.k[r][0])[c];
#pragma unroll
          for (int j = 0; j < S::kHeadsPerThread; ++j) {
            const int g = set + j * S::kHeadSets;
            if (g < G) {
              const float4 qv = reinterpret_cast<const float4*>(&sm.q[g][0])[c];
              acc[j] = fmaf(qv.x, kv.x, fmaf(qv.y, kv.y, fmaf(qv.z, kv.z, fmaf(qv.w, kv.w, acc[j]))));
            }
          }
        }
      }
#pragma unroll
      for (int j = 0; j < S::kHeadsPerThread; ++j) {
        const int g = set + j * S::kHeadSets;
        if (g < G) sm.s[g][r] = r < nrow ? acc[j] * p.scale : -CUDART_INF_F;
      }
    }
    __syncthreads();
    // ---- per-head tile max -> new running max and the rescale factor ----
    for (int g = warp; g < G; g += kGenThreads / 32) {
      float mx = fmaxf(sm.s[g][lane], sm.s[g][lane + 32]);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      if (lane == 0) {
        const float m_new = fmaxf(sm.m[g], mx);
        sm.corr[g] = sm.m[g] == -CUDART_INF_F ? 0.f : expf(sm.m[g] - m_new);
        sm.m[g] = m_new;
      }
    }
    __syncthreads();
    // ---- weights e^(s - m) ----
    for (int i = tid; i < G * kGenTile; i += kGenThreads) {
      const int g = i / kGenTile, r = i % kGenTile;
      const float sv = sm.s[g][r];
      sm.s[g][r] = sv == -CUDART_INF_F ? 0.f : expf(sv - sm.m[g]);
    }
    __syncthreads();
    // ---- l: warp g sums head g's weights (rows past nrow weigh 0) ----
    for (int g = warp; g < G; g += kGenThreads / 32) {
      float ls = sm.s[g][lane] + sm.s[g][lane + 32];
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) ls += __shfl_xor_sync(0xffffffffu, ls, off);
      if (lane == 0) sm.l[g] = sm.l[g] * sm.corr[g] + ls;
    }
    // ---- PV: thread owns outputs tid + k * kGenThreads = (g, d); four
    // independent chains over the rows ----
#pragma unroll
    for (int k = 0; k < S::kOutPerThread; ++k) {
      const int idx = tid + k * kGenThreads;
      if (idx < S::kOut) {
        const int g = idx / D, d = idx % D;
        float a0 = o[k] * sm.corr[g], a1 = 0.f, a2 = 0.f, a3 = 0.f;
        int r = 0;
        for (; r + 4 <= nrow; r += 4) {
          a0 = fmaf(sm.s[g][r], sm.v[r][d], a0);
          a1 = fmaf(sm.s[g][r + 1], sm.v[r + 1][d], a1);
          a2 = fmaf(sm.s[g][r + 2], sm.v[r + 2][d], a2);
          a3 = fmaf(sm.s[g][r + 3], sm.v[r + 3][d], a3);
        }
        for (; r < nrow; ++r) a0 = fmaf(sm.s[g][r], sm.v[r][d], a0);
        o[k] = (a0 + a1) + (a2 + a3);
      }
    }
    __syncthreads();
  }

  // ---- the split's partial: (m, l, un-normalised o) per q head ----
  const int qh0 = hkv * G;
#pragma unroll
  for (int k = 0; k < S::kOutPerThread; ++k) {
    const int idx = tid + k * kGenThreads;
    if (idx < S::kOut) {
      const int g = idx / D, d = idx % D;
      p.part_o[((long long)(qh0 + g) * p.n_splits + split) * D + d] = o[k];
    }
  }
  if (tid < G) {
    float* ml = p.part_ml + ((long long)(qh0 + tid) * p.n_splits + split) * 2;
    ml[0] = t1 > t0 ? sm.m[tid] : -CUDART_INF_F;
    ml[1] = t1 > t0 ? sm.l[tid] : 0.f;
  }
}

// One CTA of kGenThreads per q head: every split's (m, l) loaded at once by
// the first threads, the weights e^(m_i - M) formed in shared memory while
// each group of D threads has its splits' o values in flight, then the groups'
// sums added.
template <int D>
__global__ void __launch_bounds__(kGenThreads) merge_generic_kernel(const GenParams p) {
  constexpr int kGroups = kGenThreads / D;
  constexpr int kInFlight = 16;                    // o loads in flight per thread
  __shared__ float w[kGenMaxSplits];
  __shared__ float osum[kGroups][D];
  __shared__ float wmax[kGenThreads / 32], wsum[kGenThreads / 32];
  pdl_wait();
  pdl_launch_dependents();
  int pos, seq_len;
  if (!gen_lengths(p, pos, seq_len)) return;
  const int h = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int d = tid % D, grp = tid / D, n = p.n_splits;
  const float* ml = p.part_ml + (long long)h * n * 2;
  const float* po = p.part_o + (long long)h * n * D + d;
  // this thread's first o values (splits grp, grp + kGroups, ...), in flight
  float ov[kInFlight];
#pragma unroll
  for (int u = 0; u < kInFlight; ++u) {
    const int i = grp + u * kGroups;
    ov[u] = i < n ? __ldcg(po + (long long)i * D) : 0.f;
  }
  // M = max m_i over splits with l_i > 0
  float mx = -CUDART_INF_F;
  for (int i = tid; i < n; i += kGenThreads)
    if (__ldcg(ml + 2 * i + 1) > 0.f) mx = fmaxf(mx, __ldcg(ml + 2 * i));
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  if (lane == 0) wmax[warp] = mx;
  __syncthreads();
  float M = wmax[0];
#pragma unroll
  for (int k = 1; k < kGenThreads / 32; ++k) M = fmaxf(M, wmax[k]);
  // weights and L = sum w_i l_i
  float ls = 0.f;
  for (int i = tid; i < n; i += kGenThreads) {
    const float li = __ldcg(ml + 2 * i + 1);
    const float wi = (li > 0.f && M != -CUDART_INF_F) ? expf(__ldcg(ml + 2 * i) - M) : 0.f;
    w[i] = wi;
    ls = fmaf(wi, li, ls);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ls += __shfl_xor_sync(0xffffffffu, ls, off);
  if (lane == 0) wsum[warp] = ls;
  __syncthreads();
  float O = 0.f;
#pragma unroll
  for (int u = 0; u < kInFlight; ++u) {
    const int i = grp + u * kGroups;
    if (i < n && w[i] != 0.f) O = fmaf(w[i], ov[u], O);
  }
  for (int i0 = kInFlight * kGroups; i0 < n; i0 += kInFlight * kGroups) {
#pragma unroll
    for (int u = 0; u < kInFlight; ++u) {
      const int i = i0 + grp + u * kGroups;
      ov[u] = i < n ? __ldcg(po + (long long)i * D) : 0.f;
    }
#pragma unroll
    for (int u = 0; u < kInFlight; ++u) {
      const int i = i0 + grp + u * kGroups;
      if (i < n && w[i] != 0.f) O = fmaf(w[i], ov[u], O);
    }
  }
  osum[grp][d] = O;
  __syncthreads();
  if (grp == 0) {
    float L = 0.f, S = 0.f;
#pragma unroll
    for (int k = 0; k < kGenThreads / 32; ++k) L += wsum[k];
#pragma unroll
    for (int k = 0; k < kGroups; ++k) S += osum[k][d];
    p.out[(long long)h * D + d] = L > 0.f ? S / L : 0.f;
  }
}

// ---------------------------------------------------------------------------
// Launcher: split (with RoPE and the append), merge, chained by programmatic
// dependent launch.
// ---------------------------------------------------------------------------
template <typename K>
static cudaError_t gen_launch(K kernel, dim3 grid, dim3 block, const GenParams& p,
                              cudaStream_t st, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  GenParams copy = p;
  void* args[] = {&copy};
  return cudaLaunchKernelExC(&cfg, (const void*)kernel, args);
}

bool generic_shape_built(int head_dim, int group) { return head_dim == 64 && group == 7; }

int generic_max_splits() { return kGenMaxSplits; }

// Splits for a cache of up to plan_len rows: at least one tile each, enough
// CTAs to cover the device twice.
int generic_plan_splits(int n_kv, int plan_len, int n_sm) {
  int by_rows = (plan_len + kGenTile - 1) / kGenTile;
  int by_sms = (2 * n_sm + n_kv - 1) / n_kv;
  int s = by_rows < by_sms ? by_rows : by_sms;
  if (s < 1) s = 1;
  return s > kGenMaxSplits ? kGenMaxSplits : s;
}

cudaError_t launch_generic_attention(const float* qkv, float* out, float* k_cache, float* v_cache,
                                     Lengths len, int t_max, int n_q, int n_kv, int head_dim,
                                     int n_splits, int plan_len, const float* inv_freq,
                                     float* part_o, float* part_ml, int* status, cudaStream_t st,
                                     bool pdl_first, bool pdl, bool lengths_stable) {
  if (head_dim != 64 || n_q != 7 * n_kv) return cudaErrorInvalidValue;
  constexpr int D = 64, G = 7;
  GenParams p{};
  p.q = qkv;
  p.k = qkv + (long long)n_q * D;
  p.v = p.k + (long long)n_kv * D;
  p.k_cache = k_cache;
  p.v_cache = v_cache;
  p.len = len;
  p.t_max = t_max;
  p.n_q = n_q;
  p.n_kv = n_kv;
  p.n_splits = n_splits;
  // rows per split: whole tiles, covering plan_len rows
  const int per = (plan_len + n_splits - 1) / n_splits;
  p.rows_per_split = (per + kGenTile - 1) / kGenTile * kGenTile;
  p.lengths_stable = lengths_stable ? 1 : 0;
  p.inv_freq = inv_freq;
  p.scale = 1.0f / sqrtf((float)D);
  p.part_o = part_o;
  p.part_ml = part_ml;
  p.out = out;
  p.status = status;
  cudaError_t e = gen_launch(split_generic_kernel<D, G>, dim3(n_splits, n_kv),
                             dim3(kGenThreads), p, st, pdl_first);
  if (e == cudaSuccess)
    e = gen_launch(merge_generic_kernel<D>, dim3(n_q), dim3(kGenThreads), p, st, pdl);
  return e;
}

}  // namespace gqa
