// Log-sum-exp merge of split partials, shared by the combine kernel
// (gqa_decode.cu) and the cross-GPU exchange kernel (gqa_exchange.cu).
//
// A partial i of row r is (m_i, l_i, o_i[128]) over a range of cache rows:
// m_i the reference max (natural-log units), l_i = sum e^(s - m_i),
// o_i = sum e^(s - m_i) v.  The merge is M = max m_i over parts with l_i > 0,
// w_i = e^(m_i - M), L = sum w_i l_i, O = sum w_i o_i -- the reference's
// segment reduce (kernel_attention_gqa.cl:378-397) with per-segment maxima.
//
// Block of kMergeGroups x 128 threads, thread (g, d) = (threadIdx.x / 128,
// threadIdx.x % 128).  Every thread first puts the o values of its first
// kMergeChunk parts in flight; meanwhile warp 0 loads every (m, l), forms M,
// the weights (in shared memory) and L.  So one L2 round trip covers up to
// kMergeGroups * kMergeChunk parts.
#pragma once

#include <math_constants.h>

#include "gqa_common.cuh"

namespace gqa {

constexpr int kMergeGroups = 4;
constexpr int kMergeChunk = 16;        // o loads in flight per thread
constexpr int kMergeLaneParts = 8;     // (m, l) pairs held per lane of warp 0
constexpr int kMergeMaxParts = 4096;

struct MergeSmem {
  float w[kMergeMaxParts];             // weights e^(m_i - M), 0 for empty parts
  float o[kMergeGroups][kHeadDim];
  float M, L;
};

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
  return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

// Merges the c.n_parts partials of row r.  On return, thread (0, d) holds
// M, L and O[d]; the other threads hold nothing useful.  Ends with the block
// synchronised; sm may be reused after the next __syncthreads.
__device__ __forceinline__ void merge_partials(const CombineParams& c, long long r, MergeSmem& sm,
                                               float& M, float& L, float& O) {
  const int d = threadIdx.x % kHeadDim, g = threadIdx.x / kHeadDim;
  const int n = c.n_parts;
  const float* o_row = c.o + r * c.o_row_stride + d;
  float ov[kMergeChunk];
#pragma unroll
  for (int u = 0; u < kMergeChunk; ++u) {
    const int i = g + u * kMergeGroups;
    ov[u] = i < n ? __ldcg(o_row + i * c.o_part_stride) : 0.f;
  }
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    const float* m_row = c.m + r * c.ml_row_stride;
    const float* l_row = c.l + r * c.ml_row_stride;
    float mr[kMergeLaneParts], lr[kMergeLaneParts];
#pragma unroll
    for (int k = 0; k < kMergeLaneParts; ++k) {
      const int i = lane + 32 * k;
      mr[k] = i < n ? __ldcg(m_row + i * c.ml_part_stride) : -CUDART_INF_F;
      lr[k] = i < n ? __ldcg(l_row + i * c.ml_part_stride) : 0.f;
    }
    float mx = -CUDART_INF_F;
#pragma unroll
    for (int k = 0; k < kMergeLaneParts; ++k)
      if (lr[k] > 0.f) mx = fmaxf(mx, mr[k]);
    for (int i = lane + 32 * kMergeLaneParts; i < n; i += 32)
      if (__ldcg(l_row + i * c.ml_part_stride) > 0.f) mx = fmaxf(mx, __ldcg(m_row + i * c.ml_part_stride));
    mx = warp_max(mx);
    float ls = 0.f;
#pragma unroll
    for (int k = 0; k < kMergeLaneParts; ++k) {
      const int i = lane + 32 * k;
      if (i < n) {
        const float w = lr[k] > 0.f ? __expf(mr[k] - mx) : 0.f;
        sm.w[i] = w;
        ls += w * lr[k];
      }
    }
    for (int i = lane + 32 * kMergeLaneParts; i < n; i += 32) {
      const float li = __ldcg(l_row + i * c.ml_part_stride);
      const float w = li > 0.f ? __expf(__ldcg(m_row + i * c.ml_part_stride) - mx) : 0.f;
      sm.w[i] = w;
      ls += w * li;
    }
    ls = warp_sum(ls);
    if (lane == 0) {
      sm.M = mx;
      sm.L = ls;
    }
  }
  __syncthreads();
  float acc = 0.f;
#pragma unroll
  for (int u = 0; u < kMergeChunk; ++u) {
    const int i = g + u * kMergeGroups;
    if (i < n) {
      const float w = sm.w[i];
      if (w != 0.f) acc += w * ov[u];
    }
  }
  for (int i0 = kMergeGroups * kMergeChunk; i0 < n; i0 += kMergeGroups * kMergeChunk) {
#pragma unroll
    for (int u = 0; u < kMergeChunk; ++u) {
      const int i = i0 + g + u * kMergeGroups;
      ov[u] = i < n ? __ldcg(o_row + i * c.o_part_stride) : 0.f;
    }
#pragma unroll
    for (int u = 0; u < kMergeChunk; ++u) {
      const int i = i0 + g + u * kMergeGroups;
      if (i < n) {
        const float w = sm.w[i];
        if (w != 0.f) acc += w * ov[u];
      }
    }
  }
  sm.o[g][d] = acc;
  __syncthreads();
  if (g == 0) {
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < kMergeGroups; ++k) s += sm.o[k][d];
    O = s;
    M = sm.M;
    L = sm.L;
  }
}

// ---------------------------------------------------------------------------
// Slice merge: dims [d0, d0 + 16) of one row over its S partials, by one
// block of 256 threads.  Every access is coalesced: half-warp hw takes parts
// hw, hw + 16, ... and its lane j dim d0 + j (one 64-byte segment per part),
// with the first kSliceChunk parts of every thread in flight before the
// weights are known; warp 0 meanwhile forms the maximum, the weights (in
// shared memory) and L from every (m, l).  The two half-warps of a warp meet
// by one shuffle and the 8 warps in shared memory.  m is in log2 units when
// m_scale is 1 and in natural-log units when it is log2(e).
constexpr int kSliceDims = 16;
constexpr int kSliceThreads = 256;
constexpr int kSliceChunk = 8;

template <int MAXP>
struct SliceSmem {
  float w[MAXP];
  float red[kSliceThreads / 32][kSliceDims];
  float L;
};

template <int MAXP>
__device__ __forceinline__ void merge_slice16(const float* o_row, long long o_part_stride,
                                              const float* m_row, const float* l_row,
                                              long long ml_part_stride, int S, float m_scale,
                                              SliceSmem<MAXP>& sm, float* out) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int hw = tid >> 4, j = tid & 15;
  constexpr int kGroups = kSliceThreads / 16;
  const float* oc = o_row + j;
  float ov[kSliceChunk];
#pragma unroll
  for (int k = 0; k < kSliceChunk; ++k) {
    const int i = hw + kGroups * k;
    ov[k] = i < S ? __ldcg(oc + (long long)i * o_part_stride) : 0.f;
  }
  if (warp == 0) {
    constexpr int kPer = 8;
    float mr[kPer], lr[kPer];
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      const int i = lane + 32 * k;
      mr[k] = i < S ? __ldcg(m_row + (long long)i * ml_part_stride) : -CUDART_INF_F;
      lr[k] = i < S ? __ldcg(l_row + (long long)i * ml_part_stride) : 0.f;
    }
    float mx = -CUDART_INF_F;
#pragma unroll
    for (int k = 0; k < kPer; ++k)
      if (lr[k] > 0.f) mx = fmaxf(mx, mr[k]);
    for (int i = lane + 32 * kPer; i < S; i += 32)
      if (__ldcg(l_row + (long long)i * ml_part_stride) > 0.f)
        mx = fmaxf(mx, __ldcg(m_row + (long long)i * ml_part_stride));
    mx = warp_max(mx);
    float ls = 0.f;
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      const int i = lane + 32 * k;
      if (i < S) {
        const float w = lr[k] > 0.f ? exp2f((mr[k] - mx) * m_scale) : 0.f;
        sm.w[i] = w;
        ls += w * lr[k];
      }
    }
    for (int i = lane + 32 * kPer; i < S; i += 32) {
      const float li = __ldcg(l_row + (long long)i * ml_part_stride);
      const float w =
          li > 0.f ? exp2f((__ldcg(m_row + (long long)i * ml_part_stride) - mx) * m_scale) : 0.f;
      sm.w[i] = w;
      ls += w * li;
    }
    ls = warp_sum(ls);
    if (lane == 0) sm.L = ls;
  }
  __syncthreads();
  float acc = 0.f;
#pragma unroll
  for (int k = 0; k < kSliceChunk; ++k) {
    const int i = hw + kGroups * k;
    if (i < S) {
      const float w = sm.w[i];
      if (w != 0.f) acc += w * ov[k];
    }
  }
  for (int i0 = kGroups * kSliceChunk; i0 < S; i0 += kGroups * kSliceChunk) {
#pragma unroll
    for (int k = 0; k < kSliceChunk; ++k) {
      const int i = i0 + hw + kGroups * k;
      ov[k] = i < S ? __ldcg(oc + (long long)i * o_part_stride) : 0.f;
    }
#pragma unroll
    for (int k = 0; k < kSliceChunk; ++k) {
      const int i = i0 + hw + kGroups * k;
      if (i < S) {
        const float w = sm.w[i];
        if (w != 0.f) acc += w * ov[k];
      }
    }
  }
  acc += __shfl_xor_sync(0xffffffffu, acc, 16);
  if (lane < 16) sm.red[warp][j] = acc;
  __syncthreads();
  if (tid < kSliceDims) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kSliceThreads / 32; ++w) s += sm.red[w][tid];
    const float L = sm.L;
    out[tid] = L > 0.f ? s / L : 0.f;
  }
}

}  // namespace gqa
