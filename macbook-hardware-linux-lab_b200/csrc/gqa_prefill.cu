// bf16 causal prefill for sm_100a on the 5th-generation tensor cores.
//
// The reference has no prefill: it feeds a prompt through its decode layer
// call one token at a time (qwen_server.c:957-964, generate_stream.c:740-749),
// i.e. causal attention computed row by row in fp32.  Here a whole prompt is
// processed at once:
//
//   prefill_prep_kernel  RoPE of q and k in fp32 (the reference's half
//                        rotation, angle pos * inv_freq with the host-made
//                        inverse frequencies), conversion to bf16, and the
//                        tiles written as ready-made shared-memory images:
//                        128 rows x 128 (K dimension) bf16, K-major, 128-byte
//                        swizzle (two 64-wide blocks of 16 KB); V is written
//                        transposed (rows = head dim, K = key) so both MMA
//                        operands are K-major.  The fp32 rotated K rows and
//                        raw V rows are also appended to the decode caches.
//   prefill_attn_kernel  one CTA per (128-query tile, q head, sequence);
//                        warp 4 streams Q once and K / V^T tiles into a
//                        double buffer with 1-D bulk copies; warp 5 owns the
//                        tensor memory (S double-buffered in 2 x 128 columns,
//                        O in 128 columns) and issues tcgen05.mma
//                        (kind::f16, bf16 operands, fp32 accumulation,
//                        M = N = 128); warps 0-3 run the online softmax with
//                        one query row per thread (tcgen05.ld of its row, no
//                        shuffles), a lazily updated running max, rescale of
//                        its O row in tensor memory only when the max moves
//                        by more than 2^8, and P written as a bf16 swizzled
//                        operand for the P.V^T MMA.
//
// Every wait is bounded; on a timeout the CTA raises a status bit, drains
// what it issued and frees its tensor memory.
#include <cuda_bf16.h>
#include <math_constants.h>

#include "gqa_common.cuh"

namespace gqa {

constexpr int kPT = 128;                          // tile rows (queries or keys)
constexpr int kImgElems = kPT * kHeadDim;         // one tile image (bf16 elements)
constexpr int kImgBytes = kImgElems * 2;          // 32 KB
constexpr int kKBlockElems = kPT * 64;            // one 64-wide K block (16 KB)
constexpr int kPrefillThreads = 192;              // warps 0-3 softmax, 4 loader, 5 MMA
constexpr int kTmemCols = 512;                    // S0 | S1 | O (| unused)
constexpr long long kPrefillWaitBudget = 2000000000LL;

// Element offset of (row r, k) in a 128 x 128 bf16 K-major image with the
// 128-byte swizzle: 16-byte chunk c of row r is stored at chunk c ^ (r % 8)
// within its 8-row, 1 KB atom; the two 64-wide K blocks follow each other.
__device__ __forceinline__ int sw_offset(int r, int k) {
  return (k >> 6) * kKBlockElems + (r >> 3) * 512 + (r & 7) * 64 +
         ((((k & 63) >> 3) ^ (r & 7)) << 3) + (k & 7);
}

// ---------------------------------------------------------------------------
// tcgen05 helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint64_t umma_smem_desc(uint32_t saddr) {
  // start address (>>4), leading byte offset 16 B (unused by swizzled
  // K-major operands), stride byte offset 1024 B (between 8-row groups),
  // descriptor version 1, layout SWIZZLE_128B (2).
  uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Instruction descriptor: kind::f16 with bf16 A and B (both K-major), fp32
// accumulator, M = 128, N = 128.
constexpr uint32_t kIdescBf16M128N128 =
    (1u << 4) | (1u << 7) | (1u << 10) | ((128u >> 3) << 17) | ((128u >> 4) << 24);

__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t a, uint64_t b, bool acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(a), "l"(b), "r"(kIdescBf16M128N128), "r"((uint32_t)acc));
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
               ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// 32 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n\t"
      // The destination registers are written asynchronously: wait in the
      // same statement so no use can be scheduled before the data is there.
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};\n\t"
      "tcgen05.wait::st.sync.aligned;"
      ::"r"(taddr), "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])),
        "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])),
        "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
        "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])),
        "r"(__float_as_uint(v[11])), "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])),
        "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])),
        "r"(__float_as_uint(v[17])), "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])),
        "r"(__float_as_uint(v[20])), "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])),
        "r"(__float_as_uint(v[23])), "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])),
        "r"(__float_as_uint(v[26])), "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])),
        "r"(__float_as_uint(v[29])), "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
}

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// ---------------------------------------------------------------------------
// Prep: RoPE, bf16, swizzled tile images, cache append
// ---------------------------------------------------------------------------
struct PrefillPrepParams {
  const float* qkv;      // [n_seq][S][(n_q + 2 n_kv) * 128]
  long long seq_stride;  // floats between sequences
  int S;
  int n_q, n_kv;
  const float* inv_freq;
  __nv_bfloat16* qimg;   // [n_seq][n_q][S/128] images
  __nv_bfloat16* kimg;   // [n_seq][n_kv][S/128] images
  __nv_bfloat16* vimg;   // [n_seq][n_kv][S/128] images (transposed)
  float* const* k_caches;  // optional [n_seq] fp32 caches [n_kv][t_max][128]
  float* const* v_caches;
  int t_max;
};

__global__ void __launch_bounds__(256) prefill_prep_kernel(const PrefillPrepParams p) {
  __shared__ float cs[kHalf][2];
  const int s = blockIdx.x, seq = blockIdx.y, tid = threadIdx.x;
  if (tid < kHalf) {
    float sn, c;
    sincosf((float)s * p.inv_freq[tid], &sn, &c);
    cs[tid][0] = c;
    cs[tid][1] = sn;
  }
  __syncthreads();
  const int width = (p.n_q + 2 * p.n_kv) * kHeadDim;
  const float* row = p.qkv + (long long)seq * p.seq_stride + (long long)s * width;
  const int n_tiles = p.S / kPT;
  const int tile = s / kPT, r = s % kPT;
  float* kc = p.k_caches ? p.k_caches[seq] : nullptr;
  float* vc = p.v_caches ? p.v_caches[seq] : nullptr;
  // q and k heads: one rotation pair per thread-iteration
  for (int idx = tid; idx < (p.n_q + p.n_kv) * kHalf; idx += blockDim.x) {
    const int hh = idx / kHalf, i = idx % kHalf;
    const float x0 = row[hh * kHeadDim + i], x1 = row[hh * kHeadDim + i + kHalf];
    const float c = cs[i][0], sn = cs[i][1];
    const float y0 = x0 * c - x1 * sn;
    const float y1 = x0 * sn + x1 * c;
    if (hh < p.n_q) {
      __nv_bfloat16* img =
          p.qimg + ((long long)(seq * p.n_q + hh) * n_tiles + tile) * kImgElems;
      img[sw_offset(r, i)] = __float2bfloat16_rn(y0);
      img[sw_offset(r, i + kHalf)] = __float2bfloat16_rn(y1);
    } else {
      const int kh = hh - p.n_q;
      __nv_bfloat16* img =
          p.kimg + ((long long)(seq * p.n_kv + kh) * n_tiles + tile) * kImgElems;
      img[sw_offset(r, i)] = __float2bfloat16_rn(y0);
      img[sw_offset(r, i + kHalf)] = __float2bfloat16_rn(y1);
      if (kc) {
        float* dst = kc + ((long long)kh * p.t_max + s) * kHeadDim;
        dst[i] = y0;
        dst[i + kHalf] = y1;
      }
    }
  }
  // v heads: transposed image (row = head dim, K = key within the tile)
  for (int idx = tid; idx < p.n_kv * kHeadDim; idx += blockDim.x) {
    const int kh = idx / kHeadDim, d = idx % kHeadDim;
    const float x = row[(p.n_q + p.n_kv + kh) * kHeadDim + d];
    __nv_bfloat16* img = p.vimg + ((long long)(seq * p.n_kv + kh) * n_tiles + tile) * kImgElems;
    img[sw_offset(d, r)] = __float2bfloat16_rn(x);
    if (vc) vc[((long long)kh * p.t_max + s) * kHeadDim + d] = x;
  }
}

// ---------------------------------------------------------------------------
// Attention
// ---------------------------------------------------------------------------
struct PrefillAttnParams {
  const __nv_bfloat16* qimg;
  const __nv_bfloat16* kimg;
  const __nv_bfloat16* vimg;
  float* out;            // [n_seq][S][n_q * 128]
  int S;
  int n_q, n_kv;
  float scale_log2;      // softmax scale * log2(e)
  int* status;
};

struct PrefillSmem {
  __nv_bfloat16 q[kImgElems];
  __nv_bfloat16 k[2][kImgElems];
  __nv_bfloat16 vt[2][kImgElems];
  __nv_bfloat16 p[kImgElems];
  uint64_t q_full, kv_full[2], kv_empty[2], s_full[2], s_empty[2], p_full, o_done;
  uint32_t tmem_base;
  int err;
};

constexpr size_t prefill_smem_bytes() { return sizeof(PrefillSmem) + 1024; }  // + alignment slack

__global__ void __launch_bounds__(kPrefillThreads, 1) prefill_attn_kernel(const PrefillAttnParams p) {
  extern __shared__ unsigned char smem_raw[];
  // The swizzled operand images need 1 KB alignment.
  PrefillSmem& sm = *reinterpret_cast<PrefillSmem*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_tiles = p.S / kPT;
  const int i = n_tiles - 1 - (int)blockIdx.x;  // heaviest (longest causal) tiles first
  const int hq = blockIdx.y, seq = blockIdx.z;
  const int kvh = hq / (p.n_q / p.n_kv);
  const int n_kv_tiles = i + 1;

  if (tid == 0) {
    mbar_init(&sm.q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sm.kv_full[s], 1);
      mbar_init(&sm.kv_empty[s], 1);
      mbar_init(&sm.s_full[s], 1);
      mbar_init(&sm.s_empty[s], 128);
    }
    mbar_init(&sm.p_full, 128);
    mbar_init(&sm.o_done, 1);
    sm.err = 0;
    fence_barrier_init();
  }
  if (warp == 5) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 ::"r"(smem_addr(&sm.tmem_base)), "r"(kTmemCols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  const uint32_t tmem_s[2] = {tmem, tmem + 128};
  const uint32_t tmem_o = tmem + 256;

  const long long q_off = ((long long)(seq * p.n_q + hq) * n_tiles + i) * kImgElems;
  const long long kv_base = (long long)(seq * p.n_kv + kvh) * n_tiles * kImgElems;

  if (warp == 4) {
    // ---- loader ----
    if (lane == 0) {
      const uint64_t policy = l2_policy_evict_first();
      mbar_arrive_expect_tx(&sm.q_full, kImgBytes);
      bulk_copy_g2s(sm.q, p.qimg + q_off, kImgBytes, &sm.q_full, policy);
      for (int j = 0; j < n_kv_tiles; ++j) {
        const int st = j & 1;
        if (j >= 2 && !mbar_wait_bounded(&sm.kv_empty[st], ((j >> 1) - 1) & 1,
                                         kPrefillWaitBudget)) {
          atomicOr(&sm.err, 1);
          break;
        }
        mbar_arrive_expect_tx(&sm.kv_full[st], 2 * kImgBytes);
        // K and V tiles are re-read by the other q heads of the group: keep them in L2.
        asm volatile(
            "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
            ::"r"(smem_addr(sm.k[st])), "l"(p.kimg + kv_base + (long long)j * kImgElems),
              "r"(kImgBytes), "r"(smem_addr(&sm.kv_full[st])) : "memory");
        asm volatile(
            "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
            ::"r"(smem_addr(sm.vt[st])), "l"(p.vimg + kv_base + (long long)j * kImgElems),
              "r"(kImgBytes), "r"(smem_addr(&sm.kv_full[st])) : "memory");
      }
    }
    __syncwarp();  // the other lanes wait here, so the warp reaches the block barrier converged
  } else if (warp == 5) {
    // ---- MMA issuer ----
    if (lane == 0) {
      bool ok = mbar_wait_bounded(&sm.q_full, 0, kPrefillWaitBudget);
      const uint32_t q_addr = smem_addr(sm.q);
      auto issue_s = [&](int j) -> bool {
        const int st = j & 1;
        if (!mbar_wait_bounded(&sm.kv_full[st], (j >> 1) & 1, kPrefillWaitBudget)) return false;
        if (j >= 2 && !mbar_wait_bounded(&sm.s_empty[st], ((j >> 1) - 1) & 1, kPrefillWaitBudget))
          return false;
        tc_fence_after();
        const uint32_t k_addr = smem_addr(sm.k[st]);
#pragma unroll
        for (int ks = 0; ks < kHeadDim / 16; ++ks) {
          const uint32_t off = (ks >> 2) * (kKBlockElems * 2) + (ks & 3) * 32;
          umma_bf16(tmem_s[st], umma_smem_desc(q_addr + off), umma_smem_desc(k_addr + off), ks > 0);
        }
        umma_commit(&sm.s_full[st]);
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 0; ok && j < n_kv_tiles; ++j) {
        if (j + 1 < n_kv_tiles && !issue_s(j + 1)) { ok = false; break; }
        if (!mbar_wait_bounded(&sm.p_full, j & 1, kPrefillWaitBudget)) { ok = false; break; }
        tc_fence_after();
        const uint32_t p_addr = smem_addr(sm.p);
        const uint32_t v_addr = smem_addr(sm.vt[j & 1]);
#pragma unroll
        for (int ks = 0; ks < kPT / 16; ++ks) {
          const uint32_t off = (ks >> 2) * (kKBlockElems * 2) + (ks & 3) * 32;
          umma_bf16(tmem_o, umma_smem_desc(p_addr + off), umma_smem_desc(v_addr + off),
                    j > 0 || ks > 0);
        }
        umma_commit(&sm.o_done);
        umma_commit(&sm.kv_empty[j & 1]);
      }
      if (!ok) atomicOr(&sm.err, 1);
    }
    __syncwarp();
  } else {
    // ---- softmax: thread tid owns query row tid of the tile (TMEM lane tid) ----
    const int r = tid;
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    float m = -CUDART_INF_F, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv_tiles && ok; ++j) {
      const int st = j & 1;
      // Waits are voted so the warp stays converged for the warp-collective
      // tensor-memory loads and stores.
      ok = __all_sync(0xffffffffu, mbar_wait_bounded(&sm.s_full[st], (j >> 1) & 1,
                                                     kPrefillWaitBudget));
      if (!ok) break;
      tc_fence_after();
      float s[kPT];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float v[32];
        tmem_ld32(tmem_s[st] + lane_off + c * 32, v);
#pragma unroll
        for (int e = 0; e < 32; ++e) s[c * 32 + e] = v[e];
      }
      tc_fence_before();
      mbar_arrive(&sm.s_empty[st]);
      const bool diag = (j == i);
      float rowmax = -CUDART_INF_F;
#pragma unroll
      for (int c = 0; c < kPT; ++c) {
        float x = s[c] * p.scale_log2;
        if (diag && c > r) x = -CUDART_INF_F;  // causal: keys after the query
        s[c] = x;
        rowmax = fmaxf(rowmax, x);
      }
      const bool move = (j == 0) || rowmax > m + 8.0f;
      const float m_new = move ? fmaxf(m, rowmax) : m;
      const float alpha = (move && j > 0) ? fast_exp2(m - m_new) : 1.f;
      m = m_new;
      float sum = 0.f;
      uint32_t packed[kPT / 2];
#pragma unroll
      for (int c = 0; c < kPT; c += 2) {
        const float p0 = fast_exp2(s[c] - m), p1 = fast_exp2(s[c + 1] - m);
        sum += p0 + p1;
        __nv_bfloat162 b2 = __floats2bfloat162_rn(p0, p1);
        packed[c / 2] = *reinterpret_cast<uint32_t*>(&b2);
      }
      l = l * alpha + sum;
      // P.V of the previous tile must be done: O is then current and P free.
      if (j > 0) {
        ok = __all_sync(0xffffffffu,
                        mbar_wait_bounded(&sm.o_done, (j - 1) & 1, kPrefillWaitBudget));
        if (!ok) break;
        tc_fence_after();
        if (__any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            float v[32];
            tmem_ld32(tmem_o + lane_off + c * 32, v);
#pragma unroll
            for (int e = 0; e < 32; ++e) v[e] *= alpha;
            tmem_st32(tmem_o + lane_off + c * 32, v);
          }
        }
      }
      // P row -> swizzled operand image (8 bf16 = 16 B per store)
#pragma unroll
      for (int ch = 0; ch < kPT / 8; ++ch) {
        const int k0 = ch * 8;
        uint4 val = make_uint4(packed[k0 / 2], packed[k0 / 2 + 1], packed[k0 / 2 + 2],
                               packed[k0 / 2 + 3]);
        *reinterpret_cast<uint4*>(&sm.p[sw_offset(r, k0)]) = val;
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&sm.p_full);
    }
    const bool fin = __all_sync(0xffffffffu, ok && mbar_wait_bounded(&sm.o_done,
                                                                     (n_kv_tiles - 1) & 1,
                                                                     kPrefillWaitBudget));
    if (fin) {
      tc_fence_after();
      const float inv_l = l > 0.f ? 1.f / l : 0.f;
      float* dst = p.out + ((long long)seq * p.S + (long long)i * kPT + r) * p.n_q * kHeadDim +
                   (long long)hq * kHeadDim;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float v[32];
        tmem_ld32(tmem_o + lane_off + c * 32, v);
#pragma unroll
        for (int e = 0; e < 32; e += 4)
          *reinterpret_cast<float4*>(dst + c * 32 + e) =
              make_float4(v[e] * inv_l, v[e + 1] * inv_l, v[e + 2] * inv_l, v[e + 3] * inv_l);
      }
    } else {
      atomicOr(&sm.err, 1);
    }
  }

  // ---- teardown: make sure no MMA is still writing, then free TMEM ----
  tc_fence_before();
  __syncthreads();
  if (sm.err && tid == 0) atomicOr(p.status, kStatusWaitTimeout);
  if (warp == 5) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;"
                 ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

size_t prefill_image_elems(int n_seq, int S, int n_heads) {
  return (size_t)n_seq * n_heads * (size_t)S * kHeadDim;
}

cudaError_t prepare_prefill_kernels() {
  return cudaFuncSetAttribute((const void*)prefill_attn_kernel,
                              cudaFuncAttributeMaxDynamicSharedMemorySize,
                              (int)prefill_smem_bytes());
}

cudaError_t launch_prefill(const float* qkv, long long seq_stride, int n_seq, int S, int n_q,
                           int n_kv, const float* inv_freq, __nv_bfloat16* qimg,
                           __nv_bfloat16* kimg, __nv_bfloat16* vimg, float* const* k_caches,
                           float* const* v_caches, int t_max, float* out, int* status,
                           cudaStream_t st) {
  PrefillPrepParams pp{};
  pp.qkv = qkv;
  pp.seq_stride = seq_stride;
  pp.S = S;
  pp.n_q = n_q;
  pp.n_kv = n_kv;
  pp.inv_freq = inv_freq;
  pp.qimg = qimg;
  pp.kimg = kimg;
  pp.vimg = vimg;
  pp.k_caches = k_caches;
  pp.v_caches = v_caches;
  pp.t_max = t_max;
  prefill_prep_kernel<<<dim3(S, n_seq), 256, 0, st>>>(pp);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  PrefillAttnParams ap{};
  ap.qimg = qimg;
  ap.kimg = kimg;
  ap.vimg = vimg;
  ap.out = out;
  ap.S = S;
  ap.n_q = n_q;
  ap.n_kv = n_kv;
  ap.scale_log2 = (1.0f / sqrtf((float)kHeadDim)) * 1.4426950408889634f;
  ap.status = status;
  prefill_attn_kernel<<<dim3(S / kPT, n_q, n_seq), kPrefillThreads, prefill_smem_bytes(), st>>>(ap);
  return cudaGetLastError();
}

}  // namespace gqa
