// The parts of the reference's token step around the decoder layers
// (qwen_server.c:1016-1046):
//   embed_q4_kernel   the Q4_0 embedding row of the current token becomes the
//                     residual state (get_token_embedding, :188-201, done on
//                     the host there, from the GGUF file);
//   lm_head_kernel    output RMSNorm (k_output_norm, :1025-1033; CPU
//                     test_full_model_logits.c:944-948), the Q6_K LM head
//                     (gemv_q6_k, kernel_q6_k.cl:17-121) and the greedy pick
//                     of the next token (:998-1005, a host loop there).
// With the token id kept in device memory, a whole decode step -- embedding,
// layers, head, pick -- runs without a host round trip and can be one graph.
//
// Q6_K (block_q6_K, test_gemv_q6_k.c:21-26): 256 weights per 210-byte
// superblock, ql[128] (low 4 bits), qh[64] (high 2 bits), int8 scales[16],
// fp16 d.  Weight j of a superblock, with half n = j / 128, r = j % 128,
// quarter c = r / 32 and l = r % 32, has the 6-bit code
//   ((ql[64n + 32(c & 1) + l] >> 4(c >> 1)) & 15) | ((qh[32n + l] >> 2c) & 3) << 4
// and the value d * scales[8n + 2c + l / 16] * (code - 32)
// (dequantize_row_q6_k_ref, test_gemv_q6_k.c:46-74).
//
// A row of 1536 inputs is 6 superblocks, 1260 bytes, so rows and the 210-byte
// superblocks start on 2-byte boundaries only.  gqa_lm_head_pack therefore
// lays the same bytes out once, at load time, as four planes over the rows
// rounded up to a multiple of 4 (Np):
//   ql [Np][768]  qh [Np][384]  scales [Np][96]  d [Np][6] (fp16)
// -- 1260 bytes per row as before, each plane row the six superblocks' bytes
// of that kind in order, the ql and qh rows of row r rotated right by
// 16 (r % 8) bytes so that the eight rows a warp reads at one offset hit eight
// different groups of shared-memory banks.  Any run of rows starting on a
// multiple of 4 is then four 16-byte-aligned runs of bytes.
//
// The head kernel is a bulk-copy pipeline: one CTA per SM over a contiguous,
// balanced range of rows, a producer warp that copies stages of 64 rows (the
// four planes' runs, 80640 bytes) into a 2-deep ring of shared-memory stages,
// starting before the programmatic dependency wait (the weights do not depend
// on the previous kernel), and 12 consumer warps.  The products run on the
// tensor cores in 8-bit integers (mma.sync m16n8k16, unsigned codes times
// signed input digits, int32 accumulators): once per launch the CTA splits
// the normalised inputs, with one power-of-two scale s >= max|z| / 63, into
// three signed digits in [-63, 63], z = s (e1 + e2 / 126 + e3 / 126^2), and
// lays them out as the product's B operand (columns 0-2: the three digits;
// 3-7 zero), with the accumulator input -32 sum e per column and 16-input
// chunk, so that D = sum (code - 32) e exactly.  Warp w takes 16 rows (tile
// w / 3) of a stage over two superblocks (2 (w % 3), 2 (w % 3) + 1): per
// 16-weight scale group one product, its int32 result times the group's int8
// scale added into the superblock's sums K_n (|K| < 2^27), and per
// superblock the term (d s)(K1 + K2 / 126 + K3 / 126^2); the three pairs'
// terms of a row meet in shared memory, in pair order.  With z = 32 e_i (the
// reference test's unit columns) the digits are exact and a logit is
// d * (scale * (code - 32) * 32) with one rounding, as in the reference's
// order (d * scale is exact).
#include <cuda_fp16.h>

#include "gqa_common.cuh"

namespace gqa {

constexpr int kHeadK = 1536;                      // d_model
constexpr int kQ6SuperBytes = 210;
constexpr int kQ6Supers = kHeadK / 256;            // superblocks per row
constexpr int kQ6RowBytes = kQ6Supers * kQ6SuperBytes;  // 1260
constexpr int kQlRow = kQ6Supers * 128;            // plane row bytes
constexpr int kQhRow = kQ6Supers * 64;
constexpr int kScRow = kQ6Supers * 16;
constexpr int kDRow = kQ6Supers * 2;
constexpr int kHeadConsumerWarps = 16;
constexpr int kHeadConsumers = 32 * kHeadConsumerWarps;
constexpr int kHeadThreads = kHeadConsumers + 32;  // + the producer warp
constexpr float kHeadRmsEps = 1e-6f;               // EPSILON of the reference
constexpr float kNoPick = -1e30f;                  // best_val start of the greedy loop
constexpr long long kHeadWaitBudget = 2000000000LL;
constexpr int kEmbedThreads = 256;
constexpr int kQ4Bytes = 18;

struct HeadBest {
  float v;
  int i;
};


// The Q6_K head kernel: 12 consumer warps + a producer warp, stages of 64
// rows (the four planes' runs, 80640 bytes), two deep.
constexpr int kQ6Warps = 12;
constexpr int kQ6Consumers = 32 * kQ6Warps;
constexpr int kQ6Threads = kQ6Consumers + 32;
constexpr int kQ6StageRows = 64;
constexpr int kQ6Stages = 2;
constexpr int kQ6StQl = kQ6StageRows * kQlRow;
constexpr int kQ6StQh = kQ6StageRows * kQhRow;
constexpr int kQ6StSc = kQ6StageRows * kScRow;
constexpr int kQ6StD = kQ6StageRows * kDRow;
constexpr int kQ6StageBytes = kQ6StQl + kQ6StQh + kQ6StSc + kQ6StD;  // 80640
constexpr int kQ6Chunks = kHeadK / 16;  // 16-weight scale groups of a row (96)
static_assert(kQ6StageBytes % 16 == 0 && kQ6StQl % 16 == 0 && kQ6StQh % 16 == 0 &&
                  kQ6StSc % 16 == 0 && (4 * kDRow) % 16 == 0,
              "stage runs must stay 16-byte aligned");
static_assert(kQ6Consumers == 4 * kQ6Chunks && kHeadK % kQ6Consumers == 0,
              "one consumer thread per (chunk, 4 inputs)");
static_assert(kQ6Warps == 3 * (kQ6StageRows / 16), "warp = (16-row tile, superblock pair)");

struct Q6Smem {
  alignas(128) uint8_t stage[kQ6Stages][kQ6StageBytes];
  alignas(16) float sz[kHeadK];
  // B operands: word (chunk, n, t) packs digit n of inputs 16 chunk + 4t ..
  // + 3 (n >= 3: zero columns of the 8-wide product)
  alignas(16) uint32_t dig[kQ6Chunks][8][4];
  // accumulator inputs: -32 times the sum of digit n over the chunk's inputs
  alignas(16) int ncorr[kQ6Chunks][8];
  float part[2][3][kQ6StageRows];  // (stage parity, superblock pair, row) terms
  float red[kQ6Warps];
  float smax[kQ6Warps];
  HeadBest best[kQ6Warps];
  uint64_t full[kQ6Stages];
  uint64_t empty[kQ6Stages];
  int last;
};

struct HeadParams {
  const uint8_t* planes;  // gqa_lm_head_pack layout for n_rows rows
  int n_rows;
  const float* state;     // [1536]
  const float* gamma;     // [1536] output-norm weight
  float* logits;          // [n_rows] or null
  int* token;             // greedy pick, or null
  HeadBest* best;         // [gridDim.x] per-CTA picks
  unsigned* done;         // CTA arrival counter, zero between launches
  int* status;
};

__host__ __device__ constexpr long long head_padded_rows(long long n_rows) {
  return (n_rows + 3) / 4 * 4;
}

size_t lm_head_packed_bytes(long long n_rows) {
  return (size_t)head_padded_rows(n_rows) * kQ6RowBytes;
}

// ---------------------------------------------------------------------------
// GGUF rows -> planes (one CTA per row; a load-time step).  Padding rows are
// written as zeros.
// ---------------------------------------------------------------------------
__global__ void q6k_pack_kernel(const uint8_t* __restrict__ src, int n_rows,
                                uint8_t* __restrict__ dst) {
  const long long r = blockIdx.x;
  const long long np = head_padded_rows(n_rows);
  uint8_t* ql = dst + r * kQlRow;
  uint8_t* qh = dst + np * kQlRow + r * kQhRow;
  uint8_t* sc = dst + np * (kQlRow + kQhRow) + r * kScRow;
  uint8_t* dd = dst + np * (kQlRow + kQhRow + kScRow) + r * kDRow;
  const int rot = 16 * (int)(r & 7);  // ql and qh rows rotated right by 16 (r % 8) bytes
  for (int i = threadIdx.x; i < kQ6RowBytes; i += blockDim.x) {
    const int s = i / kQ6SuperBytes, o = i % kQ6SuperBytes;
    const uint8_t v = r < n_rows ? src[r * kQ6RowBytes + i] : 0;
    if (o < 128)
      ql[(128 * s + o + rot) % kQlRow] = v;
    else if (o < 192)
      qh[(64 * s + (o - 128) + rot) % kQhRow] = v;
    else if (o < 208)
      sc[16 * s + (o - 192)] = v;
    else
      dd[2 * s + (o - 208)] = v;
  }
}

// ---------------------------------------------------------------------------
// Output RMSNorm + Q6_K LM head + greedy pick
// ---------------------------------------------------------------------------
__device__ __forceinline__ void head_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// Barrier 1 over the NW consumer warps of a head kernel (its producer warp
// never takes part).
template <int NW = kHeadConsumerWarps>
__device__ __forceinline__ void consumers_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(32 * NW) : "memory");
}

// Better pick of two: larger value, then smaller row (the host loop's first
// maximum).
__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
  return v > bv || (v == bv && i < bi);
}

// Greedy pick, warp -> CTA -> grid, run by the consumer threads of a head
// kernel: (best_v, best_i) is the warp's pick (lane 0's is used).  The CTA's
// pick goes to gbest[blockIdx.x]; the last CTA to arrive (an atomic counter)
// reduces all of them with the tie rule of `better`, writes *token and
// resets the counter for the next launch.
template <int NW = kHeadConsumerWarps>
__device__ __forceinline__ void head_pick(float best_v, int best_i, HeadBest* sbest, int* slast,
                                          HeadBest* gbest, unsigned* done, int* token) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int grid = gridDim.x;
  if (lane == 0) sbest[warp] = HeadBest{best_v, best_i};
  consumers_sync<NW>();
  if (tid == 0) {
    HeadBest b = sbest[0];
    for (int w = 1; w < NW; ++w)
      if (better(sbest[w].v, sbest[w].i, b.v, b.i)) b = sbest[w];
    gbest[blockIdx.x] = b;
    __threadfence();
    *slast = atomicAdd(done, 1u) == (unsigned)grid - 1;
  }
  consumers_sync<NW>();
  if (!*slast) return;
  __threadfence();
  HeadBest b{kNoPick, 0};
  for (int i = tid; i < grid; i += 32 * NW) {
    const float v = __ldcg(&gbest[i].v);
    const int idx = __ldcg(&gbest[i].i);
    if (better(v, idx, b.v, b.i)) b = HeadBest{v, idx};
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float v = __shfl_xor_sync(0xffffffffu, b.v, off);
    const int idx = __shfl_xor_sync(0xffffffffu, b.i, off);
    if (better(v, idx, b.v, b.i)) b = HeadBest{v, idx};
  }
  consumers_sync<NW>();  // the reads of sbest above are done
  if (lane == 0) sbest[warp] = b;
  consumers_sync<NW>();
  if (tid == 0) {
    for (int w = 1; w < NW; ++w)
      if (better(sbest[w].v, sbest[w].i, b.v, b.i)) b = sbest[w];
    *token = b.i;
    *done = 0u;  // ready for the next launch
  }
}

// Exact float of an int32 below 2^22 in magnitude: 2^23 + 2^22 + i as bits,
// minus the same.
__device__ __forceinline__ float small_int_to_float(int i) {
  return __fsub_rn(__int_as_float(0x4B400000 + i), 12582912.0f);
}

// The CTA's rows: a contiguous range of the padded rows, cut on multiples of
// 4 so that every stage's runs stay 16-byte multiples; ranges differ by at
// most 4 rows, so no CTA does a whole stage more than another.
__device__ __forceinline__ void head_cta_rows(long long np, long long& r_begin, long long& r_end) {
  const long long units = np / 4;
  r_begin = units * blockIdx.x / gridDim.x * 4;
  r_end = units * (blockIdx.x + 1) / gridDim.x * 4;
}

// Barrier 2 + tile over the three consumer warps of a 16-row tile.
__device__ __forceinline__ void tile_sync(int tile) {
  asm volatile("bar.sync %0, 96;" ::"r"(2 + tile) : "memory");
}

// One m16n8k16 tensor-core product on 8-bit integers: D = A B + C with A
// 16 x 16 unsigned (a0: row g, a1: row g + 8; bytes k = 4t .. 4t + 3, g =
// lane / 4, t = lane % 4), B 16 x 8 signed (b0: column g, rows k = 4t ..
// 4t + 3) and C, D 16 x 8 int32 (d0, d1: row g, columns 2t, 2t + 1; d2, d3:
// row g + 8).
__device__ __forceinline__ void mma_u8s8_m16n8k16(int (&d)[4], uint32_t a0, uint32_t a1,
                                                  uint32_t b0, int c0, int c1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, "
      "{%7,%8,%9,%10};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a0), "r"(a1), "r"(b0), "r"(c0), "r"(c1), "r"(c0), "r"(c1));
}

// Byte b of w as a signed int (PTX prmt replicates the selected byte's sign
// bit when bit 3 of a selector nibble is set).
__device__ __forceinline__ int sext_byte(uint32_t w, int b) {
  int r;
  asm("prmt.b32 %0, %1, 0, %2;" : "=r"(r) : "r"(w), "r"(b | (8 + b) << 4 | (8 + b) << 8 | (8 + b) << 12));
  return r;
}

// Rows (row, row + 8) of a stage, superblock sb: the lane's share of the
// exact integer sums K_n = sum_g scale_g sum_i (code - 32) e_n (digit n's
// column of the product; the lane holds columns 2t, 2t + 1 of both rows in
// acc).  The codes come from the un-rotated ql / qh words of the lane's four
// weights of each group; code - 32 is formed by the accumulator input
// C = -32 sum e over the group.
__device__ __forceinline__ void q6_superblock(const uint8_t* st, int row, int rot_a, int rot_b,
                                              int sb, int lane, const Q6Smem& sm,
                                              const uint32_t (&breg)[16], int (&acc)[4]) {
  const int t = lane & 3;
  const uint32_t* qlw = reinterpret_cast<const uint32_t*>(st);
  const uint32_t* qhw = reinterpret_cast<const uint32_t*>(st + kQ6StQl);
  const uint4* scw = reinterpret_cast<const uint4*>(st + kQ6StQl + kQ6StQh);
  const uint32_t* ql_a = qlw + row * (kQlRow / 4);
  const uint32_t* ql_b = qlw + (row + 8) * (kQlRow / 4);
  const uint32_t* qh_a = qhw + row * (kQhRow / 4);
  const uint32_t* qh_b = qhw + (row + 8) * (kQhRow / 4);
  const uint4 sa = scw[row * (kScRow / 16) + sb];
  const uint4 sb4 = scw[(row + 8) * (kScRow / 16) + sb];
  const uint32_t swa[4] = {sa.x, sa.y, sa.z, sa.w};
  const uint32_t swb[4] = {sb4.x, sb4.y, sb4.z, sb4.w};
#pragma unroll
  for (int n = 0; n < 2; ++n) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int wq = sb * 32 + 16 * n + 4 * h + t;   // ql word of quarters 0 / 2 (+8: 1 / 3)
      const int wh = sb * 16 + 8 * n + 4 * h + t;    // qh word of all four quarters
      const uint32_t w0a = ql_a[(wq + rot_a) % (kQlRow / 4)];
      const uint32_t w1a = ql_a[(wq + 8 + rot_a) % (kQlRow / 4)];
      const uint32_t ha = qh_a[(wh + rot_a) % (kQhRow / 4)];
      const uint32_t w0b = ql_b[(wq + rot_b) % (kQlRow / 4)];
      const uint32_t w1b = ql_b[(wq + 8 + rot_b) % (kQlRow / 4)];
      const uint32_t hb = qh_b[(wh + rot_b) % (kQhRow / 4)];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int g = 8 * n + 2 * c + h;  // scale group of the superblock
        const int chunk = sb * 16 + g;
        const uint32_t wa = (c & 1) ? w1a : w0a, wb = (c & 1) ? w1b : w0b;
        const uint32_t qa = ((wa >> (4 * (c >> 1))) & 0x0F0F0F0Fu) | (((ha >> (2 * c)) & 0x03030303u) << 4);
        const uint32_t qb = ((wb >> (4 * (c >> 1))) & 0x0F0F0F0Fu) | (((hb >> (2 * c)) & 0x03030303u) << 4);
        const uint32_t b0 = breg[g];
        const int2 cc = *reinterpret_cast<const int2*>(&sm.ncorr[chunk][2 * t]);
        int d[4];
        mma_u8s8_m16n8k16(d, qa, qb, b0, cc.x, cc.y);
        const int sa_g = sext_byte(swa[g >> 2], g & 3), sb_g = sext_byte(swb[g >> 2], g & 3);
        acc[0] += sa_g * d[0];
        acc[1] += sa_g * d[1];
        acc[2] += sb_g * d[2];
        acc[3] += sb_g * d[3];
      }
    }
  }
}

__global__ void __launch_bounds__(kQ6Threads, 1) lm_head_kernel(const HeadParams p) {
  extern __shared__ __align__(128) unsigned char head_smem_raw[];
  Q6Smem& sm = *reinterpret_cast<Q6Smem*>(head_smem_raw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_rows = p.n_rows;
  const long long np = head_padded_rows(n_rows);
  long long r_begin, r_end;
  head_cta_rows(np, r_begin, r_end);
  const int n_stages = (int)((r_end - r_begin + kQ6StageRows - 1) / kQ6StageRows);
  if (tid == 0) {
    for (int s = 0; s < kQ6Stages; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], kQ6StageRows / 16);  // one arrival per 16-row tile
    }
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == kQ6Warps) {
    // ---------------- producer ----------------
    if (lane == 0) {
      const uint8_t* ql = p.planes;
      const uint8_t* qh = p.planes + np * kQlRow;
      const uint8_t* sc = p.planes + np * (kQlRow + kQhRow);
      const uint8_t* dd = p.planes + np * (kQlRow + kQhRow + kScRow);
      const uint64_t pol = l2_policy_evict_first();
      int k = 0;
      bool ok = true;
      for (; k < n_stages; ++k) {
        const int s = k % kQ6Stages;
        if (k >= kQ6Stages &&
            !mbar_wait_bounded(&sm.empty[s], ((k / kQ6Stages) - 1) & 1, kHeadWaitBudget)) {
          ok = false;
          break;
        }
        const long long r0 = r_begin + (long long)k * kQ6StageRows;
        const int nr = (int)min((long long)kQ6StageRows, r_end - r0);  // a multiple of 4
        uint8_t* st = sm.stage[s];
        mbar_arrive_expect_tx(&sm.full[s], (uint32_t)(nr * kQ6RowBytes));
        bulk_copy_g2s(st, ql + r0 * kQlRow, nr * kQlRow, &sm.full[s], pol);
        bulk_copy_g2s(st + kQ6StQl, qh + r0 * kQhRow, nr * kQhRow, &sm.full[s], pol);
        bulk_copy_g2s(st + kQ6StQl + kQ6StQh, sc + r0 * kScRow, nr * kScRow, &sm.full[s], pol);
        bulk_copy_g2s(st + kQ6StQl + kQ6StQh + kQ6StSc, dd + r0 * kDRow, nr * kDRow, &sm.full[s],
                      pol);
        if (k == kQ6Stages - 1) {
          pdl_wait();
          pdl_launch_dependents();
        }
      }
      if (k < kQ6Stages) {
        pdl_wait();
        pdl_launch_dependents();
      }
      if (!ok) atomicOr(p.status, kStatusWaitTimeout);
      // Every copy issued has landed before the CTA may exit: wait for the
      // last use of each stage (a no-op when the consumers already did).
      for (int kk = max(0, k - kQ6Stages); kk < k; ++kk)
        mbar_wait_bounded(&sm.full[kk % kQ6Stages], (kk / kQ6Stages) & 1, kHeadWaitBudget);
    } else {
      pdl_wait();
      pdl_launch_dependents();
    }
    return;
  }

  // ---------------- consumers ----------------
  constexpr int kPer = kHeadK / kQ6Consumers;  // 4
  float gm[kPer];
#pragma unroll
  for (int k = 0; k < kPer; ++k) gm[k] = p.gamma[tid + k * kQ6Consumers];
  pdl_wait();
  pdl_launch_dependents();

  // z = rmsnorm(state) * gamma (test_full_model_logits.c:944-948)
  float xv[kPer];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    xv[k] = p.state[tid + k * kQ6Consumers];
    ss += xv[k] * xv[k];
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  if (lane == 0) sm.red[warp] = ss;
  consumers_sync<kQ6Warps>();
  float tot = 0.f;
#pragma unroll
  for (int k = 0; k < kQ6Warps; ++k) tot += sm.red[k];
  const float scale = 1.0f / sqrtf(tot / (float)kHeadK + kHeadRmsEps);
  float mz = 0.f;
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    const float z = xv[k] * scale * gm[k];
    sm.sz[tid + k * kQ6Consumers] = z;
    mz = fmaxf(mz, fabsf(z));
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) mz = fmaxf(mz, __shfl_xor_sync(0xffffffffu, mz, off));
  if (lane == 0) sm.smax[warp] = mz;
  consumers_sync<kQ6Warps>();

  // ---- the inputs as digits: one power-of-two scale s >= max|z| / 63 for
  // the whole vector; thread (chunk, t) splits inputs 16 chunk + 4t .. + 3 ----
  float mx = 0.f;
#pragma unroll
  for (int k = 0; k < kQ6Warps; ++k) mx = fmaxf(mx, sm.smax[k]);
  const uint32_t mb = __float_as_uint(mx / 63.0f);
  const uint32_t sbits = (mb & 0x007FFFFFu) ? (mb & 0x7F800000u) + 0x00800000u : mb;
  const float s_in = mx > 0.f ? __uint_as_float(sbits) : 1.0f;
  {
    const float inv = __frcp_rn(s_in);  // exact: a power of two
    const int chunk = tid >> 2, t = tid & 3;
    const float4 zz = *reinterpret_cast<const float4*>(sm.sz + 16 * chunk + 4 * t);
    const float xs[4] = {zz.x * inv, zz.y * inv, zz.z * inv, zz.w * inv};
    uint32_t by[3][4];
    int sum[3] = {0, 0, 0};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      // round to nearest by 1.5 * 2^23 (|x| <= 63): the sum's low byte is the
      // digit, the difference its value
      constexpr float kMagic = 12582912.0f;
      const float t1 = __fadd_rn(xs[e], kMagic);
      const float d1 = __fsub_rn(t1, kMagic);
      const float r1 = __fmul_rn(__fsub_rn(xs[e], d1), 126.0f);
      const float t2 = __fadd_rn(r1, kMagic);
      const float d2 = __fsub_rn(t2, kMagic);
      const float r2 = __fmul_rn(__fsub_rn(r1, d2), 126.0f);
      const float t3 = __fadd_rn(r2, kMagic);
      const float d3 = __fsub_rn(t3, kMagic);
      by[0][e] = __float_as_uint(t1);
      by[1][e] = __float_as_uint(t2);
      by[2][e] = __float_as_uint(t3);
      sum[0] += (int)d1;
      sum[1] += (int)d2;
      sum[2] += (int)d3;
    }
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      sm.dig[chunk][k][t] = __byte_perm(__byte_perm(by[k][0], by[k][1], 0x0040),
                                        __byte_perm(by[k][2], by[k][3], 0x0040), 0x5410);
      sum[k] += __shfl_xor_sync(0xffffffffu, sum[k], 1);
      sum[k] += __shfl_xor_sync(0xffffffffu, sum[k], 2);
    }
#pragma unroll
    for (int k = 3; k < 8; ++k) sm.dig[chunk][k][t] = 0u;
    if (t == 0) {
#pragma unroll
      for (int k = 0; k < 8; ++k) sm.ncorr[chunk][k] = k < 3 ? -32 * sum[k] : 0;
    }
  }
  consumers_sync<kQ6Warps>();

  // Warp w takes rows 16 (w / 3) .. + 15 of a stage over superblocks
  // 2 (w % 3) and 2 (w % 3) + 1; lane (g, t) rows g and g + 8 of those.
  const int tile = warp / 3, pair = warp % 3, t = lane & 3;
  const int row = 16 * tile + (lane >> 2);
  // The warp's two superblocks never change: their B operands stay in registers.
  uint32_t breg[2][16];
#pragma unroll
  for (int q = 0; q < 2; ++q)
#pragma unroll
    for (int g = 0; g < 16; ++g) breg[q][g] = sm.dig[(2 * pair + q) * 16 + g][lane >> 2][t];
  float best_v = kNoPick;
  int best_i = 0;
  bool ok = true;
  const long long r_stop = min(r_end, (long long)n_rows);  // padding rows are never output
  for (int k = 0; k < n_stages; ++k) {
    const int s = k % kQ6Stages;
    if (!mbar_wait_bounded(&sm.full[s], (k / kQ6Stages) & 1, kHeadWaitBudget)) ok = false;
    ok = __all_sync(0xffffffffu, ok);
    const long long r0 = r_begin + (long long)k * kQ6StageRows;
    const int nr = (int)min((long long)kQ6StageRows, r_end - r0);
    float* part = sm.part[k & 1][pair];
    if (ok && 16 * tile < nr) {
      const uint8_t* st = sm.stage[s];
      const int rot_a = 4 * (int)((r0 + row) & 7), rot_b = 4 * (int)((r0 + row + 8) & 7);
      const unsigned short* dw =
          reinterpret_cast<const unsigned short*>(st + kQ6StQl + kQ6StQh + kQ6StSc);
      float term_a = 0.f, term_b = 0.f;
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const int sb = 2 * pair + q;
        int acc[4] = {0, 0, 0, 0};
        q6_superblock(st, row, rot_a, rot_b, sb, lane, sm, breg[q], acc);
        // K1, K2 sit in the lanes t == 0 (columns 0, 1), K3 in t == 1 (column 2).
        const int k3a = __shfl_down_sync(0xffffffffu, acc[0], 1);
        const int k3b = __shfl_down_sync(0xffffffffu, acc[2], 1);
        constexpr float kB1 = 1.0f / 126.0f, kB2 = 1.0f / 15876.0f;
        const float fa = __fmaf_rn((float)k3a, kB2, __fmaf_rn((float)acc[1], kB1, (float)acc[0]));
        const float fb = __fmaf_rn((float)k3b, kB2, __fmaf_rn((float)acc[3], kB1, (float)acc[2]));
        const float da = __half2float(__ushort_as_half(dw[row * (kDRow / 2) + sb]));
        const float db = __half2float(__ushort_as_half(dw[(row + 8) * (kDRow / 2) + sb]));
        const float ta = fa * __fmul_rn(da, s_in), tb = fb * __fmul_rn(db, s_in);  // (d s) exact
        term_a = q == 0 ? ta : __fadd_rn(term_a, ta);
        term_b = q == 0 ? tb : __fadd_rn(term_b, tb);
      }
      if (t == 0) {
        part[row] = term_a;
        part[row + 8] = term_b;
      }
    }
    // The tile's three warps have their terms in place (and have read the
    // stage); the last pair's warp sums its tile's rows and frees the stage
    // for this tile.
    tile_sync(tile);
    if (pair == 2) {
      if (lane == 0) head_arrive(&sm.empty[s]);
      const int j = 16 * tile + lane;
      if (lane < 16 && j < nr && r0 + j < r_stop && ok) {
        const float* pk = sm.part[k & 1][0];
        const float v = __fadd_rn(__fadd_rn(pk[j], pk[kQ6StageRows + j]),
                                  pk[2 * kQ6StageRows + j]);
        if (p.logits) p.logits[r0 + j] = v;
        // rows rise within a lane (stages in order): the first maximum stays
        if (v > best_v) {
          best_v = v;
          best_i = (int)(r0 + j);
        }
      }
    }
  }
  if (!ok && tid == 0) atomicOr(p.status, kStatusWaitTimeout);
  if (!p.token) return;
  // the lanes' picks meet within each warp first (first maximum on ties)
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float v = __shfl_xor_sync(0xffffffffu, best_v, off);
    const int idx = __shfl_xor_sync(0xffffffffu, best_i, off);
    if (better(v, idx, best_v, best_i)) {
      best_v = v;
      best_i = idx;
    }
  }
  head_pick<kQ6Warps>(best_v, best_i, sm.best, &sm.last, p.best, p.done, p.token);
}

// ---------------------------------------------------------------------------
// Output RMSNorm + Q8_0 LM head + greedy pick (Qwen2.5-0.5B)
//
// The 0.5B generator's head is Q8_0 over 896 inputs (gemv_q8_0,
// kernel_q8_0.cl:10-61; generate_stream_05b.c:845-864): 28 blocks of 34
// bytes per row (fp16 d, then 32 int8 codes q), logit = sum_b d_b * sum_j
// q_bj * z_32b+j.  952-byte rows start on 8-byte boundaries only, so
// gqa_lm_head_q8_0_pack lays them out once, at load time, as two planes over
// the rows rounded up to a multiple of 4 (Np):
//   qs [Np][896]  the int8 codes, reordered per row so that block
//                 b = li + 14s (li < 14, s < 2), codes 16mq .. 16mq + 15
//                 (mq < 2), sit at the 16 bytes from 16 * ((2s + mq) * 14 + li)
//   d  [Np][28]   the fp16 scales
// -- 952 bytes per row as before.  The kernel is the Q6_K head's pipeline with
// stages of 64 rows (3 deep) over a contiguous, balanced row range per CTA: a
// consumer warp takes four rows of a stage, two per half-warp, computed side by
// side; lane li of a half owns blocks li and li + 14 (lanes 14 and 15 idle) and
// reads a block's codes as two 16-byte words -- the second half-warp reads its
// blocks in the other order, so the two halves' loads fall on different banks.
// The products are integer: once per launch each lane splits its 64
// normalised inputs, per block of 32 with s = max|z| / 127, into three signed
// 8-bit digits, z = s (e1 + e2 / 254 + e3 / 254^2) to about 1e-7 of max|z|;
// per row, dp4a gives the exact int32 sums I_k = sum_j q_j e_kj, which become
// floats exactly (|I_k| < 2^22: 2^23 + 2^22 magic), and the block's term is
// d * s * (I_1 + I_2 / 254 + I_3 / 254^2): three dp4a per 4 weights instead of
// four byte_perm, two f32x2 adds and two f32x2 FMAs.
// ---------------------------------------------------------------------------
constexpr int kQ8K = 896;
constexpr int kQ8Blocks = kQ8K / 32;                   // 28
constexpr int kQ8BlockBytes = 34;
constexpr int kQ8RowBytes = kQ8Blocks * kQ8BlockBytes;  // 952
constexpr int kQ8Lanes = kQ8Blocks / 2;                 // lanes with blocks, per half-warp
constexpr int kQ8DRow = kQ8Blocks * 2;                  // 56
constexpr int kQ8StageRows = 4 * kHeadConsumerWarps;    // 64: two rows per half-warp
constexpr int kQ8StQs = kQ8StageRows * kQ8K;
constexpr int kQ8StageBytes = kQ8StQs + kQ8StageRows * kQ8DRow;  // 60928
constexpr int kQ8Stages = 3;
static_assert(kQ8StQs % 16 == 0 && kQ8StageBytes % 16 == 0 && (4 * kQ8DRow) % 16 == 0,
              "stage runs must stay 16-byte aligned");

struct Q8Smem {
  alignas(128) uint8_t stage[kQ8Stages][kQ8StageBytes];
  alignas(16) float sz[kQ8K];
  // the inputs' digits: word (k, mq, b, m4) packs digit k of inputs
  // 16mq + 4m4 .. + 3 of block b -- a lane's four words of one (k, mq) are one
  // 16-byte load, the 14 lanes of a half-warp on consecutive ones
  alignas(16) uint32_t dig[3][2][kQ8Blocks][4];
  float bscale[kQ8Blocks], binv[kQ8Blocks];
  float red[kHeadConsumerWarps];
  HeadBest best[kHeadConsumerWarps];
  uint64_t full[kQ8Stages];
  uint64_t empty[kQ8Stages];
  int last;
};

size_t lm_head_q8_packed_bytes(long long n_rows) {
  return (size_t)head_padded_rows(n_rows) * kQ8RowBytes;
}

// GGUF rows -> planes (one CTA per padded row; load time).  Padding rows get
// code 0 and scale 0.
__global__ void q8_pack_kernel(const uint8_t* __restrict__ src, int n_rows,
                               uint8_t* __restrict__ dst) {
  const long long r = blockIdx.x;
  const long long np = head_padded_rows(n_rows);
  uint8_t* qs = dst + r * kQ8K;
  uint8_t* dd = dst + np * kQ8K + r * kQ8DRow;
  for (int i = threadIdx.x; i < kQ8RowBytes; i += blockDim.x) {
    const int b = i / kQ8BlockBytes, o = i % kQ8BlockBytes;
    if (o < 2) {
      dd[2 * b + o] = r < n_rows ? src[r * kQ8RowBytes + i] : 0;
    } else {
      const int j = o - 2, sl = b / kQ8Lanes, li = b % kQ8Lanes;
      const int at = 16 * ((2 * sl + (j >> 4)) * kQ8Lanes + li) + (j & 15);
      qs[at] = r < n_rows ? src[r * kQ8RowBytes + i] : (uint8_t)0;
    }
  }
}

// Rows ja and jb of a stage, lane's part: blocks b_u = li + 14 (u ^ h) for
// u = 0, 1.  e[u][k][m] packs the k-th digits of the inputs of codes
// 4m .. 4m + 3 of block b_u (four int8), s[u] the block's digit scale; both
// rows use them, and their chains are independent.  The second half-warp
// visits the lane's two blocks in the other order, so each block's term is
// rounded on its own and the pair summed with a plain (commutative) add: a
// row's logit does not depend on which half-warp computes it, and equal rows
// give equal logits for the tie rule.
__device__ __forceinline__ void q8_rows_dot(const uint8_t* sb, int ja, int jb,
                                            const int (&qoff)[2], const int (&boff)[2],
                                            const int (&e)[2][3][8], const float (&s)[2],
                                            float& out_a, float& out_b) {
  const uint8_t* qa = sb + ja * kQ8K;
  const uint8_t* qb = sb + jb * kQ8K;
  const unsigned short* dsc = reinterpret_cast<const unsigned short*>(sb + kQ8StQs);
  float va[2], vb[2];
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    int a1 = 0, a2 = 0, a3 = 0, b1 = 0, b2 = 0, b3 = 0;
#pragma unroll
    for (int mq = 0; mq < 2; ++mq) {
      const uint4 wa = *reinterpret_cast<const uint4*>(qa + qoff[u] + 16 * kQ8Lanes * mq);
      const uint4 wb = *reinterpret_cast<const uint4*>(qb + qoff[u] + 16 * kQ8Lanes * mq);
      const int wsa[4] = {(int)wa.x, (int)wa.y, (int)wa.z, (int)wa.w};
      const int wsb[4] = {(int)wb.x, (int)wb.y, (int)wb.z, (int)wb.w};
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const int k = 4 * mq + m;
        a1 = __dp4a(wsa[m], e[u][0][k], a1);
        a2 = __dp4a(wsa[m], e[u][1][k], a2);
        a3 = __dp4a(wsa[m], e[u][2][k], a3);
        b1 = __dp4a(wsb[m], e[u][0][k], b1);
        b2 = __dp4a(wsb[m], e[u][1][k], b2);
        b3 = __dp4a(wsb[m], e[u][2][k], b3);
      }
    }
    constexpr float kD1 = 1.0f / 254.0f, kD2 = 1.0f / 64516.0f;
    const float fa = __fmaf_rn(small_int_to_float(a3), kD2,
                               __fmaf_rn(small_int_to_float(a2), kD1, small_int_to_float(a1)));
    const float fb = __fmaf_rn(small_int_to_float(b3), kD2,
                               __fmaf_rn(small_int_to_float(b2), kD1, small_int_to_float(b1)));
    const float da = __half2float(__ushort_as_half(dsc[ja * kQ8Blocks + boff[u]]));
    const float db = __half2float(__ushort_as_half(dsc[jb * kQ8Blocks + boff[u]]));
    va[u] = __fmul_rn(__fmul_rn(da, s[u]), fa);
    vb[u] = __fmul_rn(__fmul_rn(db, s[u]), fb);
  }
  out_a = __fadd_rn(va[0], va[1]);
  out_b = __fadd_rn(vb[0], vb[1]);
}

__global__ void __launch_bounds__(kHeadThreads, 1) lm_head_q8_kernel(const HeadParams p) {
  extern __shared__ __align__(128) unsigned char head_smem_raw[];
  Q8Smem& sm = *reinterpret_cast<Q8Smem*>(head_smem_raw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_rows = p.n_rows;
  const long long np = head_padded_rows(n_rows);
  long long r_begin, r_end;
  head_cta_rows(np, r_begin, r_end);
  const int n_stages = (int)((r_end - r_begin + kQ8StageRows - 1) / kQ8StageRows);
  if (tid == 0) {
    for (int s = 0; s < kQ8Stages; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], kHeadConsumerWarps);
    }
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == kHeadConsumerWarps) {
    // ---------------- producer ----------------
    if (lane == 0) {
      const uint8_t* qs = p.planes;
      const uint8_t* dd = p.planes + np * kQ8K;
      const uint64_t pol = l2_policy_evict_first();
      int k = 0;
      bool ok = true;
      for (; k < n_stages; ++k) {
        const int s = k % kQ8Stages;
        if (k >= kQ8Stages &&
            !mbar_wait_bounded(&sm.empty[s], ((k / kQ8Stages) - 1) & 1, kHeadWaitBudget)) {
          ok = false;
          break;
        }
        const long long r0 = r_begin + (long long)k * kQ8StageRows;
        const int nr = (int)min((long long)kQ8StageRows, r_end - r0);  // a multiple of 4
        uint8_t* st = sm.stage[s];
        mbar_arrive_expect_tx(&sm.full[s], (uint32_t)(nr * kQ8RowBytes));
        bulk_copy_g2s(st, qs + r0 * kQ8K, nr * kQ8K, &sm.full[s], pol);
        bulk_copy_g2s(st + kQ8StQs, dd + r0 * kQ8DRow, nr * kQ8DRow, &sm.full[s], pol);
        if (k == kQ8Stages - 1) {
          pdl_wait();
          pdl_launch_dependents();
        }
      }
      if (k < kQ8Stages) {
        pdl_wait();
        pdl_launch_dependents();
      }
      if (!ok) atomicOr(p.status, kStatusWaitTimeout);
      // Every copy issued has landed before the CTA may exit.
      for (int kk = max(0, k - kQ8Stages); kk < k; ++kk)
        mbar_wait_bounded(&sm.full[kk % kQ8Stages], (kk / kQ8Stages) & 1, kHeadWaitBudget);
    } else {
      pdl_wait();
      pdl_launch_dependents();
    }
    return;
  }

  // ---------------- consumers ----------------
  constexpr int kPer = (kQ8K + kHeadConsumers - 1) / kHeadConsumers;
  auto in_range = [&](int k) { return tid + k * kHeadConsumers < kQ8K; };
  float gm[kPer];
#pragma unroll
  for (int k = 0; k < kPer; ++k) gm[k] = in_range(k) ? p.gamma[tid + k * kHeadConsumers] : 0.f;
  pdl_wait();
  pdl_launch_dependents();

  // z = rmsnorm(state) * gamma (the k_output_norm step, generate_stream_05b.c:845-851)
  float xv[kPer];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    xv[k] = in_range(k) ? p.state[tid + k * kHeadConsumers] : 0.f;
    ss += xv[k] * xv[k];
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  if (lane == 0) sm.red[warp] = ss;
  consumers_sync();
  float tot = 0.f;
#pragma unroll
  for (int k = 0; k < kHeadConsumerWarps; ++k) tot += sm.red[k];
  const float scale = 1.0f / sqrtf(tot / (float)kQ8K + kHeadRmsEps);
#pragma unroll
  for (int k = 0; k < kPer; ++k)
    if (in_range(k)) sm.sz[tid + k * kHeadConsumers] = xv[k] * scale * gm[k];
  consumers_sync();

  // ---- the inputs as three 8-bit digits per block of 32:
  // z = s (e1 + e2 / 254 + e3 / 254^2), s = max|z| / 127 ----
  for (int b = warp; b < kQ8Blocks; b += kHeadConsumerWarps) {
    float mx = fabsf(sm.sz[32 * b + lane]);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    if (lane == 0) {
      sm.bscale[b] = mx / 127.0f;
      sm.binv[b] = mx > 0.f ? 127.0f / mx : 0.f;
    }
  }
  consumers_sync();
  if (tid < kQ8K / 4) {  // one word of four inputs per thread
    const int b = tid >> 3, m = tid & 7;
    const float4 zz = *reinterpret_cast<const float4*>(sm.sz + 4 * tid);
    const float inv = sm.binv[b];
    const float xs[4] = {zz.x * inv, zz.y * inv, zz.z * inv, zz.w * inv};
    uint32_t by[3][4];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      // round to nearest by 1.5 * 2^23 (|x| <= 127): the sum's low byte is the
      // digit, the difference its value
      constexpr float kMagic = 12582912.0f;
      const float t1 = __fadd_rn(xs[c], kMagic);
      const float r1 = __fmul_rn(__fsub_rn(xs[c], __fsub_rn(t1, kMagic)), 254.0f);
      const float t2 = __fadd_rn(r1, kMagic);
      const float r2 = __fmul_rn(__fsub_rn(r1, __fsub_rn(t2, kMagic)), 254.0f);
      const float t3 = __fadd_rn(r2, kMagic);
      by[0][c] = __float_as_uint(t1);
      by[1][c] = __float_as_uint(t2);
      by[2][c] = __float_as_uint(t3);
    }
#pragma unroll
    for (int k = 0; k < 3; ++k)
      sm.dig[k][m >> 2][b][m & 3] = __byte_perm(__byte_perm(by[k][0], by[k][1], 0x0040),
                                                __byte_perm(by[k][2], by[k][3], 0x0040), 0x5410);
  }
  consumers_sync();

  const int h = lane >> 4, li = lane & 15;
  const bool active = li < kQ8Lanes;
  int qoff[2], boff[2];
  int e[2][3][8];  // the lane's inputs as three 8-bit digits, four per word
  float sc[2];     // their scale per block
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    const int sl = u ^ h;
    const int b = active ? li + kQ8Lanes * sl : 0;
    qoff[u] = 16 * (2 * sl * kQ8Lanes + (active ? li : 0));
    boff[u] = b;
    sc[u] = sm.bscale[b];
#pragma unroll
    for (int k = 0; k < 3; ++k)
#pragma unroll
      for (int mq = 0; mq < 2; ++mq) {
        const uint4 w = *reinterpret_cast<const uint4*>(&sm.dig[k][mq][b][0]);
        e[u][k][4 * mq + 0] = (int)w.x;
        e[u][k][4 * mq + 1] = (int)w.y;
        e[u][k][4 * mq + 2] = (int)w.z;
        e[u][k][4 * mq + 3] = (int)w.w;
      }
  }

  float best_v = kNoPick;
  int best_i = 0;
  bool ok = true;
  const long long r_stop = min(r_end, (long long)n_rows);  // padding rows are never output
  const int ja = 2 * warp + h, jb = ja + kQ8StageRows / 2;
  for (int k = 0; k < n_stages; ++k) {
    const int s = k % kQ8Stages;
    if (!mbar_wait_bounded(&sm.full[s], (k / kQ8Stages) & 1, kHeadWaitBudget)) {
      ok = false;
      break;
    }
    const long long r0 = r_begin + (long long)k * kQ8StageRows;
    float acc_a = 0.f, acc_b = 0.f;
    // (jb > ja: a half-warp whose first row is past the CTA's rows has none;
    // the rows past a short last stage hold stale bytes and are not output)
    if (active && r0 + ja < r_stop) q8_rows_dot(sm.stage[s], ja, jb, qoff, boff, e, sc, acc_a, acc_b);
#pragma unroll
    for (int off = 8; off > 0; off >>= 1) {
      acc_a += __shfl_xor_sync(0xffffffffu, acc_a, off);
      acc_b += __shfl_xor_sync(0xffffffffu, acc_b, off);
    }
    if (li == 0) {
      // rows rise within a half-warp (ja < jb, stages in order): the first
      // maximum stays
      if (r0 + ja < r_stop) {
        if (p.logits) p.logits[r0 + ja] = acc_a;
        if (acc_a > best_v) {
          best_v = acc_a;
          best_i = (int)(r0 + ja);
        }
      }
      if (r0 + jb < r_stop) {
        if (p.logits) p.logits[r0 + jb] = acc_b;
        if (acc_b > best_v) {
          best_v = acc_b;
          best_i = (int)(r0 + jb);
        }
      }
    }
    __syncwarp();
    if (lane == 0) head_arrive(&sm.empty[s]);
  }
  if (!ok && lane == 0) atomicOr(p.status, kStatusWaitTimeout);
  if (!p.token) return;
  {  // the two half-warps' picks meet in lane 0
    const float v = __shfl_down_sync(0xffffffffu, best_v, 16);
    const int idx = __shfl_down_sync(0xffffffffu, best_i, 16);
    if (better(v, idx, best_v, best_i)) {
      best_v = v;
      best_i = idx;
    }
  }
  head_pick(best_v, best_i, sm.best, &sm.last, p.best, p.done, p.token);
}

// ---------------------------------------------------------------------------
// Token embedding: state = Q4_0 row *token of the table
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kEmbedThreads) embed_q4_kernel(const uint8_t* table, int n_rows,
                                                                 int d_model, const int* token,
                                                                 float* state, int* status) {
  pdl_wait();
  pdl_launch_dependents();
  const int t = *token;
  if (t < 0 || t >= n_rows) {
    if (threadIdx.x == 0) atomicOr(status, kStatusBadToken);
    return;
  }
  const uint8_t* row = table + (size_t)t * (d_model / 32) * kQ4Bytes;
  for (int j = threadIdx.x; j < d_model; j += kEmbedThreads) {
    const uint8_t* blk = row + (j >> 5) * kQ4Bytes;
    const int w = j & 31;
    const float d = __half2float(__ushort_as_half((unsigned short)(blk[0] | (blk[1] << 8))));
    const uint32_t qs = blk[2 + (w & 15)];
    const uint32_t code = w < 16 ? (qs & 15u) : (qs >> 4);
    // (float)((int)code - 8) * d, as get_token_embedding
    state[j] = (__uint_as_float(0x4B000000u | code) - 8388616.0f) * d;
  }
}

// ---------------------------------------------------------------------------
// Launchers
// ---------------------------------------------------------------------------
int lm_head_grid(int n_sm) { return n_sm; }

cudaError_t prepare_head_kernels() {
  cudaError_t e = cudaFuncSetAttribute((const void*)lm_head_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)sizeof(Q6Smem));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute((const void*)lm_head_q8_kernel,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(Q8Smem));
  return e;
}

cudaError_t launch_q8_pack(const void* src, int n_rows, void* dst, cudaStream_t st) {
  q8_pack_kernel<<<(unsigned)head_padded_rows(n_rows), 256, 0, st>>>(
      static_cast<const uint8_t*>(src), n_rows, static_cast<uint8_t*>(dst));
  return cudaGetLastError();
}

cudaError_t launch_q6k_pack(const void* src, int n_rows, void* dst, cudaStream_t st) {
  q6k_pack_kernel<<<(unsigned)head_padded_rows(n_rows), 256, 0, st>>>(
      static_cast<const uint8_t*>(src), n_rows, static_cast<uint8_t*>(dst));
  return cudaGetLastError();
}

// q8: the Q8_0 head (lm_head_q8_kernel) instead of the Q6_K one.
cudaError_t launch_lm_head(bool q8, const void* planes, int n_rows, const float* gamma,
                           const float* state, float* logits, int* token, void* best,
                           unsigned* done, int* status, int grid, cudaStream_t st, bool pdl) {
  HeadParams p{};
  p.planes = static_cast<const uint8_t*>(planes);
  p.n_rows = n_rows;
  p.state = state;
  p.gamma = gamma;
  p.logits = logits;
  p.token = token;
  p.best = static_cast<HeadBest*>(best);
  p.done = done;
  p.status = status;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(q8 ? kHeadThreads : kQ6Threads);
  cfg.dynamicSmemBytes = q8 ? sizeof(Q8Smem) : sizeof(Q6Smem);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  void* args[] = {&p};
  return cudaLaunchKernelExC(&cfg, q8 ? (const void*)lm_head_q8_kernel : (const void*)lm_head_kernel,
                             args);
}

size_t lm_head_best_bytes(int grid) { return sizeof(HeadBest) * (size_t)grid; }

cudaError_t launch_embed_q4(const void* table, int n_rows, int d_model, const int* token,
                            float* state, int* status, cudaStream_t st, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(kEmbedThreads);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  const uint8_t* tb = static_cast<const uint8_t*>(table);
  void* args[] = {&tb, &n_rows, &d_model, &token, &state, &status};
  return cudaLaunchKernelExC(&cfg, (const void*)embed_q4_kernel, args);
}

}  // namespace gqa
