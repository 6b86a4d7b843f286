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
// -- 1260 bytes per row as before.  Half-superblock hh = 2 * superblock + n of
// a row owns ql bytes [64hh, 64hh + 64), qh bytes [32hh, 32hh + 32) and scale
// bytes [8hh, 8hh + 8); within its ql bytes the two 32-byte halves (quarters
// 0/2 and 1/3) are swapped when hh & 2, so that the warp's loads below hit 32
// different shared-memory banks, and its scale bytes are reordered so that
// scales[8n + 2c + g] sits at 8hh + 4g + c: a lane's four scales are one
// 32-bit word; the qh bytes are stored XOR 0xAA (the high bit of each 2-bit
// field flipped), so that an assembled code byte is code ^ 32.  Any run of rows
// starting on a multiple of 4 is then four 16-byte-aligned runs of bytes.
//
// The head kernel is a bulk-copy pipeline: one CTA per SM over a contiguous,
// balanced range of rows, a producer warp that copies stages of 32 rows (the
// four planes' runs, 40320 bytes) into a 4-deep ring of shared-memory stages,
// starting before the programmatic dependency wait (the weights do not depend
// on the previous kernel), and 16 consumer warps that each take two rows of a
// stage, computed side by side.  Lane (hh0 = lane / 8, q = lane % 8) owns, in
// every row, the three 16-weight units hh = hh0 + 4u (u = 0, 1, 2),
// l = 4q .. 4q + 3, all four quarters; the digit words of the units' 48 inputs
// (below) stay in registers for the whole kernel.  Per unit the lane reads two
// ql words, one qh word, its four scale bytes and d; four code words (one byte
// per weight) come from AND/OR steps.  The products are integer: once per
// launch the CTA splits each unit's 16 normalised inputs, with a power-of-two
// scale s >= max|z| / 63, into three signed digits in [-63, 63],
// z = s (e1 + e2 / 126 + e3 / 126^2); per row, the code bytes become code - 32
// as signed bytes (y = code ^ 32 from the packed qh, plus 6 (y & 32): two
// instructions per word), dp4a against the digit words gives exact int32
// sums, the quarters' int8 scales combine them exactly (|K| < 2^22), and the
// unit's term is (d s) (K1 + K2 / 126 + K3 / 126^2).  With z = 32 e_i (a power
// of two) the digits are exact and a logit is d * (scale * (code - 32) * 32)
// with one rounding, as in the reference's order (d * scale is exact).
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
constexpr int kStageRows = 2 * kHeadConsumerWarps;  // two rows per consumer warp
constexpr int kHeadStages = 4;
constexpr int kStQl = kStageRows * kQlRow;
constexpr int kStQh = kStageRows * kQhRow;
constexpr int kStSc = kStageRows * kScRow;
constexpr int kStD = kStageRows * kDRow;
constexpr int kStageBytes = kStQl + kStQh + kStSc + kStD;  // 40320
constexpr float kHeadRmsEps = 1e-6f;               // EPSILON of the reference
constexpr float kNoPick = -1e30f;                  // best_val start of the greedy loop
constexpr long long kHeadWaitBudget = 2000000000LL;
constexpr int kEmbedThreads = 256;
constexpr int kQ4Bytes = 18;
static_assert(kStageBytes % 16 == 0 && kStQl % 16 == 0 && kStQh % 16 == 0 && kStSc % 16 == 0,
              "stage runs must stay 16-byte aligned");

struct HeadBest {
  float v;
  int i;
};

constexpr int kHeadUnits = kHeadK / 16;  // 16-weight units of a row (96)

struct HeadSmem {
  alignas(128) uint8_t stage[kHeadStages][kStageBytes];
  alignas(16) float sz[kHeadK];
  // the inputs' digits: word (k, unit, c) packs digit k of the unit's four
  // inputs of quarter c; a lane's four quarters of a (k, unit) are one
  // 16-byte load, consecutive units on consecutive lanes
  alignas(16) uint32_t dig[3][kHeadUnits][4];
  float uscale[kHeadUnits];
  float red[kHeadConsumerWarps];
  HeadBest best[kHeadConsumerWarps];
  uint64_t full[kHeadStages];
  uint64_t empty[kHeadStages];
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
  for (int i = threadIdx.x; i < kQ6RowBytes; i += blockDim.x) {
    const int s = i / kQ6SuperBytes, o = i % kQ6SuperBytes;
    const uint8_t v = r < n_rows ? src[r * kQ6RowBytes + i] : 0;
    if (o < 128) {
      const int hh = 2 * s + (o >> 6), b = o & 63;
      ql[64 * hh + (b ^ ((hh & 2) ? 32 : 0))] = v;
    } else if (o < 192) {
      // the high bit of each 2-bit field flipped: assembled codes are code ^ 32
      qh[64 * s + (o - 128)] = r < n_rows ? (uint8_t)(v ^ 0xAA) : (uint8_t)0;
    } else if (o < 208) {
      // scales[8n + 2c + g] -> byte 8hh + 4g + c
      const int j = o - 192, n = j >> 3, c = (j & 7) >> 1, g = j & 1;
      sc[8 * (2 * s + n) + 4 * g + c] = v;
    } else {
      dd[2 * s + (o - 208)] = v;
    }
  }
}

// ---------------------------------------------------------------------------
// Output RMSNorm + Q6_K LM head + greedy pick
// ---------------------------------------------------------------------------
__device__ __forceinline__ void head_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void consumers_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kHeadConsumers) : "memory");
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
__device__ __forceinline__ void head_pick(float best_v, int best_i, HeadBest* sbest, int* slast,
                                          HeadBest* gbest, unsigned* done, int* token) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int grid = gridDim.x;
  if (lane == 0) sbest[warp] = HeadBest{best_v, best_i};
  consumers_sync();
  if (tid == 0) {
    HeadBest b = sbest[0];
    for (int w = 1; w < kHeadConsumerWarps; ++w)
      if (better(sbest[w].v, sbest[w].i, b.v, b.i)) b = sbest[w];
    gbest[blockIdx.x] = b;
    __threadfence();
    *slast = atomicAdd(done, 1u) == (unsigned)grid - 1;
  }
  consumers_sync();
  if (!*slast) return;
  __threadfence();
  HeadBest b{kNoPick, 0};
  for (int i = tid; i < grid; i += kHeadConsumers) {
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
  consumers_sync();  // the reads of sbest above are done
  if (lane == 0) sbest[warp] = b;
  consumers_sync();
  if (tid == 0) {
    for (int w = 1; w < kHeadConsumerWarps; ++w)
      if (better(sbest[w].v, sbest[w].i, b.v, b.i)) b = sbest[w];
    *token = b.i;
    *done = 0u;  // ready for the next launch
  }
}

// The consumer lane's fixed part of the row arithmetic.
struct LaneConst {
  int hh0, q, o0, o1;   // unit base, 4-weight group, word offsets of W0 / W1
  int g;                // which 16 of the 32 l values: scale word 2hh + g
};

// Exact float of an int32 below 2^22 in magnitude: 2^23 + 2^22 + i as bits,
// minus the same.
__device__ __forceinline__ float small_int_to_float(int i) {
  return __fsub_rn(__int_as_float(0x4B400000 + i), 12582912.0f);
}

// The lane's inputs as digits (see the file comment): for unit u, quarter c
// and digit k, e[u][c][k] packs the digits of weights 4q .. 4q + 3; s[u] is
// the unit's power-of-two scale.
struct LaneDigits {
  int e[3][4][3];
  float s[3];
};

// Unit u's term of row j of a stage for this lane: (d s) (K1 + K2/126 + K3/126^2).
__device__ __forceinline__ float unit_term(const uint8_t* sb, int j, int u, const LaneConst& lc,
                                           const LaneDigits& x) {
  const uint32_t* qlw = reinterpret_cast<const uint32_t*>(sb) + j * (kQlRow / 4);
  const uint32_t* qhw = reinterpret_cast<const uint32_t*>(sb + kStQl) + j * (kQhRow / 4);
  const uint32_t* scw = reinterpret_cast<const uint32_t*>(sb + kStQl + kStQh) + j * (kScRow / 4);
  const unsigned short* dw =
      reinterpret_cast<const unsigned short*>(sb + kStQl + kStQh + kStSc) + j * (kDRow / 2);
  const int hh = lc.hh0 + 4 * u;
  const uint32_t W0 = qlw[16 * hh + lc.o0 + lc.q], W1 = qlw[16 * hh + lc.o1 + lc.q];
  const uint32_t H = qhw[8 * hh + lc.q];
  const uint32_t sv = scw[2 * hh + lc.g];
  const float d = __half2float(__ushort_as_half(dw[hh >> 1]));
  // byte e of Q[c] = (6-bit code of weight (quarter c, l = 4q + e)) ^ 32
  uint32_t Q[4];
  Q[0] = (W0 & 0x0F0F0F0Fu) | ((H << 4) & 0x30303030u);
  Q[1] = (W1 & 0x0F0F0F0Fu) | ((H << 2) & 0x30303030u);
  Q[2] = ((W0 >> 4) & 0x0F0F0F0Fu) | (H & 0x30303030u);
  Q[3] = ((W1 >> 4) & 0x0F0F0F0Fu) | ((H >> 2) & 0x30303030u);
  int K[3] = {0, 0, 0};
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    // code - 32 as a signed byte: y when y < 32, y - 64 (= y | 0xC0) otherwise
    const int v = (int)((Q[c] & 0x20202020u) * 6u + Q[c]);
    // the quarter's int8 scale, sign-extended: PTX prmt replicates the
    // selected byte's sign bit when bit 3 of a selector nibble is set (the
    // __byte_perm intrinsic reads only bits 0-2 of each nibble)
    int sc;
    asm("prmt.b32 %0, %1, 0, %2;"
        : "=r"(sc)
        : "r"(sv), "r"(c | (8 + c) << 4 | (8 + c) << 8 | (8 + c) << 12));
#pragma unroll
    for (int k = 0; k < 3; ++k) K[k] += sc * __dp4a(v, x.e[u][c][k], 0);
  }
  constexpr float kB1 = 1.0f / 126.0f, kB2 = 1.0f / 15876.0f;
  const float f = __fmaf_rn(small_int_to_float(K[2]), kB2,
                            __fmaf_rn(small_int_to_float(K[1]), kB1, small_int_to_float(K[0])));
  return f * __fmul_rn(d, x.s[u]);  // (d s) exact: s is a power of two
}

// Rows ja and jb of a stage with the lane's inputs (lane's partial sums; the
// caller reduces over the warp): two independent chains sharing the digits.
__device__ __forceinline__ void rows_dot(const uint8_t* sb, int ja, int jb, const LaneConst& lc,
                                         const LaneDigits& x, float& acc_a, float& acc_b) {
  acc_a = 0.f;
  acc_b = 0.f;
#pragma unroll
  for (int u = 0; u < 3; ++u) {
    const float ta = unit_term(sb, ja, u, lc, x);
    const float tb = unit_term(sb, jb, u, lc, x);
    acc_a = __fadd_rn(acc_a, ta);
    acc_b = __fadd_rn(acc_b, tb);
  }
}

// The CTA's rows: a contiguous range of the padded rows, cut on multiples of
// 4 so that every stage's runs stay 16-byte multiples; ranges differ by at
// most 4 rows, so no CTA does a whole stage more than another.
__device__ __forceinline__ void head_cta_rows(long long np, long long& r_begin, long long& r_end) {
  const long long units = np / 4;
  r_begin = units * blockIdx.x / gridDim.x * 4;
  r_end = units * (blockIdx.x + 1) / gridDim.x * 4;
}

__global__ void __launch_bounds__(kHeadThreads, 1) lm_head_kernel(const HeadParams p) {
  extern __shared__ __align__(128) unsigned char head_smem_raw[];
  HeadSmem& sm = *reinterpret_cast<HeadSmem*>(head_smem_raw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_rows = p.n_rows;
  const long long np = head_padded_rows(n_rows);
  long long r_begin, r_end;
  head_cta_rows(np, r_begin, r_end);
  const int n_stages = (int)((r_end - r_begin + kStageRows - 1) / kStageRows);
  if (tid == 0) {
    for (int s = 0; s < kHeadStages; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], kHeadConsumerWarps);
    }
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == kHeadConsumerWarps) {
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
        const int s = k % kHeadStages;
        if (k >= kHeadStages &&
            !mbar_wait_bounded(&sm.empty[s], ((k / kHeadStages) - 1) & 1, kHeadWaitBudget)) {
          ok = false;
          break;
        }
        const long long r0 = r_begin + (long long)k * kStageRows;
        const int nr = (int)min((long long)kStageRows, r_end - r0);  // a multiple of 4
        uint8_t* st = sm.stage[s];
        mbar_arrive_expect_tx(&sm.full[s], (uint32_t)(nr * kQ6RowBytes));
        bulk_copy_g2s(st, ql + r0 * kQlRow, nr * kQlRow, &sm.full[s], pol);
        bulk_copy_g2s(st + kStQl, qh + r0 * kQhRow, nr * kQhRow, &sm.full[s], pol);
        bulk_copy_g2s(st + kStQl + kStQh, sc + r0 * kScRow, nr * kScRow, &sm.full[s], pol);
        bulk_copy_g2s(st + kStQl + kStQh + kStSc, dd + r0 * kDRow, nr * kDRow, &sm.full[s], pol);
        if (k == kHeadStages - 1) {
          pdl_wait();
          pdl_launch_dependents();
        }
      }
      if (k < kHeadStages) {
        pdl_wait();
        pdl_launch_dependents();
      }
      if (!ok) atomicOr(p.status, kStatusWaitTimeout);
      // Every copy issued has landed before the CTA may exit: wait for the
      // last use of each stage (a no-op when the consumers already did).
      for (int kk = max(0, k - kHeadStages); kk < k; ++kk)
        mbar_wait_bounded(&sm.full[kk % kHeadStages], (kk / kHeadStages) & 1, kHeadWaitBudget);
    } else {
      pdl_wait();
      pdl_launch_dependents();
    }
    return;
  }

  // ---------------- consumers ----------------
  constexpr int kPer = kHeadK / kHeadConsumers;
  float gm[kPer];
#pragma unroll
  for (int k = 0; k < kPer; ++k) gm[k] = p.gamma[tid + k * kHeadConsumers];
  pdl_wait();
  pdl_launch_dependents();

  // z = rmsnorm(state) * gamma (test_full_model_logits.c:944-948)
  float xv[kPer];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    xv[k] = p.state[tid + k * kHeadConsumers];
    ss += xv[k] * xv[k];
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  if (lane == 0) sm.red[warp] = ss;
  consumers_sync();
  float tot = 0.f;
#pragma unroll
  for (int k = 0; k < kHeadConsumerWarps; ++k) tot += sm.red[k];
  const float scale = 1.0f / sqrtf(tot / (float)kHeadK + kHeadRmsEps);
#pragma unroll
  for (int k = 0; k < kPer; ++k) sm.sz[tid + k * kHeadConsumers] = xv[k] * scale * gm[k];
  consumers_sync();

  // ---- the inputs as digits, one word (unit, quarter) per thread: unit
  // (hh, q) holds inputs 128hh + 32c + 4q + e, c, e < 4 ----
  if (tid < kHeadUnits * 4) {
    const int unit = tid >> 2, c = tid & 3, hh = unit >> 3, q = unit & 7;
    const float4 zz = *reinterpret_cast<const float4*>(sm.sz + 128 * hh + 32 * c + 4 * q);
    float mx = fmaxf(fmaxf(fabsf(zz.x), fabsf(zz.y)), fmaxf(fabsf(zz.z), fabsf(zz.w)));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));  // the unit's four words are
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));  // four consecutive lanes
    // s = the smallest power of two >= mx / 63 (1 when the unit is all zero)
    const uint32_t mb = __float_as_uint(mx / 63.0f);
    const uint32_t sb = (mb & 0x007FFFFFu) ? (mb & 0x7F800000u) + 0x00800000u : mb;
    const float sunit = mx > 0.f ? __uint_as_float(sb) : 1.0f;
    const float inv = __frcp_rn(sunit);  // exact: a power of two
    const float xs[4] = {zz.x * inv, zz.y * inv, zz.z * inv, zz.w * inv};
    uint32_t by[3][4];
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
      by[0][e] = __float_as_uint(t1);
      by[1][e] = __float_as_uint(t2);
      by[2][e] = __float_as_uint(t3);
    }
#pragma unroll
    for (int k = 0; k < 3; ++k)
      sm.dig[k][unit][c] = __byte_perm(__byte_perm(by[k][0], by[k][1], 0x0040),
                                       __byte_perm(by[k][2], by[k][3], 0x0040), 0x5410);
    if (c == 0) sm.uscale[unit] = sunit;
  }
  consumers_sync();

  LaneConst lc;
  lc.hh0 = lane >> 3;
  lc.q = lane & 7;
  lc.o0 = (lc.hh0 & 2) ? 8 : 0;  // the pack swapped the halves of these units
  lc.o1 = 8 - lc.o0;
  lc.g = (lane & 7) >> 2;
  LaneDigits x;
#pragma unroll
  for (int u = 0; u < 3; ++u) {
    const int unit = 8 * (lc.hh0 + 4 * u) + lc.q;  // = lane + 32u: consecutive per lane
    x.s[u] = sm.uscale[unit];
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      const uint4 w = *reinterpret_cast<const uint4*>(&sm.dig[k][unit][0]);
      x.e[u][0][k] = (int)w.x;
      x.e[u][1][k] = (int)w.y;
      x.e[u][2][k] = (int)w.z;
      x.e[u][3][k] = (int)w.w;
    }
  }

  float best_v = kNoPick;
  int best_i = 0;
  bool ok = true;
  const long long r_stop = min(r_end, (long long)n_rows);  // padding rows are never output
  const int ja = warp, jb = warp + kStageRows / 2;
  for (int k = 0; k < n_stages; ++k) {
    const int s = k % kHeadStages;
    if (!mbar_wait_bounded(&sm.full[s], (k / kHeadStages) & 1, kHeadWaitBudget)) {
      ok = false;
      break;
    }
    const long long r0 = r_begin + (long long)k * kStageRows;
    // (jb > ja: a warp whose first row is past the CTA's rows has none; the
    // rows past a short last stage hold stale bytes and are not output)
    if (r0 + ja < r_stop) {
      float acc_a, acc_b;
      rows_dot(sm.stage[s], ja, jb, lc, x, acc_a, acc_b);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        acc_a += __shfl_xor_sync(0xffffffffu, acc_a, off);
        acc_b += __shfl_xor_sync(0xffffffffu, acc_b, off);
      }
      // rows rise within a warp (ja < jb, stages in order): the first maximum stays
      if (p.logits && lane == 0) p.logits[r0 + ja] = acc_a;
      if (acc_a > best_v) {
        best_v = acc_a;
        best_i = (int)(r0 + ja);
      }
      if (r0 + jb < r_stop) {
        if (p.logits && lane == 0) p.logits[r0 + jb] = acc_b;
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

  head_pick(best_v, best_i, sm.best, &sm.last, p.best, p.done, p.token);
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
                                       (int)sizeof(HeadSmem));
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
  cfg.blockDim = dim3(kHeadThreads);
  cfg.dynamicSmemBytes = q8 ? sizeof(Q8Smem) : sizeof(HeadSmem);
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
