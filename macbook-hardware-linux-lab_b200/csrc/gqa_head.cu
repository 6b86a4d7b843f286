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
// lays the same bytes out once, at load time, as four planes:
//   ql [rows][768]  qh [rows][384]  scales [rows][96]  d [rows][6] (fp16)
// -- 1260 bytes per row as before, every plane row 4-byte (scales 8-byte)
// aligned.  Half-superblock hh = 2 * superblock + n of a row is then ql bytes
// [64hh, 64hh + 64), qh bytes [32hh, 32hh + 32) and scale bytes [8hh, 8hh + 8).
//
// One warp per row, rows interleaved over all warps of the grid.  Lane
// (hh0 = lane / 8, q = lane % 8) owns, in every row, the three 16-weight units
// hh = hh0 + 4u (u = 0, 1, 2), l = 4q .. 4q + 3, all four quarters: the units'
// 48 inputs stay in registers for the whole kernel.  Per unit the lane loads
// two ql words, one qh word, the half's 8 scale bytes and d; four code words
// (one byte per weight) come from three AND/OR steps each; each code becomes
// an exact float by byte_perm into 2^23 + code and a subtraction of 2^23 + 32
// (the q4 kernels' trick), and the products run as f32x2 pairs.
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
constexpr int kHeadThreads = 256;
constexpr int kHeadWarps = kHeadThreads / 32;
constexpr float kHeadRmsEps = 1e-6f;               // EPSILON of the reference
constexpr float kNoPick = -1e30f;                  // best_val start of the greedy loop
constexpr int kEmbedThreads = 256;
constexpr int kQ4Bytes = 18;

struct HeadBest {
  float v;
  int i;
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
};

size_t lm_head_packed_bytes(long long n_rows) { return (size_t)n_rows * kQ6RowBytes; }

// ---------------------------------------------------------------------------
// GGUF rows -> planes (one CTA per row; a load-time step)
// ---------------------------------------------------------------------------
__global__ void q6k_pack_kernel(const uint8_t* __restrict__ src, int n_rows,
                                uint8_t* __restrict__ dst) {
  const long long r = blockIdx.x;
  const uint8_t* row = src + r * kQ6RowBytes;
  uint8_t* ql = dst + r * kQlRow;
  uint8_t* qh = dst + (size_t)n_rows * kQlRow + r * kQhRow;
  uint8_t* sc = dst + (size_t)n_rows * (kQlRow + kQhRow) + r * kScRow;
  uint8_t* dd = dst + (size_t)n_rows * (kQlRow + kQhRow + kScRow) + r * kDRow;
  for (int i = threadIdx.x; i < kQ6RowBytes; i += blockDim.x) {
    const int s = i / kQ6SuperBytes, o = i % kQ6SuperBytes;
    const uint8_t v = row[i];
    if (o < 128) ql[128 * s + o] = v;
    else if (o < 192) qh[64 * s + (o - 128)] = v;
    else if (o < 208) sc[16 * s + (o - 192)] = v;
    else dd[2 * s + (o - 208)] = v;
  }
}

// ---------------------------------------------------------------------------
// Output RMSNorm + Q6_K LM head + greedy pick
// ---------------------------------------------------------------------------
// Exact float of (code - 32) for a code byte of w picked by `sel`
// (byte_perm selector 0x5440 + byte): 2^23 + code, minus 2^23 + 32.
constexpr float kQ6Magic = 8388640.0f;

__device__ __forceinline__ float code_f(uint32_t w, uint32_t sel) {
  return __uint_as_float(__byte_perm(w, 0x4B00u, sel));
}

__device__ __forceinline__ void pair_add(float& d0, float& d1, float a0, float a1, float b0,
                                         float b1) {
  asm("{\n\t.reg .b64 a, b, d;\n\t"
      "mov.b64 a, {%2, %3};\n\tmov.b64 b, {%4, %5};\n\t"
      "add.rn.f32x2 d, a, b;\n\t"
      "mov.b64 {%0, %1}, d;\n\t}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}

__device__ __forceinline__ void pair_fma(float& d0, float& d1, float a0, float a1, float b0,
                                         float b1, float c0, float c1) {
  asm("{\n\t.reg .b64 a, b, c, d;\n\t"
      "mov.b64 a, {%2, %3};\n\tmov.b64 b, {%4, %5};\n\tmov.b64 c, {%6, %7};\n\t"
      "fma.rn.f32x2 d, a, b, c;\n\t"
      "mov.b64 {%0, %1}, d;\n\t}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1), "f"(c0), "f"(c1));
}

// Better pick of two: larger value, then smaller row (the host loop's first
// maximum).
__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
  return v > bv || (v == bv && i < bi);
}

template <int kBatch>
__global__ void __launch_bounds__(kHeadThreads) lm_head_kernel(const HeadParams p) {
  __shared__ __align__(16) float sz[kHeadK];
  __shared__ float red[kHeadWarps];
  __shared__ HeadBest s_best[kHeadWarps];
  __shared__ int s_last;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int q = lane & 7, hh0 = lane >> 3;
  const int gsh = (q >> 2) * 8;  // this lane's scale byte within each scale pair
  const int n_rows = p.n_rows;
  const uint32_t* ql = reinterpret_cast<const uint32_t*>(p.planes);
  const uint32_t* qh = reinterpret_cast<const uint32_t*>(p.planes + (size_t)n_rows * kQlRow);
  const uint2* sc =
      reinterpret_cast<const uint2*>(p.planes + (size_t)n_rows * (kQlRow + kQhRow));
  const unsigned short* dd = reinterpret_cast<const unsigned short*>(
      p.planes + (size_t)n_rows * (kQlRow + kQhRow + kScRow));

  constexpr int kPer = kHeadK / kHeadThreads;
  float gm[kPer];
#pragma unroll
  for (int k = 0; k < kPer; ++k) gm[k] = p.gamma[tid + k * kHeadThreads];
  pdl_wait();
  pdl_launch_dependents();

  // ---- z = rmsnorm(state) * gamma (test_full_model_logits.c:944-948) ----
  float xv[kPer];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    xv[k] = p.state[tid + k * kHeadThreads];
    ss += xv[k] * xv[k];
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int k = 0; k < kHeadWarps; ++k) tot += red[k];
  const float scale = 1.0f / sqrtf(tot / (float)kHeadK + kHeadRmsEps);
#pragma unroll
  for (int k = 0; k < kPer; ++k) sz[tid + k * kHeadThreads] = xv[k] * scale * gm[k];
  __syncthreads();

  // ---- this lane's 48 inputs: unit u, quarter c, weights 4q .. 4q + 3 ----
  float x[3][4][4];
#pragma unroll
  for (int u = 0; u < 3; ++u)
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const float4 v = *reinterpret_cast<const float4*>(sz + 128 * (hh0 + 4 * u) + 32 * c + 4 * q);
      x[u][c][0] = v.x;
      x[u][c][1] = v.y;
      x[u][c][2] = v.z;
      x[u][c][3] = v.w;
    }

  const int wg = blockIdx.x * kHeadWarps + warp, nw = gridDim.x * kHeadWarps;
  float best_v = kNoPick;
  int best_i = 0;
  for (int r0 = wg; r0 < n_rows; r0 += nw * kBatch) {
    uint32_t w0[kBatch][3], w1[kBatch][3], hq[kBatch][3];
    uint2 s8[kBatch][3];
    unsigned short dv[kBatch][3];
#pragma unroll
    for (int b = 0; b < kBatch; ++b) {
      const int r = r0 + b * nw;
      const bool ok = r < n_rows;
      const size_t rq = ok ? (size_t)r : 0;
#pragma unroll
      for (int u = 0; u < 3; ++u) {
        const int hh = hh0 + 4 * u;
        w0[b][u] = __ldg(ql + rq * (kQlRow / 4) + 16 * hh + q);
        w1[b][u] = __ldg(ql + rq * (kQlRow / 4) + 16 * hh + 8 + q);
        hq[b][u] = __ldg(qh + rq * (kQhRow / 4) + 8 * hh + q);
        s8[b][u] = __ldg(sc + rq * (kScRow / 8) + hh);
        dv[b][u] = __ldg(dd + rq * (kDRow / 2) + (hh >> 1));
      }
    }
#pragma unroll
    for (int b = 0; b < kBatch; ++b) {
      float acc = 0.f;
#pragma unroll
      for (int u = 0; u < 3; ++u) {
        const uint32_t W0 = w0[b][u], W1 = w1[b][u], H = hq[b][u];
        // byte e of Q[c] = 6-bit code of weight (quarter c, l = 4q + e)
        uint32_t Q[4];
        Q[0] = (W0 & 0x0F0F0F0Fu) | ((H << 4) & 0x30303030u);
        Q[1] = (W1 & 0x0F0F0F0Fu) | ((H << 2) & 0x30303030u);
        Q[2] = ((W0 >> 4) & 0x0F0F0F0Fu) | (H & 0x30303030u);
        Q[3] = ((W1 >> 4) & 0x0F0F0F0Fu) | ((H >> 2) & 0x30303030u);
        // scales[8n + 2c + g] of this lane's g: byte 0 / 2 of each 32-bit half
        const uint32_t slo = s8[b][u].x >> gsh, shi = s8[b][u].y >> gsh;
        const float scf[4] = {(float)(signed char)(slo & 0xFFu),
                              (float)(signed char)((slo >> 16) & 0xFFu),
                              (float)(signed char)(shi & 0xFFu),
                              (float)(signed char)((shi >> 16) & 0xFFu)};
        float t0 = 0.f, t1 = 0.f;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          float v0, v1, v2, v3;
          pair_add(v0, v1, code_f(Q[c], 0x5440u), code_f(Q[c], 0x5441u), -kQ6Magic, -kQ6Magic);
          pair_add(v2, v3, code_f(Q[c], 0x5442u), code_f(Q[c], 0x5443u), -kQ6Magic, -kQ6Magic);
          float a0, a1;
          pair_fma(a0, a1, v0, v1, x[u][c][0], x[u][c][1], 0.f, 0.f);
          pair_fma(a0, a1, v2, v3, x[u][c][2], x[u][c][3], a0, a1);
          pair_fma(t0, t1, a0, a1, scf[c], scf[c], t0, t1);
        }
        const float d = __half2float(__ushort_as_half(dv[b][u]));
        acc = fmaf(d, t0 + t1, acc);
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
      const int r = r0 + b * nw;
      if (r < n_rows) {
        if (p.logits && lane == 0) p.logits[r] = acc;
        if (acc > best_v) {  // rows rise within a warp: the first maximum stays
          best_v = acc;
          best_i = r;
        }
      }
    }
  }
  if (!p.token) return;

  // ---- greedy pick: warp -> CTA -> grid (the last CTA to arrive) ----
  if (lane == 0) s_best[warp] = HeadBest{best_v, best_i};
  __syncthreads();
  if (tid == 0) {
    HeadBest b = s_best[0];
    for (int w = 1; w < kHeadWarps; ++w)
      if (better(s_best[w].v, s_best[w].i, b.v, b.i)) b = s_best[w];
    p.best[blockIdx.x] = b;
    __threadfence();
    s_last = atomicAdd(p.done, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  HeadBest b{kNoPick, 0};
  for (int i = tid; i < (int)gridDim.x; i += kHeadThreads) {
    const float v = __ldcg(&p.best[i].v);
    const int idx = __ldcg(&p.best[i].i);
    if (better(v, idx, b.v, b.i)) b = HeadBest{v, idx};
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float v = __shfl_xor_sync(0xffffffffu, b.v, off);
    const int idx = __shfl_xor_sync(0xffffffffu, b.i, off);
    if (better(v, idx, b.v, b.i)) b = HeadBest{v, idx};
  }
  __syncthreads();  // s_best reads above are done
  if (lane == 0) s_best[warp] = b;
  __syncthreads();
  if (tid == 0) {
    for (int w = 1; w < kHeadWarps; ++w)
      if (better(s_best[w].v, s_best[w].i, b.v, b.i)) b = s_best[w];
    *p.token = b.i;
    *p.done = 0u;  // ready for the next launch
  }
}

// ---------------------------------------------------------------------------
// Token embedding: state = Q4_0 row *token of the table
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kEmbedThreads) embed_q4_kernel(const uint8_t* table, int n_rows,
                                                                 const int* token, float* state,
                                                                 int* status) {
  pdl_wait();
  pdl_launch_dependents();
  const int t = *token;
  if (t < 0 || t >= n_rows) {
    if (threadIdx.x == 0) atomicOr(status, kStatusBadToken);
    return;
  }
  const uint8_t* row = table + (size_t)t * (kHeadK / 32) * kQ4Bytes;
  for (int j = threadIdx.x; j < kHeadK; j += kEmbedThreads) {
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
constexpr int kHeadBatch = 2;

int lm_head_grid(int n_sm) {
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, lm_head_kernel<kHeadBatch>,
                                                    kHeadThreads, 0) != cudaSuccess ||
      per_sm < 1)
    per_sm = 1;
  return n_sm * per_sm;
}

cudaError_t launch_q6k_pack(const void* src, int n_rows, void* dst, cudaStream_t st) {
  q6k_pack_kernel<<<n_rows, 256, 0, st>>>(static_cast<const uint8_t*>(src), n_rows,
                                          static_cast<uint8_t*>(dst));
  return cudaGetLastError();
}

cudaError_t launch_lm_head(const void* planes, int n_rows, const float* gamma, const float* state,
                           float* logits, int* token, void* best, unsigned* done, int grid,
                           cudaStream_t st, bool pdl) {
  HeadParams p{};
  p.planes = static_cast<const uint8_t*>(planes);
  p.n_rows = n_rows;
  p.state = state;
  p.gamma = gamma;
  p.logits = logits;
  p.token = token;
  p.best = static_cast<HeadBest*>(best);
  p.done = done;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kHeadThreads);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  void* args[] = {&p};
  return cudaLaunchKernelExC(&cfg, (const void*)lm_head_kernel<kHeadBatch>, args);
}

size_t lm_head_best_bytes(int grid) { return sizeof(HeadBest) * (size_t)grid; }

cudaError_t launch_embed_q4(const void* table, int n_rows, const int* token, float* state,
                            int* status, cudaStream_t st, bool pdl) {
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
  void* args[] = {&tb, &n_rows, &token, &state, &status};
  return cudaLaunchKernelExC(&cfg, (const void*)embed_q4_kernel, args);
}

}  // namespace gqa
