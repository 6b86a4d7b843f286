// Q4_0 projections on either side of the attention step: the attention half
// of the reference's decoder layer step.
//
//   gemv_q4_kernel<true>   RMSNorm of the residual state (reference:
//                          test_28_layers_real.c:200-209) and the QKV
//                          projection with bias (kernel_decoder_layer.cl:83-143,
//                          CPU attention_gqa_benchmark.c:86-106);
//   gemv_q4_kernel<false>  the output projection Wo added into the residual
//                          state (kernel_decoder_layer.cl:386-443).
// RoPE and the KV append stay fused in the split-KV attention kernel that
// runs between the two (gqa_decode.cu), which also lets that kernel stream
// its cache rows before the QKV projection has finished.
//
// Q4_0 (the reference's block_q4_0, attention_gqa_benchmark.c:26-29): 32
// weights per 18-byte block, an fp16 scale d followed by 16 bytes of 4-bit
// codes; weight j < 16 is d * ((qs[j] & 15) - 8), weight j + 16 is
// d * ((qs[j] >> 4) - 8).  A row of d_model = 1536 inputs is 48 blocks =
// 864 bytes (a multiple of 16, so rows are whole 1-D bulk copies).
//
// Each CTA owns 8 consecutive output rows, one warp per row.  It copies
// their weights into shared memory (and the QKV kernel its RMSNorm weights
// into registers) before its programmatic-dependency wait -- the weights do
// not depend on the previous kernel -- then reads the input vector.  Lane
// 2i + h of a row's warp takes, in each of 3 passes, the low (h = 0) or high
// (h = 1) nibbles of block i + 16 * pass, i.e. 16 weights, with 16-bit code
// loads and float4 loads of the input; the 32 partial sums meet by shuffles.
#include <cuda_fp16.h>

#include "gqa_common.cuh"

namespace gqa {

constexpr int kQ4BlockBytes = 18;
constexpr int kDModel = 1536;                                // inputs per row
constexpr int kQ4RowBytes = (kDModel / 32) * kQ4BlockBytes;  // 864
constexpr int kGemvRows = 8;                                 // rows per CTA, a warp each
constexpr int kGemvThreads = 32 * kGemvRows;
constexpr int kGemvPasses = (kDModel / 32) / 16;             // 3 (16 blocks per pass)
constexpr int kGemvInPerThread = kDModel / kGemvThreads;     // 6
constexpr float kRmsEps = 1e-6f;                             // EPSILON of the reference
constexpr long long kGemvWaitBudget = 2000000000LL;

struct GemvParams {
  const uint8_t* w;     // Q4_0 rows
  const float* bias;    // QKV: [M]; Wo: unused
  const float* gamma;   // QKV: RMSNorm weight [kDModel]; Wo: unused
  const float* x;       // QKV: residual state; Wo: attention output  [kDModel]
  float* y;             // QKV: qkv [M] (written); Wo: residual state [M] (added to)
  int M;
  int* status;
};

struct GemvSmem {
  alignas(128) uint8_t w[kGemvRows * kQ4RowBytes];
  alignas(16) float z[kDModel];
  float red[kGemvThreads / 32];
  uint64_t full;
};

// Exact float of (code - 8) for a 4-bit code: 2^23 + code, minus 2^23 + 8.
__device__ __forceinline__ float q4_weight(uint32_t code) {
  return __uint_as_float(0x4B000000u | code) - 8388616.0f;
}

template <bool kQKV>
__global__ void __launch_bounds__(kGemvThreads) gemv_q4_kernel(const GemvParams p) {
  __shared__ GemvSmem sm;
  const int tid = threadIdx.x, row = tid >> 5, lane = tid & 31;
  const int r0 = blockIdx.x * kGemvRows;
  if (tid == 0) {
    mbar_init(&sm.full, 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (tid == 0) {
    mbar_arrive_expect_tx(&sm.full, kGemvRows * kQ4RowBytes);
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(smem_addr(sm.w)), "l"(p.w + (size_t)r0 * kQ4RowBytes),
          "r"(kGemvRows * kQ4RowBytes), "r"(smem_addr(&sm.full)) : "memory");
  }
  float gm[kGemvInPerThread];
  if (kQKV) {
#pragma unroll
    for (int k = 0; k < kGemvInPerThread; ++k) gm[k] = p.gamma[tid + k * kGemvThreads];
  }
  const float bias = (kQKV && lane == 0) ? p.bias[r0 + row] : 0.f;
  // Dependents are released only once this grid runs for real: launched
  // earlier, their waiting CTAs would hold SM space this grid needs.
  pdl_wait();
  pdl_launch_dependents();
  // The residual this row adds to, loaded now rather than after the dot product.
  const float resid = (!kQKV && lane == 0) ? p.y[r0 + row] : 0.f;

  // ---- the input vector (RMSNorm'ed for the QKV projection) ----
  float xv[kGemvInPerThread];
#pragma unroll
  for (int k = 0; k < kGemvInPerThread; ++k) xv[k] = p.x[tid + k * kGemvThreads];
  if (kQKV) {
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < kGemvInPerThread; ++k) ss += xv[k] * xv[k];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    if (lane == 0) sm.red[row] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int k = 0; k < kGemvThreads / 32; ++k) tot += sm.red[k];
    const float scale = 1.0f / sqrtf(tot / (float)kDModel + kRmsEps);
#pragma unroll
    for (int k = 0; k < kGemvInPerThread; ++k) xv[k] = xv[k] * scale * gm[k];
  }
#pragma unroll
  for (int k = 0; k < kGemvInPerThread; ++k) sm.z[tid + k * kGemvThreads] = xv[k];
  __syncthreads();

  // ---- weights landed? (bounded wait; the copy always completes) ----
  if (!mbar_wait_bounded(&sm.full, 0, kGemvWaitBudget)) {
    if (tid == 0) atomicOr(p.status, kStatusWaitTimeout);
    return;
  }

  // ---- one warp per row: lane = (block within the pass, nibble half) ----
  const uint8_t* wrow = sm.w + row * kQ4RowBytes;
  const int half = lane & 1, shift = 4 * half;
  float acc = 0.f;
#pragma unroll
  for (int pass = 0; pass < kGemvPasses; ++pass) {
    const int b = (lane >> 1) + 16 * pass;
    const uint8_t* blk = wrow + b * kQ4BlockBytes;
    const float d = __half2float(*reinterpret_cast<const __half*>(blk));
    const uint16_t* qs = reinterpret_cast<const uint16_t*>(blk + 2);
    const float4* z4 = reinterpret_cast<const float4*>(sm.z + 32 * b + 16 * half);
    float a = 0.f;
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const float4 z = z4[m];
      const uint32_t v0 = qs[2 * m], v1 = qs[2 * m + 1];
      // weights 4m .. 4m+3 of this half: byte 4m+e holds weight 4m+e (low
      // nibble, half 0) or 16+4m+e (high nibble, half 1)
      a = fmaf(q4_weight((v0 >> shift) & 15u), z.x, a);
      a = fmaf(q4_weight((v0 >> (8 + shift)) & 15u), z.y, a);
      a = fmaf(q4_weight((v1 >> shift) & 15u), z.z, a);
      a = fmaf(q4_weight((v1 >> (8 + shift)) & 15u), z.w, a);
    }
    acc = fmaf(d, a, acc);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (lane == 0) {
    if (kQKV)
      p.y[r0 + row] = acc + bias;
    else
      p.y[r0 + row] = resid + acc;
  }
}

static cudaError_t launch_gemv(const void* fn, const GemvParams& p, cudaStream_t st, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.M / kGemvRows);
  cfg.blockDim = dim3(kGemvThreads);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  GemvParams copy = p;
  void* args[] = {&copy};
  return cudaLaunchKernelExC(&cfg, fn, args);
}

int q4_row_bytes() { return kQ4RowBytes; }
int block_d_model() { return kDModel; }

// state -> RMSNorm -> W_qkv (+ bias) -> qkv[M]
cudaError_t launch_qkv_gemv(const void* w, const float* bias, const float* gamma,
                            const float* state, float* qkv, int M, int* status, cudaStream_t st,
                            bool pdl) {
  if (M % kGemvRows) return cudaErrorInvalidValue;
  GemvParams p{static_cast<const uint8_t*>(w), bias, gamma, state, qkv, M, status};
  return launch_gemv((const void*)gemv_q4_kernel<true>, p, st, pdl);
}

// state[M] += W_o * attn
cudaError_t launch_wo_gemv(const void* w, const float* attn, float* state, int M, int* status,
                           cudaStream_t st, bool pdl) {
  if (M % kGemvRows) return cudaErrorInvalidValue;
  GemvParams p{static_cast<const uint8_t*>(w), nullptr, nullptr, attn, state, M, status};
  return launch_gemv((const void*)gemv_q4_kernel<false>, p, st, pdl);
}

}  // namespace gqa
