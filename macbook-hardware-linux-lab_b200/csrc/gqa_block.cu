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
// Each CTA owns 16 consecutive output rows.  It copies their weights into
// shared memory before its programmatic-dependency wait (the weights do not
// depend on the previous kernel), then reads the input vector, and 16
// threads per row each take 3 blocks; the 16 partial sums meet by shuffles.
#include <cuda_fp16.h>

#include "gqa_common.cuh"

namespace gqa {

constexpr int kQ4BlockBytes = 18;
constexpr int kDModel = 1536;                                // inputs per row
constexpr int kQ4RowBytes = (kDModel / 32) * kQ4BlockBytes;  // 864
constexpr int kGemvRows = 16;                                // rows per CTA
constexpr int kGemvThreads = 256;                            // 16 threads per row
constexpr int kGemvBlocksPerThread = (kDModel / 32) / 16;    // 3
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
  float z[kDModel];
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
  const int tid = threadIdx.x, r0 = blockIdx.x * kGemvRows;
  const int row = tid >> 4, sub = tid & 15;
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
  const float bias = (kQKV && sub == 0) ? p.bias[r0 + row] : 0.f;
  pdl_launch_dependents();
  pdl_wait();

  // ---- the input vector (RMSNorm'ed for the QKV projection) ----
  if (kQKV) {
    float ss = 0.f;
    for (int i = tid; i < kDModel; i += kGemvThreads) {
      const float v = p.x[i];
      sm.z[i] = v;
      ss += v * v;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    if ((tid & 31) == 0) sm.red[tid >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int k = 0; k < kGemvThreads / 32; ++k) tot += sm.red[k];
    const float scale = 1.0f / sqrtf(tot / (float)kDModel + kRmsEps);
    for (int i = tid; i < kDModel; i += kGemvThreads) sm.z[i] = sm.z[i] * scale * p.gamma[i];
  } else {
    for (int i = tid; i < kDModel; i += kGemvThreads) sm.z[i] = p.x[i];
  }
  __syncthreads();

  // ---- weights landed? (bounded wait; the copy always completes) ----
  if (!mbar_wait_bounded(&sm.full, 0, kGemvWaitBudget)) {
    if (tid == 0) atomicOr(p.status, kStatusWaitTimeout);
    return;
  }

  // ---- 16 threads per row, blocks sub, sub + 16, sub + 32 ----
  const uint8_t* wrow = sm.w + row * kQ4RowBytes;
  float acc = 0.f;
#pragma unroll
  for (int k = 0; k < kGemvBlocksPerThread; ++k) {
    const int b = sub + 16 * k;
    const uint8_t* blk = wrow + b * kQ4BlockBytes;
    const float d = __half2float(*reinterpret_cast<const __half*>(blk));
    const float* z = sm.z + 32 * b;
    float a0 = 0.f, a1 = 0.f;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const uint32_t q = blk[2 + j];
      a0 = fmaf(q4_weight(q & 15u), z[j], a0);
      a1 = fmaf(q4_weight(q >> 4), z[16 + j], a1);
    }
    acc = fmaf(d, a0 + a1, acc);
  }
#pragma unroll
  for (int off = 8; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (sub == 0) {
    if (kQKV)
      p.y[r0 + row] = acc + bias;
    else
      p.y[r0 + row] += acc;
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
