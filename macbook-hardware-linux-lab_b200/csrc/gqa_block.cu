// Q4_0 projections of the decoder layer around the attention step.
//
//   kQkv     RMSNorm of the residual state (reference: test_28_layers_real.c:
//            200-209) and the QKV projection with bias (kernel_decoder_layer.cl:
//            83-143, CPU attention_gqa_benchmark.c:86-106);
//   kWo      the output projection Wo added into the residual state
//            (kernel_decoder_layer.cl:386-443);
//   kGateUp  RMSNorm (FFN) and the gate and up projections with
//            h = silu(gate) * up (test_28_layers_real.c:298-311, :110-131);
//   kDown    the down projection added into the residual state (:313-317).
// RoPE and the KV append stay fused in the split-KV attention kernel that
// runs between kQkv and kWo (gqa_decode.cu), which also lets that kernel
// stream its cache rows before the QKV projection has finished.
//
// Q4_0 (the reference's block_q4_0, attention_gqa_benchmark.c:26-29): 32
// weights per 18-byte block, an fp16 scale d followed by 16 bytes of 4-bit
// codes; weight j < 16 is d * ((qs[j] & 15) - 8), weight j + 16 is
// d * ((qs[j] >> 4) - 8).  A row of K inputs is K / 32 blocks: 864 bytes for
// K = d_model = 1536, 5040 bytes for K = d_ffn = 8960 (Qwen2.5-1.5B); 504 and
// 2736 bytes for the Qwen2.5-0.5B sizes 896 and 4864 (generate_stream_05b.c:
// 22-26).  A CTA's rows are one 1-D bulk copy, so rows per CTA x row bytes is
// a multiple of 16 for every instance.
//
// Each CTA owns 8 consecutive output rows, one warp per row (two rows --
// gate and up -- for kGateUp; for kDown 4 rows, several warps per row, each
// taking a part of K).  It copies their weights into shared memory (and the
// RMSNorm weights into registers) before its programmatic-dependency wait --
// the weights do not depend on the previous kernel -- then reads the input
// vector into shared memory, block b's 32 values rotated by 4b so that the
// 16 blocks a warp reads at once start on different banks.  Lane 2i + h takes,
// in each pass, the low (h = 0) or high (h = 1) nibbles of block i + 16 * pass,
// i.e. 16 weights: the block's scale and codes come from five aligned 32-bit
// shared loads (the 18-byte blocks sit at 2 or 0 mod 4), the inputs from four
// float4 loads; codes turn into floats four to a word through byte_perm and
// the products run as f32x2 pairs; the 32 partial sums meet by shuffles.
// Dependents are released after the wait, not before.
#include <cuda_fp16.h>

#include "gqa_common.cuh"

namespace gqa {

constexpr int kQ4BlockBytes = 18;
constexpr float kRmsEps = 1e-6f;              // EPSILON of the reference
constexpr long long kGemvWaitBudget = 2000000000LL;

enum GemvMode { kQkv = 0, kWo = 1, kGateUp = 2, kDown = 3 };

// The decoder sizes each instance is built for: model 0 is Qwen2.5-1.5B
// (qwen_server.c), model 1 Qwen2.5-0.5B (generate_stream_05b.c:22-26).
template <int kModel>
struct ModelDims;
template <>
struct ModelDims<0> {
  static constexpr int kDModel = 1536, kDFfn = 8960;
  static constexpr int kDownWarps = 20, kDownSplit = 5;  // 4 rows x 5 parts of 56 blocks
};
template <>
struct ModelDims<1> {
  static constexpr int kDModel = 896, kDFfn = 4864;
  static constexpr int kDownWarps = 16, kDownSplit = 4;  // 4 rows x 4 parts of 38 blocks
};

constexpr int q4_row_bytes_of(int k) { return (k / 32) * kQ4BlockBytes; }

struct GemvParams {
  const uint8_t* w;     // Q4_0 rows (kGateUp: gate)
  const uint8_t* w2;    // kGateUp: up; else unused
  const float* bias;    // kQkv: [M]; else unused
  const float* gamma;   // kQkv / kGateUp: RMSNorm weight [d_model]
  const float* x;       // input vector [K]
  float* y;             // kQkv: qkv, kGateUp: h (written); kWo / kDown: state (added to)
  int M;
  int* status;
};

template <int kMode, int kModel>
struct GemvShape {
  using M = ModelDims<kModel>;
  static constexpr int K = kMode == kDown ? M::kDFfn : M::kDModel;
  static constexpr int kRowBytes = q4_row_bytes_of(K);
  static constexpr int kMats = kMode == kGateUp ? 2 : 1;
  // The down projection (K = d_ffn) splits each row over several warps, 4
  // rows per CTA, for enough warps per SM; the others take a row (or a
  // gate/up pair) per warp, 8 per CTA.
  static constexpr int kWarps = kMode == kDown ? M::kDownWarps : 8;
  static constexpr int kThreads = 32 * kWarps;
  static constexpr int kSplitK = kMode == kDown ? M::kDownSplit : 1;  // warps per row
  static constexpr int kRows = kWarps / kSplitK;                      // rows per CTA
  static constexpr int kWBytes = kMats * kRows * kRowBytes + 16;  // + tail for 32-bit reads
  static constexpr int kInPerThread = (K + kThreads - 1) / kThreads;
  static constexpr bool kEvenIn = K % kThreads == 0;
  static constexpr int kBlocks = K / 32;
  static constexpr bool kNorm = kMode == kQkv || kMode == kGateUp;
  static constexpr bool kAdd = kMode == kWo || kMode == kDown;
  static_assert(K % 32 == 0 && kBlocks % kSplitK == 0 && kWarps % kSplitK == 0, "even split");
  static_assert((kRows * kRowBytes) % 16 == 0, "a CTA's rows must be one bulk copy");
  // dynamic shared memory: weights | z[K] | red[2 * kWarps] | full barrier
  static constexpr size_t kRedBytes = (sizeof(float) * 2 * kWarps + 15) / 16 * 16;
  static constexpr size_t kSmem = (size_t)kWBytes + sizeof(float) * K + kRedBytes + 16;
};

// The reference's stable_silu (test_28_layers_real.c:53-60).
__device__ __forceinline__ float silu_ref(float x) {
  if (x >= 0.0f) return x / (1.0f + expf(-x));
  const float ex = expf(x);
  return x * ex / (1.0f + ex);
}

// Shared-memory index of input j: block j / 32 rotated by 4 per block.
__device__ __forceinline__ int z_index(int j) {
  const int b = j >> 5;
  return (b << 5) + (((j & 31) + 4 * b) & 31);
}

// Dot products of blocks [b_begin, b_end) of kN Q4_0 rows held in shared
// memory (rows 16-byte aligned, row_stride bytes apart) with z, by one warp;
// the rows share the input loads.  The lane's 16 codes of a block come as
// four words of four nibbles, one per byte; each code becomes an exact float
// by byte_perm into 2^23 + code minus 2^23 + 8, and the products run as f32x2
// pairs.  out[i] is the full sum for row i in every lane.
template <int kN>
__device__ __forceinline__ void warp_rows_dot(const uint8_t* wrow, int row_stride, const float* z,
                                              int lane, int b_begin, int b_end, float (&out)[kN]) {
  const int half = lane & 1, shift = 4 * half;
  const float2 code_off = make_float2(-8388616.0f, -8388616.0f);  // -(2^23 + 8)
#pragma unroll
  for (int i = 0; i < kN; ++i) out[i] = 0.f;
#pragma unroll 3
  for (int b = b_begin + (lane >> 1); b < b_end; b += 16) {
    // Block b spans bytes [18b, 18b + 18); words from the 4-byte boundary at
    // or below 18b: an even block starts on it, an odd one 2 bytes past it.
    const int off = b * kQ4BlockBytes;
    const bool odd = (off & 3) != 0;
    const int zb = b << 5;
    float4 zz[4];
#pragma unroll
    for (int m = 0; m < 4; ++m)
      zz[m] = *reinterpret_cast<const float4*>(z + zb + ((16 * half + 4 * m + 4 * b) & 31));
#pragma unroll
    for (int i = 0; i < kN; ++i) {
      const uint32_t* wp = reinterpret_cast<const uint32_t*>(wrow + i * row_stride + (off & ~3));
      const uint32_t w0 = wp[0], w1 = wp[1], w2 = wp[2], w3 = wp[3], w4 = wp[4];
      const float d = __half2float(__ushort_as_half((unsigned short)(odd ? (w0 >> 16) : w0)));
      // codes byte 4m .. 4m+3 (block bytes 2 + 4m ..): word m+1 for an odd
      // block, the upper half of word m and lower half of word m+1 otherwise
      const uint32_t q[4] = {odd ? w1 : __funnelshift_r(w0, w1, 16),
                             odd ? w2 : __funnelshift_r(w1, w2, 16),
                             odd ? w3 : __funnelshift_r(w2, w3, 16),
                             odd ? w4 : __funnelshift_r(w3, w4, 16)};
      float2 a = make_float2(0.f, 0.f);
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        // byte e of Q: the code of weight 4m + e of this half (low nibble of
        // code byte 4m + e for half 0, high nibble for half 1)
        const uint32_t Q = (q[m] >> shift) & 0x0F0F0F0Fu;
        const float2 w01 = __fadd2_rn(
            make_float2(__uint_as_float(__byte_perm(Q, 0x4B00u, 0x5440u)),
                        __uint_as_float(__byte_perm(Q, 0x4B00u, 0x5441u))), code_off);
        const float2 w23 = __fadd2_rn(
            make_float2(__uint_as_float(__byte_perm(Q, 0x4B00u, 0x5442u)),
                        __uint_as_float(__byte_perm(Q, 0x4B00u, 0x5443u))), code_off);
        a = __ffma2_rn(w01, make_float2(zz[m].x, zz[m].y), a);
        a = __ffma2_rn(w23, make_float2(zz[m].z, zz[m].w), a);
      }
      out[i] = fmaf(d, a.x + a.y, out[i]);
    }
  }
#pragma unroll
  for (int i = 0; i < kN; ++i)
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) out[i] += __shfl_xor_sync(0xffffffffu, out[i], off);
}

template <int kMode, int kModel>
__global__ void __launch_bounds__(GemvShape<kMode, kModel>::kThreads)
    gemv_q4_kernel(const GemvParams p) {
  using S = GemvShape<kMode, kModel>;
  extern __shared__ __align__(128) unsigned char gemv_smem[];
  uint8_t* sw = gemv_smem;
  float* sz = reinterpret_cast<float*>(gemv_smem + S::kWBytes);
  float* red = sz + S::K;
  uint64_t* full = reinterpret_cast<uint64_t*>(gemv_smem + S::kWBytes + sizeof(float) * S::K +
                                               S::kRedBytes);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int row = warp / S::kSplitK, part = warp % S::kSplitK;
  const int r0 = blockIdx.x * S::kRows;
  if (tid == 0) {
    mbar_init(full, 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (tid == 0) {
    mbar_arrive_expect_tx(full, S::kMats * S::kRows * S::kRowBytes);
    for (int mat = 0; mat < S::kMats; ++mat) {
      const uint8_t* src = (mat == 0 ? p.w : p.w2) + (size_t)r0 * S::kRowBytes;
      asm volatile(
          "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
          ::"r"(smem_addr(sw + mat * S::kRows * S::kRowBytes)), "l"(src),
            "r"(S::kRows * S::kRowBytes), "r"(smem_addr(full)) : "memory");
    }
  }
  // input j = tid + k * kThreads of this thread exists when in_range(k)
  auto in_range = [&](int k) { return S::kEvenIn || tid + k * S::kThreads < S::K; };
  float gm[S::kInPerThread];
  if (S::kNorm) {
#pragma unroll
    for (int k = 0; k < S::kInPerThread; ++k)
      gm[k] = in_range(k) ? p.gamma[tid + k * S::kThreads] : 0.f;
  }
  const float bias = (kMode == kQkv && lane == 0 && part == 0) ? p.bias[r0 + row] : 0.f;
  // Dependents are released only once this grid runs for real: launched
  // earlier, their waiting CTAs would hold SM space this grid needs.
  pdl_wait();
  pdl_launch_dependents();
  // The residual this row adds to, loaded now rather than after the dot product.
  const float resid = (S::kAdd && lane == 0 && part == 0) ? p.y[r0 + row] : 0.f;

  // ---- the input vector (RMSNorm'ed for the QKV and gate/up projections) ----
  float xv[S::kInPerThread];
#pragma unroll
  for (int k = 0; k < S::kInPerThread; ++k) xv[k] = in_range(k) ? p.x[tid + k * S::kThreads] : 0.f;
  if (S::kNorm) {
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < S::kInPerThread; ++k) ss += xv[k] * xv[k];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int k = 0; k < S::kWarps; ++k) tot += red[k];
    const float scale = 1.0f / sqrtf(tot / (float)S::K + kRmsEps);
#pragma unroll
    for (int k = 0; k < S::kInPerThread; ++k) xv[k] = xv[k] * scale * gm[k];
  }
#pragma unroll
  for (int k = 0; k < S::kInPerThread; ++k)
    if (in_range(k)) sz[z_index(tid + k * S::kThreads)] = xv[k];
  __syncthreads();

  // ---- weights landed? (bounded wait; the copy always completes) ----
  // The decision is made for the whole CTA, which synchronises again below.
  if (!__syncthreads_and(mbar_wait_bounded(full, 0, kGemvWaitBudget))) {
    if (tid == 0) atomicOr(p.status, kStatusWaitTimeout);
    return;
  }

  constexpr int kPartBlocks = S::kBlocks / S::kSplitK;
  float acc[S::kMats];
  warp_rows_dot<S::kMats>(sw + row * S::kRowBytes, S::kRows * S::kRowBytes, sz, lane,
                          part * kPartBlocks, (part + 1) * kPartBlocks, acc);
  if (S::kSplitK > 1) {
    // the other parts of the row's blocks, from the row's other warps
    if (lane == 0) red[S::kWarps + warp] = acc[0];
    __syncthreads();
    if (part != 0) return;
    if (lane == 0)
#pragma unroll
      for (int k = 1; k < S::kSplitK; ++k) acc[0] += red[S::kWarps + warp + k];
  }
  float out;
  if (kMode == kGateUp) {
    out = silu_ref(acc[0]) * acc[S::kMats - 1];
  } else if (kMode == kQkv) {
    out = acc[0] + bias;
  } else {
    out = resid + acc[0];
  }
  if (lane == 0) p.y[r0 + row] = out;
}

template <int kMode, int kModel>
static cudaError_t launch_gemv_model(const GemvParams& p, cudaStream_t st, bool pdl) {
  using S = GemvShape<kMode, kModel>;
  if (p.M % S::kRows) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.M / S::kRows);
  cfg.blockDim = dim3(S::kThreads);
  cfg.dynamicSmemBytes = S::kSmem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  GemvParams copy = p;
  void* args[] = {&copy};
  return cudaLaunchKernelExC(&cfg, (const void*)gemv_q4_kernel<kMode, kModel>, args);
}

template <int kMode>
static cudaError_t launch_gemv(int model, const GemvParams& p, cudaStream_t st, bool pdl) {
  switch (model) {
    case 0: return launch_gemv_model<kMode, 0>(p, st, pdl);
    case 1: return launch_gemv_model<kMode, 1>(p, st, pdl);
    default: return cudaErrorInvalidValue;
  }
}

int block_d_model(int model) {
  return model == 0 ? ModelDims<0>::kDModel : model == 1 ? ModelDims<1>::kDModel : 0;
}
int block_d_ffn(int model) {
  return model == 0 ? ModelDims<0>::kDFfn : model == 1 ? ModelDims<1>::kDFfn : 0;
}
int block_max_d_ffn() { return ModelDims<0>::kDFfn > ModelDims<1>::kDFfn ? ModelDims<0>::kDFfn
                                                                         : ModelDims<1>::kDFfn; }

template <int kMode, int kModel>
static cudaError_t allow_smem() {
  return cudaFuncSetAttribute((const void*)gemv_q4_kernel<kMode, kModel>,
                              cudaFuncAttributeMaxDynamicSharedMemorySize,
                              (int)GemvShape<kMode, kModel>::kSmem);
}

cudaError_t prepare_block_kernels() {
  cudaError_t e = allow_smem<kDown, 0>();
  if (e == cudaSuccess) e = allow_smem<kDown, 1>();
  if (e == cudaSuccess) e = allow_smem<kGateUp, 0>();
  if (e == cudaSuccess) e = allow_smem<kGateUp, 1>();
  return e;
}

// state -> RMSNorm -> W_qkv (+ bias) -> qkv[M]
cudaError_t launch_qkv_gemv(int model, const void* w, const float* bias, const float* gamma,
                            const float* state, float* qkv, int M, int* status, cudaStream_t st,
                            bool pdl) {
  GemvParams p{static_cast<const uint8_t*>(w), nullptr, bias, gamma, state, qkv, M, status};
  return launch_gemv<kQkv>(model, p, st, pdl);
}

// state[M] += W_o * attn
cudaError_t launch_wo_gemv(int model, const void* w, const float* attn, float* state, int M,
                           int* status, cudaStream_t st, bool pdl) {
  GemvParams p{static_cast<const uint8_t*>(w), nullptr, nullptr, nullptr, attn, state, M, status};
  return launch_gemv<kWo>(model, p, st, pdl);
}

// state -> RMSNorm -> h[d_ffn] = silu(W_gate z) * (W_up z)
cudaError_t launch_gateup_gemv(int model, const void* w_gate, const void* w_up,
                               const float* gamma, const float* state, float* h, int* status,
                               cudaStream_t st, bool pdl) {
  GemvParams p{static_cast<const uint8_t*>(w_gate), static_cast<const uint8_t*>(w_up), nullptr,
               gamma, state, h, block_d_ffn(model), status};
  return launch_gemv<kGateUp>(model, p, st, pdl);
}

// state[d_model] += W_down * h
cudaError_t launch_down_gemv(int model, const void* w_down, const float* h, float* state,
                             int* status, cudaStream_t st, bool pdl) {
  GemvParams p{static_cast<const uint8_t*>(w_down), nullptr, nullptr, nullptr, h, state,
               block_d_model(model), status};
  return launch_gemv<kDown>(model, p, st, pdl);
}

}  // namespace gqa
