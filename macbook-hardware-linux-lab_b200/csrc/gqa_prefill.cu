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
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <math_constants.h>

#include "gqa_common.cuh"

namespace gqa {

constexpr int kPT = 128;                          // tile rows (queries or keys)
constexpr int kImgElems = kPT * kHeadDim;         // one tile image (bf16 elements)
constexpr int kImgBytes = kImgElems * 2;          // 32 KB
constexpr int kKBlockElems = kPT * 64;            // one 64-wide K block (16 KB)
constexpr int kPrefillThreads = 320;              // warps 0-7 softmax, 8 loader, 9 MMA
constexpr int kTmemCols = 512;                    // S_A | S_B | O_A | O_B
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

// 128 consecutive fp32 columns of this thread's TMEM lane, waited in the same statement.
__device__ __forceinline__ void tmem_ld128(uint32_t taddr, float (&v)[128]) {
  uint32_t r[128];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x128.b32 {"
      "%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, "
      "%32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, "
      "%48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63, "
      "%64, %65, %66, %67, %68, %69, %70, %71, %72, %73, %74, %75, %76, %77, %78, %79, "
      "%80, %81, %82, %83, %84, %85, %86, %87, %88, %89, %90, %91, %92, %93, %94, %95, "
      "%96, %97, %98, %99, %100, %101, %102, %103, %104, %105, %106, %107, %108, %109, %110, %111, "
      "%112, %113, %114, %115, %116, %117, %118, %119, %120, %121, %122, %123, %124, %125, %126, %127}, [%128];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]),
        "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]),
        "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]),
        "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]),
        "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63]),
        "=r"(r[64]), "=r"(r[65]), "=r"(r[66]), "=r"(r[67]), "=r"(r[68]), "=r"(r[69]), "=r"(r[70]), "=r"(r[71]),
        "=r"(r[72]), "=r"(r[73]), "=r"(r[74]), "=r"(r[75]), "=r"(r[76]), "=r"(r[77]), "=r"(r[78]), "=r"(r[79]),
        "=r"(r[80]), "=r"(r[81]), "=r"(r[82]), "=r"(r[83]), "=r"(r[84]), "=r"(r[85]), "=r"(r[86]), "=r"(r[87]),
        "=r"(r[88]), "=r"(r[89]), "=r"(r[90]), "=r"(r[91]), "=r"(r[92]), "=r"(r[93]), "=r"(r[94]), "=r"(r[95]),
        "=r"(r[96]), "=r"(r[97]), "=r"(r[98]), "=r"(r[99]), "=r"(r[100]), "=r"(r[101]), "=r"(r[102]), "=r"(r[103]),
        "=r"(r[104]), "=r"(r[105]), "=r"(r[106]), "=r"(r[107]), "=r"(r[108]), "=r"(r[109]), "=r"(r[110]), "=r"(r[111]),
        "=r"(r[112]), "=r"(r[113]), "=r"(r[114]), "=r"(r[115]), "=r"(r[116]), "=r"(r[117]), "=r"(r[118]), "=r"(r[119]),
        "=r"(r[120]), "=r"(r[121]), "=r"(r[122]), "=r"(r[123]), "=r"(r[124]), "=r"(r[125]), "=r"(r[126]), "=r"(r[127])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 128; ++i) v[i] = __uint_as_float(r[i]);
}

// 64 consecutive 32-bit columns of this thread's TMEM lane, waited in the same statement.
__device__ __forceinline__ void tmem_st64(uint32_t taddr, const uint32_t (&v)[64]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x64.b32 [%0], {"
      "%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32, "
      "%33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, %48, "
      "%49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63, %64};\n\t"
      "tcgen05.wait::st.sync.aligned;"
      ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
        "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]),
        "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]),
        "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31]),
        "r"(v[32]), "r"(v[33]), "r"(v[34]), "r"(v[35]), "r"(v[36]), "r"(v[37]), "r"(v[38]), "r"(v[39]),
        "r"(v[40]), "r"(v[41]), "r"(v[42]), "r"(v[43]), "r"(v[44]), "r"(v[45]), "r"(v[46]), "r"(v[47]),
        "r"(v[48]), "r"(v[49]), "r"(v[50]), "r"(v[51]), "r"(v[52]), "r"(v[53]), "r"(v[54]), "r"(v[55]),
        "r"(v[56]), "r"(v[57]), "r"(v[58]), "r"(v[59]), "r"(v[60]), "r"(v[61]), "r"(v[62]), "r"(v[63])
      : "memory");
}

// max of three (one instruction on sm_100).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Two floats to a bf16 pair (lo = a), round to nearest even.
__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 b2 = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&b2);
}

__device__ __forceinline__ void named_barrier_sync(int id, int n_threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n_threads) : "memory");
}

// Packed fp32 pair arithmetic (one f32x2 instruction for two lanes of work).
__device__ __forceinline__ void ffma2(float& d0, float& d1, float a0, float a1, float b0, float b1,
                                      float c0, float c1) {
  asm("{\n\t.reg .b64 a, b, c, d;\n\t"
      "mov.b64 a, {%2, %3};\n\tmov.b64 b, {%4, %5};\n\tmov.b64 c, {%6, %7};\n\t"
      "fma.rn.f32x2 d, a, b, c;\n\t"
      "mov.b64 {%0, %1}, d;\n\t}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1), "f"(c0), "f"(c1));
}

__device__ __forceinline__ void fadd2(float& d0, float& d1, float a0, float a1, float b0, float b1) {
  asm("{\n\t.reg .b64 a, b, d;\n\t"
      "mov.b64 a, {%2, %3};\n\tmov.b64 b, {%4, %5};\n\t"
      "add.rn.f32x2 d, a, b;\n\t"
      "mov.b64 {%0, %1}, d;\n\t}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// ---------------------------------------------------------------------------
// Prep: RoPE, bf16, swizzled tile images, cache append
// ---------------------------------------------------------------------------
// RoPE table for the prefill: cs[pos][i] = (cos, sin) of pos * inv_freq[i],
// the angle formed in fp32 exactly as the decode kernels form it.
__global__ void prefill_rope_table_kernel(const float* inv_freq, float2* cs, int n_pos) {
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= n_pos * kHalf) return;
  float sn, c;
  sincosf((float)(idx / kHalf) * inv_freq[idx % kHalf], &sn, &c);
  cs[idx] = make_float2(c, sn);
}

struct PrefillPrepParams {
  const float* qkv;      // [n_seq][S][(n_q + 2 n_kv) * 128]
  long long seq_stride;  // floats between sequences
  int S;
  int n_q, n_kv;
  const float2* rope_cs; // [>= S][64] (cos, sin)
  __nv_bfloat16* qimg;   // [n_seq][n_q][S/128] images
  __nv_bfloat16* kimg;   // [n_seq][n_kv][S/128] images
  __nv_bfloat16* vimg;   // [n_seq][n_kv][S/128] images (transposed)
  float* const* k_caches;  // optional [n_seq] fp32 caches [n_kv][t_max][128]
  float* const* v_caches;
  int t_max;
};

__device__ __forceinline__ uint32_t bf16x2_rn(float lo, float hi) {
  __nv_bfloat162 b = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&b);
}

// One block per (head slot, 128-token tile, sequence).  Head slots 0..n_q-1
// are q heads, then n_kv k heads, then n_kv v heads.  Every thread produces
// whole 16-byte chunks (8 bf16) of the swizzled image, so image stores are
// 16-byte vectors; reads of the fp32 rows are 32-byte pieces of one row
// across neighbouring threads.
__global__ void __launch_bounds__(256) prefill_prep_kernel(const PrefillPrepParams p) {
  const int unit = blockIdx.x, tile = blockIdx.y, seq = blockIdx.z, tid = threadIdx.x;
  // The attention kernel may set itself up (barriers, tensor memory) while
  // this grid finishes; it waits for all of it before it reads an image.
  pdl_launch_dependents();
  const int width = (p.n_q + 2 * p.n_kv) * kHeadDim;
  const int n_tiles = p.S / kPT;
  const float* base = p.qkv + (long long)seq * p.seq_stride + (long long)tile * kPT * width +
                      (long long)unit * kHeadDim;
  if (unit < p.n_q + p.n_kv) {
    // q or k head: rotate pairs (i, i + 64); item = (row r, chunk c of 8 pairs)
    const bool is_q = unit < p.n_q;
    const int kh = unit - p.n_q;
    __nv_bfloat16* img =
        is_q ? p.qimg + ((long long)(seq * p.n_q + unit) * n_tiles + tile) * kImgElems
             : p.kimg + ((long long)(seq * p.n_kv + kh) * n_tiles + tile) * kImgElems;
    float* kc = (!is_q && p.k_caches) ? p.k_caches[seq] : nullptr;
    for (int item = tid; item < kPT * 8; item += blockDim.x) {
      const int r = item >> 3, c = item & 7;
      const int pos = tile * kPT + r;
      const float* row = base + (long long)r * width;
      const float4 a0 = *reinterpret_cast<const float4*>(row + 8 * c);
      const float4 a1 = *reinterpret_cast<const float4*>(row + 8 * c + 4);
      const float4 b0 = *reinterpret_cast<const float4*>(row + kHalf + 8 * c);
      const float4 b1 = *reinterpret_cast<const float4*>(row + kHalf + 8 * c + 4);
      const float4* csp = reinterpret_cast<const float4*>(p.rope_cs + (long long)pos * kHalf + 8 * c);
      const float4 t0 = csp[0], t1 = csp[1], t2 = csp[2], t3 = csp[3];  // (cos, sin) x 8
      const float x0[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float x1[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
      const float co[8] = {t0.x, t0.z, t1.x, t1.z, t2.x, t2.z, t3.x, t3.z};
      const float si[8] = {t0.y, t0.w, t1.y, t1.w, t2.y, t2.w, t3.y, t3.w};
      float y0[8], y1[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        y0[e] = x0[e] * co[e] - x1[e] * si[e];
        y1[e] = x0[e] * si[e] + x1[e] * co[e];
      }
      *reinterpret_cast<uint4*>(img + sw_offset(r, 8 * c)) =
          make_uint4(bf16x2_rn(y0[0], y0[1]), bf16x2_rn(y0[2], y0[3]), bf16x2_rn(y0[4], y0[5]),
                     bf16x2_rn(y0[6], y0[7]));
      *reinterpret_cast<uint4*>(img + sw_offset(r, kHalf + 8 * c)) =
          make_uint4(bf16x2_rn(y1[0], y1[1]), bf16x2_rn(y1[2], y1[3]), bf16x2_rn(y1[4], y1[5]),
                     bf16x2_rn(y1[6], y1[7]));
      if (kc) {
        float* dst = kc + ((long long)kh * p.t_max + pos) * kHeadDim;
        if ((reinterpret_cast<uintptr_t>(kc) & 15) == 0) {
          *reinterpret_cast<float4*>(dst + 8 * c) = make_float4(y0[0], y0[1], y0[2], y0[3]);
          *reinterpret_cast<float4*>(dst + 8 * c + 4) = make_float4(y0[4], y0[5], y0[6], y0[7]);
          *reinterpret_cast<float4*>(dst + kHalf + 8 * c) = make_float4(y1[0], y1[1], y1[2], y1[3]);
          *reinterpret_cast<float4*>(dst + kHalf + 8 * c + 4) =
              make_float4(y1[4], y1[5], y1[6], y1[7]);
        } else {  // a cache that is only 4-byte aligned
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            dst[8 * c + e] = y0[e];
            dst[kHalf + 8 * c + e] = y1[e];
          }
        }
      }
    }
  } else {
    // v head: transposed image, row = head dim d, K = token; item = (d, 8 tokens)
    const int vh = unit - p.n_q - p.n_kv;
    __nv_bfloat16* img = p.vimg + ((long long)(seq * p.n_kv + vh) * n_tiles + tile) * kImgElems;
    float* vc = p.v_caches ? p.v_caches[seq] : nullptr;
    for (int item = tid; item < kPT * (kPT / 8); item += blockDim.x) {
      const int d = item & (kHeadDim - 1), rg = item >> 7;
      float x[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) x[e] = base[(long long)(8 * rg + e) * width + d];
      *reinterpret_cast<uint4*>(img + sw_offset(d, 8 * rg)) =
          make_uint4(bf16x2_rn(x[0], x[1]), bf16x2_rn(x[2], x[3]), bf16x2_rn(x[4], x[5]),
                     bf16x2_rn(x[6], x[7]));
      if (vc) {
#pragma unroll
        for (int e = 0; e < 8; ++e)
          vc[((long long)vh * p.t_max + tile * kPT + 8 * rg + e) * kHeadDim + d] = x[e];
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Attention
// ---------------------------------------------------------------------------
struct PrefillAttnParams {
  // out as a 2-D fp32 tensor (columns n_q * 128, rows n_seq * S), stored
  // through 32 x 32 boxes with the 128-byte swizzle.
  CUtensorMap out_map;
  const __nv_bfloat16* qimg;
  const __nv_bfloat16* kimg;
  const __nv_bfloat16* vimg;
  float* out;            // [n_seq][S][n_q * 128]
  int S;
  int n_q, n_kv;
  int n_seq;
  float scale_log2;      // softmax scale * log2(e)
  int* status;
  int* sched;            // [2] next item, CTAs done; zero between launches
};

// A work item is (128-token query tile, pair of q heads of one KV group,
// sequence): both heads share every K / V^T tile the CTA stages, which feeds
// two S = QK^T and two O += PV MMAs.  The kernel is persistent: one CTA per
// SM walks a list of items, so the Q load of the next item and the output
// stores of the last one overlap the MMAs.
struct PrefillSmem {
  __nv_bfloat16 q[2][kImgElems];   // the two Q tiles (head 2h, 2h+1)
  __nv_bfloat16 k[2][kImgElems];   // K tile ring
  __nv_bfloat16 vt[2][kImgElems];  // V^T tile ring
  float stage[8][32 * 32];         // per softmax warp: 32 rows x 32 floats of output
  int item_ring[4];                // item ids handed out by the loader (-1: none left)
  uint64_t item_full[4], item_empty[4];
  uint64_t q_full[2], q_empty[2], k_full[2], k_empty[2], v_full[2], v_empty[2];
  uint64_t s_full[2], p_full[2], o_final[2], drain;
  uint32_t tmem_base;
  int err;
};

constexpr size_t prefill_smem_bytes() { return sizeof(PrefillSmem) + 1024; }  // + alignment slack

// try_wait with a suspend-time hint: a thread whose phase is not complete
// sleeps in the barrier unit (until the phase completes or the hint runs out)
// instead of spinning, so a waiting warp leaves the issue slots of its
// scheduler to the softmax warp that shares it.
constexpr uint32_t kSuspendHintNs = 20000;

__device__ __forceinline__ bool mbar_try_wait_suspend(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity), "r"(kSuspendHintNs)
      : "memory");
  return ok != 0;
}

// Bounded wait that also gives up as soon as another role has raised `err`.
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, volatile int* err) {
  if (mbar_try_wait_suspend(bar, parity)) return true;
  const long long start = clock64();
  while (!mbar_try_wait_suspend(bar, parity)) {
    if (*err) return false;
    if (clock64() - start > kPrefillWaitBudget) {
      atomicOr((int*)err, 1);
      return false;
    }
  }
  return true;
}

// O += P.V with P (bf16, M = 128 query rows x K = 16 keys) read from tensor
// memory: row = TMEM lane, two consecutive keys per 32-bit column.
__device__ __forceinline__ void umma_bf16_tmem_a(uint32_t d_tmem, uint32_t a_tmem, uint64_t b,
                                                 bool acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
      ::"r"(d_tmem), "r"(a_tmem), "l"(b), "r"(kIdescBf16M128N128), "r"((uint32_t)acc));
}

// Items are numbered in decreasing causal length (query tile n_tiles-1 first)
// and handed out dynamically: the loader of a CTA takes the next number from a
// global counter when it is ready for another item, so SMs that finish early
// take more of the short tail items.  The loader publishes each number in a
// 4-slot ring that the MMA thread and the eight softmax warps read in order.
struct PrefillItem {
  int i, pair, seq;
};

constexpr int kItemConsumers = 9;  // the MMA thread and one arrival per softmax warp

// Number n of this CTA's item sequence (blocks until the loader published it);
// -1 when none is left.  `ok` turns false on a timeout or another role's error.
__device__ __forceinline__ int item_take(PrefillSmem& sm, int n, volatile int* err, bool& ok) {
  const int slot = n & 3;
  ok = wait_or_abort(&sm.item_full[slot], (n >> 2) & 1, err);
  return ok ? *reinterpret_cast<volatile int*>(&sm.item_ring[slot]) : -1;
}

__device__ __forceinline__ PrefillItem prefill_item(int k, int n_tiles, int n_pairs, int n_seq) {
  const int per_tile = n_pairs * n_seq;
  const int t = k / per_tile, rem = k % per_tile;
  return PrefillItem{n_tiles - 1 - t, rem % n_pairs, rem / n_pairs};
}

// Tensor memory plan (512 columns, all 128 lanes): S of head g in columns
// [128 g, 128 g + 128), O of head g in [256 + 128 g, 384 + 128 g).  P of head g
// (bf16 pairs) overwrites the first 64 columns of its own S once the softmax
// thread has read that S row into registers; the next S MMA of head g is
// issued after the P.V MMA that reads it, and tcgen05.mma operations of one
// thread execute in issue order.
//
// The MMA warp walks the key tiles of all its items as one sequence t and
// issues, per t (heads A = 0, B = 1):
//   PV_A(t), S_A(t+1), PV_B(t), S_B(t+1)
// where t+1 may be the first tile of the next item (other Q, other causal
// range).  The softmax of one head thus always overlaps two MMAs of the other,
// and the commit that signals S_g(t+1) also covers PV_g(t): when the softmax
// thread sees S its O row is final up to tile t and may be rescaled.  The
// next item's first P.V (which overwrites O with accumulate = 0) is issued
// only after the softmax warps signalled that P, and they read O for the
// epilogue before they produce it.
__global__ void __launch_bounds__(kPrefillThreads, 1)
    prefill_attn_kernel(const __grid_constant__ PrefillAttnParams p) {
  extern __shared__ unsigned char smem_raw[];
  // The swizzled operand images need 1 KB alignment.
  PrefillSmem& sm = *reinterpret_cast<PrefillSmem*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_tiles = p.S / kPT;
  const int n_pairs = p.n_q / 2;
  const int n_items = n_tiles * n_pairs * p.n_seq;
  const int group = p.n_q / p.n_kv;
  volatile int* err = &sm.err;

  if (tid == 0) {
    for (int s = 0; s < 4; ++s) {
      mbar_init(&sm.item_full[s], 1);
      mbar_init(&sm.item_empty[s], kItemConsumers);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sm.q_full[s], 1);
      mbar_init(&sm.q_empty[s], 1);
      mbar_init(&sm.k_full[s], 1);
      mbar_init(&sm.k_empty[s], 1);
      mbar_init(&sm.v_full[s], 1);
      mbar_init(&sm.v_empty[s], 1);
      mbar_init(&sm.s_full[s], 1);
      mbar_init(&sm.p_full[s], 4);  // one arrival per softmax warp
      mbar_init(&sm.o_final[s], 1);
    }
    mbar_init(&sm.drain, 1);
    sm.err = 0;
    fence_barrier_init();
  }
  if (warp == 9) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 ::"r"(smem_addr(&sm.tmem_base)), "r"(kTmemCols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  // The images and the item counter come from the prep kernel before this one.
  pdl_wait();

  if (warp == 8) {
    // ---- loader ----
    if (lane == 0) {
      const uint64_t policy = l2_policy_evict_first();
      int kv = 0, q_issued = 0, k_issued = 0, v_issued = 0;
      bool ok = true;
      for (int rd = 0; ok; ++rd) {
        const int slot = rd & 3;
        if (rd >= 4 && !wait_or_abort(&sm.item_empty[slot], ((rd >> 2) - 1) & 1, err)) {
          ok = false;
          break;
        }
        int k = atomicAdd(p.sched, 1);
        if (k >= n_items) k = -1;
        sm.item_ring[slot] = k;
        mbar_arrive(&sm.item_full[slot]);  // release: the ring entry is visible to the waiters
        if (k < 0) break;
        const PrefillItem it = prefill_item(k, n_tiles, n_pairs, p.n_seq);
        const int kvh = (2 * it.pair) / group;
        for (int g = 0; g < 2 && ok; ++g) {
          if (rd > 0 && !wait_or_abort(&sm.q_empty[g], (rd - 1) & 1, err)) { ok = false; break; }
          const long long q_off =
              ((long long)(it.seq * p.n_q + 2 * it.pair + g) * n_tiles + it.i) * kImgElems;
          mbar_arrive_expect_tx(&sm.q_full[g], kImgBytes);
          bulk_copy_g2s(sm.q[g], p.qimg + q_off, kImgBytes, &sm.q_full[g], policy);
          ++q_issued;
        }
        const long long kv_base = (long long)(it.seq * p.n_kv + kvh) * n_tiles * kImgElems;
        for (int j = 0; j <= it.i && ok; ++j, ++kv) {
          const int st = kv & 1;
          const uint32_t reuse = ((kv >> 1) - 1) & 1;
          // K and V tiles are re-read by the other q heads of the group: keep them in L2.
          if (kv >= 2 && !wait_or_abort(&sm.k_empty[st], reuse, err)) { ok = false; break; }
          mbar_arrive_expect_tx(&sm.k_full[st], kImgBytes);
          asm volatile(
              "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
              ::"r"(smem_addr(sm.k[st])), "l"(p.kimg + kv_base + (long long)j * kImgElems),
                "r"(kImgBytes), "r"(smem_addr(&sm.k_full[st])) : "memory");
          ++k_issued;
          if (kv >= 2 && !wait_or_abort(&sm.v_empty[st], reuse, err)) { ok = false; break; }
          mbar_arrive_expect_tx(&sm.v_full[st], kImgBytes);
          asm volatile(
              "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
              ::"r"(smem_addr(sm.vt[st])), "l"(p.vimg + kv_base + (long long)j * kImgElems),
                "r"(kImgBytes), "r"(smem_addr(&sm.v_full[st])) : "memory");
          ++v_issued;
        }
      }
      if (*err) {
        // Let the copies already issued land before the CTA's shared memory
        // can be handed to another CTA (copies always complete).
        for (int n = q_issued - 2; n < q_issued; ++n)
          if (n >= 0) mbar_wait_bounded(&sm.q_full[n & 1], (n >> 1) & 1, kPrefillWaitBudget);
        for (int n = k_issued - 2; n < k_issued; ++n)
          if (n >= 0) mbar_wait_bounded(&sm.k_full[n & 1], (n >> 1) & 1, kPrefillWaitBudget);
        for (int n = v_issued - 2; n < v_issued; ++n)
          if (n >= 0) mbar_wait_bounded(&sm.v_full[n & 1], (n >> 1) & 1, kPrefillWaitBudget);
      }
    }
    __syncwarp();  // the other lanes wait here, so the warp reaches the block barrier converged
  } else if (warp == 9) {
    // ---- MMA issuer ----
    if (lane == 0) {
      auto issue_s = [&](int g, int kv) {
        const uint32_t q_addr = smem_addr(sm.q[g]);
        const uint32_t k_addr = smem_addr(sm.k[kv & 1]);
#pragma unroll
        for (int ks = 0; ks < kHeadDim / 16; ++ks) {
          const uint32_t off = (ks >> 2) * (kKBlockElems * 2) + (ks & 3) * 32;
          umma_bf16(tmem + 128 * g, umma_smem_desc(q_addr + off),
                    umma_smem_desc(k_addr + off), ks > 0);
        }
        umma_commit(&sm.s_full[g]);
      };
      auto issue_pv = [&](int g, int kv, bool acc) {
        const uint32_t v_addr = smem_addr(sm.vt[kv & 1]);
#pragma unroll
        for (int ks = 0; ks < kPT / 16; ++ks) {
          const uint32_t off = (ks >> 2) * (kKBlockElems * 2) + (ks & 3) * 32;
          umma_bf16_tmem_a(tmem + 256 + 128 * g, tmem + 128 * g + ks * 8,
                           umma_smem_desc(v_addr + off), acc || ks > 0);
        }
      };
      // Position in the flat tile sequence: item round rd, tile j of it, and
      // the running K/V tile index kv.
      int rd = 0, kv = 0;
      bool ok = true;
      int k = item_take(sm, 0, err, ok);
      if (ok) mbar_arrive(&sm.item_empty[0]);
      ok = ok && k >= 0;
      PrefillItem it{};
      if (ok) {
        it = prefill_item(k, n_tiles, n_pairs, p.n_seq);
        ok = wait_or_abort(&sm.q_full[0], 0, err) && wait_or_abort(&sm.k_full[0], 0, err);
        if (ok) {
          tc_fence_after();
          issue_s(0, 0);
          if (it.i == 0) umma_commit(&sm.q_empty[0]);
          ok = wait_or_abort(&sm.q_full[1], 0, err);
        }
        if (ok) {
          tc_fence_after();
          issue_s(1, 0);
          if (it.i == 0) umma_commit(&sm.q_empty[1]);
          umma_commit(&sm.k_empty[0]);
        }
      }
      int j = 0;
      while (ok) {
        // the tile after (rd, j): same item, or the first tile of the next one
        int rd_n = rd, j_n = j + 1;
        PrefillItem it_n = it;
        bool more = true;
        if (j_n > it.i) {
          rd_n = rd + 1;
          j_n = 0;
          const int kn = item_take(sm, rd_n, err, ok);
          if (!ok) break;
          mbar_arrive(&sm.item_empty[rd_n & 3]);
          more = kn >= 0;
          if (more) it_n = prefill_item(kn, n_tiles, n_pairs, p.n_seq);
        }
        const int kv_n = kv + 1;
        const bool last_of_item = (j == it.i);
        const bool n_last = more && (j_n == it_n.i);  // tile t+1 is the last of its item
        if (!wait_or_abort(&sm.p_full[0], kv & 1, err) ||
            !wait_or_abort(&sm.v_full[kv & 1], (kv >> 1) & 1, err)) { ok = false; break; }
        tc_fence_after();
        issue_pv(0, kv, j > 0);
        if (last_of_item) umma_commit(&sm.o_final[0]);
        if (more) {
          if ((j_n == 0 && !wait_or_abort(&sm.q_full[0], rd_n & 1, err)) ||
              !wait_or_abort(&sm.k_full[kv_n & 1], (kv_n >> 1) & 1, err)) { ok = false; break; }
          tc_fence_after();
          issue_s(0, kv_n);
          if (n_last) umma_commit(&sm.q_empty[0]);
        }
        if (!wait_or_abort(&sm.p_full[1], kv & 1, err)) { ok = false; break; }
        tc_fence_after();
        issue_pv(1, kv, j > 0);
        umma_commit(&sm.v_empty[kv & 1]);
        if (last_of_item) umma_commit(&sm.o_final[1]);
        if (more) {
          if (j_n == 0 && !wait_or_abort(&sm.q_full[1], rd_n & 1, err)) { ok = false; break; }
          tc_fence_after();
          issue_s(1, kv_n);
          if (n_last) umma_commit(&sm.q_empty[1]);
          umma_commit(&sm.k_empty[kv_n & 1]);
        } else {
          break;
        }
        rd = rd_n;
        j = j_n;
        it = it_n;
        kv = kv_n;
      }
      // Whatever happened, no MMA may still be running when TMEM is freed.
      umma_commit(&sm.drain);
      mbar_wait_bounded(&sm.drain, 0, kPrefillWaitBudget);
    }
    __syncwarp();
  } else {
    // ---- softmax: warps 4g..4g+3 serve head g; thread owns query row r ----
    const int g = warp >> 2, r = tid & 127;
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t t_s = tmem + lane_off + 128 * g;
    const uint32_t t_o = tmem + lane_off + 256 + 128 * g;
    const float sc = p.scale_log2;
    float* slice = sm.stage[warp];
    int tc = 0;  // S tiles of this head so far (s_full / p_full parity)
    bool ok = true;
    for (int rd = 0; ok; ++rd) {
      int k = item_take(sm, rd, err, ok);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.item_empty[rd & 3]);
      if (k < 0) break;
      const PrefillItem it = prefill_item(k, n_tiles, n_pairs, p.n_seq);
      float m = -CUDART_INF_F, l = 0.f;
      for (int j = 0; j <= it.i; ++j, ++tc) {
        // Waits are voted so the warp stays converged for the warp-collective
        // tensor-memory loads and stores.
        ok = __all_sync(0xffffffffu, wait_or_abort(&sm.s_full[g], tc & 1, err));
        if (!ok) break;
        tc_fence_after();
        // Weights against the running reference max m.  The row max is taken
        // only on the first tile of the item, or when the weights of this
        // tile sum past 2^8 in some row of the warp (a score moved well above
        // m; the sum also catches an overflow): then the S rows are loaded
        // again, m moves to the row max, the tile is recomputed, and l and
        // the O row are rescaled.  Otherwise no max pass is spent on the tile.
        float alpha = 1.f, sum0 = 0.f, sum1 = 0.f;
        uint32_t pk[kPT / 2];
        bool fresh = (j == 0);
#pragma unroll 1
        for (int pass = 0; pass < 2; ++pass) {
          float s[kPT];
          tmem_ld128(t_s, s);
          if (j == it.i) {
#pragma unroll
            for (int c = 0; c < kPT; ++c)
              if (c > r) s[c] = -CUDART_INF_F;  // causal: keys after the query
          }
          if (fresh) {
            float mx0 = s[0], mx1 = s[1], mx2 = s[2], mx3 = s[3];
#pragma unroll
            for (int c = 4; c < kPT; c += 8) {
              mx0 = fmax3(mx0, s[c], s[c + 1]);
              mx1 = fmax3(mx1, s[c + 2], s[c + 3]);
              mx2 = fmax3(mx2, s[c + 4], s[c + 5]);
              mx3 = fmax3(mx3, s[c + 6], s[c + 7]);
            }
            const float mn = fmaxf(m, fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3)) * sc);
            if (j > 0) alpha = fast_exp2(m - mn);
            m = mn;
          }
          const float nm = -m;
          sum0 = 0.f;
          sum1 = 0.f;
#pragma unroll
          for (int c = 0; c < kPT; c += 2) {
            float x0, x1;
            ffma2(x0, x1, s[c], s[c + 1], sc, sc, nm, nm);
            const float p0 = fast_exp2(x0), p1 = fast_exp2(x1);
            fadd2(sum0, sum1, sum0, sum1, p0, p1);
            pk[c / 2] = pack_bf16(p0, p1);
          }
          if (fresh || !__any_sync(0xffffffffu, !(sum0 + sum1 <= 256.f))) break;
          fresh = true;
        }
        __syncwarp();
        tmem_st64(t_s, pk);
        l = l * alpha + (sum0 + sum1);
        if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            float v[32];
            tmem_ld32(t_o + c * 32, v);
#pragma unroll
            for (int e = 0; e < 32; ++e) v[e] *= alpha;
            tmem_st32(t_o + c * 32, v);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.p_full[g]);
      }
      if (!ok) break;
      ok = __all_sync(0xffffffffu, wait_or_abort(&sm.o_final[g], rd & 1, err));
      if (!ok) break;
      tc_fence_after();
      // The O row leaves tensor memory here, before this warp signals the
      // next item's first P (whose P.V overwrites O).
      float o[kPT];
      tmem_ld128(t_o, o);
      const float inv_l = l > 0.f ? 1.f / l : 0.f;
      // Output through this warp's 4 KB slice, a quarter of the columns at a
      // time: each lane writes 32 floats of its row (16-byte chunk c at
      // c ^ (row % 8), the 128-byte swizzle), then one lane hands the 32 x 32
      // box to the tensor-store engine.  The slice is rewritten only after the
      // previous store has read it.
      const int x0 = (2 * it.pair + g) * kHeadDim;
      const int y0 = it.seq * p.S + it.i * kPT + (warp & 3) * 32;
#pragma unroll
      for (int qc = 0; qc < 4; ++qc) {
        if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
        __syncwarp();
#pragma unroll
        for (int c = 0; c < 8; ++c)
          *reinterpret_cast<float4*>(slice + lane * 32 + ((c ^ (lane & 7)) << 2)) =
              make_float4(o[32 * qc + 4 * c] * inv_l, o[32 * qc + 4 * c + 1] * inv_l,
                          o[32 * qc + 4 * c + 2] * inv_l, o[32 * qc + 4 * c + 3] * inv_l);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          asm volatile(
              "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];"
              ::"l"(reinterpret_cast<uint64_t>(&p.out_map)), "r"(x0 + 32 * qc), "r"(y0),
                "r"(smem_addr(slice)) : "memory");
          asm volatile("cp.async.bulk.commit_group;" ::: "memory");
        }
      }
    }
    // The CTA's shared memory must outlive the stores that read it.
    if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    __syncwarp();
    if (!ok) atomicOr(&sm.err, 1);
  }

  // ---- teardown: the MMA warp drained its MMAs; free TMEM ----
  tc_fence_before();
  __syncthreads();
  if (tid == 0) {
    if (sm.err) atomicOr(p.status, kStatusWaitTimeout);
    // The last CTA out returns the item counter to zero for the next launch
    // (every loader has taken its last number before its CTA gets here).
    __threadfence();
    if (atomicAdd(p.sched + 1, 1) == (int)gridDim.x - 1) {
      atomicExch(p.sched, 0);
      atomicExch(p.sched + 1, 0);
    }
  }
  if (warp == 9) {
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

// cuTensorMapEncodeTiled from the driver, looked up once through the runtime.
static PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      f = nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  }();
  return fn;
}

cudaError_t launch_prefill_rope_table(const float* inv_freq, float2* cs, int n_pos,
                                      cudaStream_t st) {
  const int n = n_pos * kHalf;
  prefill_rope_table_kernel<<<(n + 255) / 256, 256, 0, st>>>(inv_freq, cs, n_pos);
  return cudaGetLastError();
}

cudaError_t launch_prefill(const float* qkv, long long seq_stride, int n_seq, int S, int n_q,
                           int n_kv, const float2* rope_cs, __nv_bfloat16* qimg,
                           __nv_bfloat16* kimg, __nv_bfloat16* vimg, float* const* k_caches,
                           float* const* v_caches, int t_max, float* out, int* status,
                           int* sched, int n_sm, cudaStream_t st) {
  PrefillPrepParams pp{};
  pp.qkv = qkv;
  pp.seq_stride = seq_stride;
  pp.S = S;
  pp.n_q = n_q;
  pp.n_kv = n_kv;
  pp.rope_cs = rope_cs;
  pp.qimg = qimg;
  pp.kimg = kimg;
  pp.vimg = vimg;
  pp.k_caches = k_caches;
  pp.v_caches = v_caches;
  pp.t_max = t_max;
  prefill_prep_kernel<<<dim3(n_q + 2 * n_kv, S / kPT, n_seq), 256, 0, st>>>(pp);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  PrefillAttnParams ap{};
  PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
  if (!encode) return cudaErrorNotSupported;
  const cuuint64_t dims[2] = {(cuuint64_t)n_q * kHeadDim, (cuuint64_t)n_seq * S};
  const cuuint64_t strides[1] = {(cuuint64_t)n_q * kHeadDim * sizeof(float)};
  const cuuint32_t box[2] = {32, 32};
  const cuuint32_t estr[2] = {1, 1};
  if (encode(&ap.out_map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, out, dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return cudaErrorInvalidValue;
  ap.qimg = qimg;
  ap.kimg = kimg;
  ap.vimg = vimg;
  ap.out = out;
  ap.S = S;
  ap.n_q = n_q;
  ap.n_kv = n_kv;
  ap.n_seq = n_seq;
  ap.scale_log2 = (1.0f / sqrtf((float)kHeadDim)) * 1.4426950408889634f;
  ap.status = status;
  ap.sched = sched;
  const long long n_items = (long long)(S / kPT) * (n_q / 2) * n_seq;
  const int grid = (int)(n_items < n_sm ? n_items : n_sm);
  // Programmatic dependent launch on the prep kernel: the CTAs start as the
  // prep grid drains and set themselves up before their dependency wait.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kPrefillThreads);
  cfg.dynamicSmemBytes = prefill_smem_bytes();
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, prefill_attn_kernel, ap);
}

}  // namespace gqa
