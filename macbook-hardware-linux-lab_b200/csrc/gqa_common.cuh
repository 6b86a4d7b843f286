// Shared definitions for the sm_100a GQA attention kernels.
//
// Shapes follow the reference's Qwen2.5-1.5B attention (compute/attention-gqa-
// resident/attention_gqa_benchmark.c:15-22): head_dim 128, 6 query heads per KV
// head, KV cache laid out [n_kv][t_max][128] fp32 per layer per sequence
// (kernel_attention_gqa.cl:153-154, qwen_server.c:314-317).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace gqa {

constexpr int kHeadDim = 128;
constexpr int kHalf = kHeadDim / 2;
constexpr int kRowBytes = kHeadDim * 4;  // one fp32 K or V row

// Device status bits, OR-ed into the context's status word by kernels that
// detect a problem they cannot report through a return value.
enum : int {
  kStatusBadLength = 1 << 0,    // a device-side pos / seq_len was out of range
  kStatusWaitTimeout = 1 << 1,  // an mbarrier wait ran out of its budget
  kStatusBadSplit = 1 << 2,     // split bookkeeping inconsistent
  kStatusBadToken = 1 << 3,     // a device-side token id was outside the vocabulary
};

// ---------------------------------------------------------------------------
// PTX helpers (mbarrier, bulk async copy, programmatic dependent launch)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
}

// Makes mbarrier initialisation visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: gives up after ~`budget` SM clock cycles and returns false.
// Every wait in these kernels is bounded so that a lost transfer can never
// hang the GPU; the caller records kStatusWaitTimeout and drains.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  long long budget) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long start = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - start > budget) return false;
  }
  return true;
}

// Global -> shared bulk copy (no tensor map, no multicast) completing on `bar`.
// Both addresses must be 16-byte aligned and `bytes` a multiple of 16.
__device__ __forceinline__ void bulk_copy_g2s(void* dst, const void* src, uint32_t bytes,
                                              uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// Programmatic dependent launch.  `wait` blocks until the preceding grid in
// the stream has completed and its memory is visible; it is a no-op when the
// kernel was launched without the programmatic-serialization attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Thread-block cluster helpers (distributed shared memory reads only).
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;"
               ::: "memory");
}
// Address of `p` (this CTA's shared memory) in the shared memory of cluster CTA `rank`.
__device__ __forceinline__ uint32_t cluster_map(const void* p, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(smem_addr(p)), "r"(rank));
  return out;
}
__device__ __forceinline__ float ld_cluster_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Asks the memory system to bring [p, p + bytes) into L2 (no shared memory, no
// completion to wait for).  p 16-byte aligned, bytes a multiple of 16.  L2 is
// the point of coherence, so a line brought in early still sees later writes.
__device__ __forceinline__ void bulk_prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// One 64-bit word {float bits (low half), tag (high half)}, stored and loaded
// whole: a scalar 64-bit access is single-copy atomic, so a reader that sees
// the tag of a store also sees its value.  No fence is implied.
__device__ __forceinline__ void st_tagged(unsigned long long* p, float v, unsigned tag) {
  const unsigned long long w = ((unsigned long long)tag << 32) | __float_as_uint(v);
  asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
// Two consecutive tagged words by one vector load (16-byte aligned); each
// element is its own single-copy-atomic 64-bit access.
__device__ __forceinline__ void ld_tagged2(const unsigned long long* p, unsigned long long& w0,
                                           unsigned long long& w1) {
  asm volatile("ld.relaxed.gpu.global.v2.b64 {%0, %1}, [%2];" : "=l"(w0), "=l"(w1) : "l"(p)
               : "memory");
}
__device__ __forceinline__ unsigned long long ld_tagged(const unsigned long long* p) {
  unsigned long long w;
  asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
  return w;
}
// The same at system scope, for words another GPU stores or polls over NVLink.
__device__ __forceinline__ void st_tagged_sys(unsigned long long* p, float v, unsigned tag) {
  const unsigned long long w = ((unsigned long long)tag << 32) | __float_as_uint(v);
  asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ unsigned long long ld_tagged_sys(const unsigned long long* p) {
  unsigned long long w;
  asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
  return w;
}
__device__ __forceinline__ unsigned tag_of(unsigned long long w) { return (unsigned)(w >> 32); }
__device__ __forceinline__ float value_of(unsigned long long w) {
  return __uint_as_float((unsigned)w);
}

__device__ __forceinline__ void st_relaxed_gpu(unsigned* p, unsigned v) {
  asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_relaxed_gpu_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// ---------------------------------------------------------------------------
// Kernel parameter blocks
// ---------------------------------------------------------------------------

// Where the token count of each sequence comes from.
//   pos_dev != nullptr : pos = *pos_dev, seq_len = pos + 1 (one sequence;
//                        used by graph replays that advance pos on device)
//   seq_lens != nullptr: seq_len = seq_lens[s], pos = seq_len - 1
//   otherwise          : pos = pos_imm, seq_len = seqlen_imm
struct Lengths {
  const int* pos_dev;
  const int* seq_lens;
  int pos_imm;
  int seqlen_imm;
};

// Grid-merged partials: per (q head, split) one row of kGridRowWords tagged
// words, o[0..127] then m and l; 144 words (1152 bytes, 9 x 128) keep every
// 16-dim slice of a row inside one 128-byte line.
constexpr int kGridRowWords = 144;
constexpr int kGridMaxParts = 128;   // splits per KV head in a grid-merged launch
constexpr int kGridEpochWords = 64;  // per-KV-head epochs of one context (n_kv <= 64)
// Cross-GPU slice exchange of a grid-merged KV-range shard: per (parity, source GPU, q head,
// 16-dim slice) one slot of kXSlotWords tagged words: M, L, O[16] (padded to 256 bytes).
constexpr int kXSlotWords = 32;
constexpr int kXSlices = 8;          // 16-dim slices per q head
constexpr int kXMaxWorld = 16;

struct DecodeParams {
  // KV caches.  Per sequence s the cache is k_ptrs[s] (device array of
  // pointers) or, when k_ptrs is null, k_base + s * seq_stride.
  float* const* k_ptrs;
  float* const* v_ptrs;
  float* k_base;
  float* v_base;
  long long seq_stride;  // floats between consecutive sequences' caches
  int t_max;             // cache rows per KV head (row stride t_max * 128)
  int n_kv;              // KV heads

  // Inputs.  For sequence s, q = qkv + s*qkv_stride holds n_kv*G heads of
  // 128 floats; in the fused mode k and v of the new token follow q.
  const float* qkv;
  long long qkv_stride;

  Lengths len;
  // 1 when the lengths (and cache rows below pos) are not written by the
  // kernel launched immediately before this one, so the fused kernel may read
  // them and start streaming the cache before its dependency wait.
  int lengths_stable;
  // KV-range shards: with rope_override set, the angle of the new token's
  // RoPE is taken at rope_pos (its global position) while `pos` is the row
  // index in this shard's cache; skip_append makes the fused kernel neither
  // write nor substitute the new row (the shard does not hold it).  All zero
  // (the default of a zero-initialised block) keeps the plain behaviour.
  int rope_override;
  int rope_pos;
  int skip_append;
  int t_begin;   // first cache row attended (0 except for KV-range shards)
  int t_end;     // if > 0: attend rows [t_begin, t_end) instead of [t_begin, seq_len)

  int n_splits;   // grid.x
  int min_chunk;  // tokens; every split covers a multiple of `quant` tokens
  int quant;      // set by the launcher from the kernel shape

  const float* inv_freq;  // [64] RoPE inverse frequencies
  float q_scale;          // softmax scale * log2(e), folded into q

  // Split outputs: part_o [n_seq][n_q][n_splits][128] (un-normalised),
  // part_ml [n_seq][n_q][n_splits][2] = (m in natural-log units, l).
  float* part_o;
  float* part_ml;

  // Final output when n_splits == 1 (normalised), row stride per sequence.
  float* out;
  long long out_stride;

  int* status;

  // Cluster reduction (single-sequence launches only).  When cluster > 1 the
  // grid is launched in clusters of `cluster` CTAs along the split axis; the
  // clusters reduce through distributed shared memory, write one partial
  // per cluster to part_o/part_ml, and the last CTA of each (sequence, KV
  // head) -- found with counters[seq * n_kv + hkv], which must start at zero
  // and is left at zero -- merges them into `out`.
  int cluster;
  int* counters;

  // Grid merge (single-sequence launches, the GRID instance).  Every CTA
  // stores its partial as tagged words (value, epoch) in grid_words
  // [q head][split][kGridRowWords]; each CTA then merges a slice of the
  // outputs, polling (bounded) the words it needs until they carry this
  // launch's epoch, so the launch leaves the final output with no barrier,
  // fence or combine launch.  The epoch of KV head h is grid_epoch[h] + 1,
  // read after the dependency wait; a merging CTA stores it back once it has
  // seen every split of its KV head, i.e. once every CTA of that KV head has
  // read the old value.  Both buffers start at zero and are used by no other
  // path, so a stale word never carries a current epoch.  The launcher makes
  // sure every CTA of the grid can be resident at once (mergers wait on the
  // others).
  unsigned* grid_epoch;
  unsigned long long* grid_words;
  // With allow_empty set, a launch that attends no row (seq_len 0) is not an
  // error: every CTA publishes an empty partial (a KV-range shard wholly after
  // the position still takes part in the exchange).
  int allow_empty;
  // Cross-GPU exchange of a KV-range-split sequence (grid-merged launches
  // only; null x_inbox: none).  Each merging CTA stores its slice's merged
  // (M, L, O[16]) as tagged words, at system scope, into slot
  // [parity][x_rank][head][slice] of every GPU's inbox (x_inbox[r]), polls its
  // own inbox for the x_world sources' words of the step and writes the
  // output.  The step epoch of (head, slice) is x_epoch[head * 8 + slice] + 1,
  // stored back by its merging CTA; slots alternate by epoch parity.  A GPU
  // cannot run two steps ahead of a peer: its step e + 1 waits for the peer's
  // step-e + 1 words, which the peer stores only after its step-e launch (and
  // every read of the slots it reuses) has finished.
  unsigned long long* const* x_inbox;
  unsigned* x_epoch;
  int x_rank, x_world;
};

struct CombineParams {
  const float* m;  // m[p * ml_part_stride + r * ml_row_stride]
  const float* l;
  const float* o;  // o[p * o_part_stride + r * o_row_stride + d]
  long long ml_part_stride, ml_row_stride;
  long long o_part_stride, o_row_stride;
  int n_parts;
  int rows_per_seq;  // q heads per sequence
  // Output: row r = (seq, h) -> out + seq*out_stride + h*128.
  float* out;
  long long out_stride;
  // When out_m/out_l are set, the combined triple (M, L, un-normalised O) is
  // written instead of O / L (a partial over the union of the parts).
  float* out_m;
  float* out_l;
  // When set, the combine advances every sequence's length by one once the
  // split kernel before it (which read them) has finished: advance_lens[seq]++.
  int* advance_lens;
};

}  // namespace gqa
