/*
 * gqa.h -- C ABI of the B200 (sm_100a) grouped-query-attention decode path.
 *
 * Drop-in for the attention slice of the reference's resident Qwen2.5 decoder
 * (fbetancourt-dev/macbook-hardware-linux-lab).  Plain C types only: device
 * pointers are `float*`, streams are an opaque `void*` (a cudaStream_t; NULL is
 * the legacy default stream).  Every call returns a gqa_status; nothing calls
 * exit().  Calls are stream-ordered and asynchronous unless stated otherwise.
 * One context per device; a context is not thread-safe (use one per thread or
 * serialise), matching the reference's single in-order queue.  A context owns
 * one split-KV scratch area, so its calls must not run concurrently on
 * different streams; captured graphs keep using it (the context must outlive
 * its graphs, and the scratch cannot grow while a graph exists).
 *
 * Shapes: head_dim 128, n_heads_q = 6 * n_heads_kv (Qwen2.5-1.5B: 12 / 2).
 * KV cache per layer per sequence: [n_heads_kv][t_max][128] fp32, K stored
 * after RoPE, exactly the reference's LayerKVDevice layout.
 * qkv per token: [q (n_heads_q*128) | k (n_heads_kv*128) | v (n_heads_kv*128)].
 */
#ifndef GQA_B200_H
#define GQA_B200_H

#if defined(__GNUC__)
#define GQA_API __attribute__((visibility("default")))
#else
#define GQA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef struct gqa_ctx gqa_ctx;
typedef struct gqa_graph gqa_graph;
typedef void *gqa_stream_t;

typedef enum {
    GQA_OK = 0,
    GQA_ERR_INVALID_ARG = -1,  /* bad size, pointer, alignment or shape */
    GQA_ERR_CUDA = -2,         /* a CUDA runtime call failed (see gqa_last_error_string) */
    GQA_ERR_UNSUPPORTED = -3,  /* shape/config not built (e.g. head_dim != 128) */
    GQA_ERR_DEVICE = -4,       /* a kernel flagged a problem (gqa_device_status) */
    GQA_ERR_NO_MEMORY = -5,    /* allocation failed or not allowed while capturing */
    GQA_ERR_TIMEOUT = -6       /* a bounded device wait gave up */
} gqa_status;

/* Model shape.  Replaces the reference's compile-time #defines
 * (qwen_server.c:20-32: HEAD_DIM, N_HEADS_Q, N_HEADS_KV, T_MAX, ROPE_BASE). */
typedef struct {
    int n_heads_q;     /* 12 */
    int n_heads_kv;    /* 2 */
    int head_dim;      /* 128 with 6 q heads per KV head; or 64 with 7 (Qwen2.5-0.5B) */
    int t_max;         /* cache rows per KV head (reference: 4096) */
    float rope_theta;  /* 1e6 */
} gqa_config;

/* One layer's resident KV cache: the reference's LayerKVDevice
 * {k_cache, v_cache} (qwen_server.c:314-317), device pointers. */
typedef struct {
    float *k_cache;
    float *v_cache;
} gqa_layer_kv;

/* ---- context ---------------------------------------------------------- */

/* Creates a context on `device` (makes it current).  Replaces the OpenCL
 * context/queue/program set-up of qwen_server.c:560-640.  Two shapes are
 * built: head_dim 128 with 6 q heads per KV head (Qwen2.5-1.5B, every entry
 * point) and head_dim 64 with 7 (Qwen2.5-0.5B, generate_stream_05b.c:19-31:
 * gqa_kv_alloc/free, gqa_reserve, gqa_layer_attention(_out),
 * gqa_decode_layers and the layer graphs, on shape-generic kernels; the other
 * entry points return GQA_ERR_UNSUPPORTED for it). */
GQA_API int gqa_create(const gqa_config *cfg, int device, gqa_ctx **out);
GQA_API int gqa_destroy(gqa_ctx *ctx);

/* Human-readable text of the last error on the calling thread. */
GQA_API const char *gqa_last_error_string(void);

/* Options.  GQA_OPT_PDL: 1 lets the library's own launches overlap their
 * start with the previous kernel in the stream (programmatic dependent
 * launch); KV rows below pos are then streamed before the previous kernel
 * finishes, so the caller must not write those rows in the kernel launched
 * immediately before.  Default 0 for single calls; the multi-layer step and
 * graph APIs always use it between their own launches.
 * GQA_OPT_TARGET_CTAS: CTAs one single-sequence decode aims for (default:
 * the device's SM count).
 * GQA_OPT_BATCH_ADVANCE: 1 makes gqa_decode_batched(_host) add one to every
 * seq_lens[s] on the device after the step has used them (the serving
 * loop's own advance to the next token, done by the step's last kernel
 * instead of a separate launch); seq_lens is then written.  Default 0. */
enum { GQA_OPT_PDL = 1, GQA_OPT_TARGET_CTAS = 2, GQA_OPT_BATCH_ADVANCE = 8 };
GQA_API int gqa_set_option(gqa_ctx *ctx, int option, long long value);

/* Pre-sizes the split-KV scratch for up to n_seq sequences of up to max_len
 * tokens (call before stream capture; launches otherwise grow it on demand,
 * which is refused while a capture is in progress). */
GQA_API int gqa_reserve(gqa_ctx *ctx, int n_seq, int max_len);

/* Reads and optionally clears the device status word (bitmask; 0 = fine).
 * Synchronises the context's device. */
GQA_API int gqa_device_status(gqa_ctx *ctx, int *status, int clear);

/* ---- KV cache --------------------------------------------------------- */

/* Allocates n_layers zero-filled caches of [n_heads_kv][t_max][128] fp32.
 * Replaces qwen_server.c:646-647 (clCreateBuffer) and :671-676 (zero fill). */
GQA_API int gqa_kv_alloc(gqa_ctx *ctx, int n_layers, gqa_layer_kv *out);
GQA_API int gqa_kv_free(gqa_ctx *ctx, int n_layers, gqa_layer_kv *kv);

/* ---- the layer call (the drop-in boundary) ---------------------------- */

/* Attention slice of gpu_decoder_layer_step() (qwen_server.c:344-455, launches
 * :446-450): RoPE (theta from cfg, half rotation) on q and k of the new token,
 * append rotated k and raw v at row pos, attention of every q head over cache
 * rows [0, seq_len), and the result written to qkv[0 : n_heads_q*128] as the
 * reference's segment reduce does (qwen_server.c:402-404).  qkv[n_heads_q*128:]
 * is left unchanged.  0 <= pos < t_max, 1 <= seq_len <= t_max (callers pass
 * seq_len = pos + 1).  qkv and the caches must be 16-byte aligned. */
GQA_API int gqa_layer_attention(gqa_ctx *ctx, gqa_stream_t stream, const gqa_layer_kv *kv, float *qkv,
                        int pos, int seq_len);

/* Same as gqa_layer_attention, result to a separate buffer out[n_heads_q*128]
 * (qkv is then left unchanged). */
GQA_API int gqa_layer_attention_out(gqa_ctx *ctx, gqa_stream_t stream, const gqa_layer_kv *kv,
                            const float *qkv, int pos, int seq_len, float *out);

/* The caller's per-token loop over layers (qwen_server.c:1021-1023,
 * generate_stream.c:747-749): for each layer l, gqa_layer_attention_out on
 * kv[l] with qkv + l*qkv_layer_stride -> out + l*out_layer_stride.  pos is read
 * from device memory (*d_pos, seq_len = pos + 1); if advance is non-zero, *d_pos
 * is incremented on the device after the last layer, wrapping to wrap_lo when
 * it reaches wrap_hi (wrap_hi <= wrap_lo disables wrapping). */
GQA_API int gqa_decode_layers(gqa_ctx *ctx, gqa_stream_t stream, int n_layers, const gqa_layer_kv *kv,
                      const float *qkv, long long qkv_layer_stride, float *out,
                      long long out_layer_stride, int *d_pos, int advance, int wrap_lo,
                      int wrap_hi);

/* gqa_decode_layers captured once into a CUDA graph and replayed by
 * gqa_graph_launch (one launch = one decode step over all layers).  The
 * pointers are baked into the graph. */
GQA_API int gqa_graph_create_layers(gqa_ctx *ctx, int n_layers, const gqa_layer_kv *kv,
                            const float *qkv, long long qkv_layer_stride, float *out,
                            long long out_layer_stride, int *d_pos, int advance, int wrap_lo,
                            int wrap_hi, gqa_graph **out_graph);
GQA_API int gqa_graph_launch(gqa_graph *g, gqa_stream_t stream);
GQA_API int gqa_graph_destroy(gqa_graph *g);

/* One decode step with HOST buffers (the reference's write -> kernels ->
 * read loop, attention_gqa_benchmark.c:531-545): copies h_qkv
 * [n_layers][qkv_layer_stride] to d_qkv, replays g, copies d_out
 * [n_layers][out_layer_stride] back to h_out.  Asynchronous on `stream`;
 * pass page-locked host memory for the copies to overlap. */
GQA_API int gqa_graph_step_host(gqa_graph *g, gqa_stream_t stream, const float *h_qkv, float *h_out);

/* ---- kernel-level operations ------------------------------------------ */

/* kernel_rope_and_kv_append (kernel_attention_gqa.cl:149-194): q[n_heads_q*128]
 * rotated in place; k, v [n_heads_kv*128]; rotated k and v written to row pos.
 * q, k, v must be the three consecutive slices of one qkv row, as the
 * reference's sub-buffers are (qwen_server.c:664-669). */
GQA_API int gqa_rope_kv_append(gqa_ctx *ctx, gqa_stream_t stream, const gqa_layer_kv *kv, float *q,
                       const float *k, const float *v, int pos);

/* Fused replacement of kernel_gqa_scores + kernel_softmax_gqa +
 * kernel_gqa_value_combine_segmented + kernel_gqa_reduce_segments
 * (kernel_attention_gqa.cl:202-397): attention of already-rotated q over
 * cache rows [0, seq_len) -> out[n_heads_q*128]. */
GQA_API int gqa_decode(gqa_ctx *ctx, gqa_stream_t stream, const gqa_layer_kv *kv, const float *q_rot,
               int seq_len, float *out);

/* Batched decode of n_seq independent sequences, one new token each: for
 * sequence s, RoPE + append at pos = seq_lens[s] - 1 into k_caches[s] /
 * v_caches[s], then attention over seq_lens[s] rows.  k_caches, v_caches,
 * seq_lens are DEVICE arrays; qkv + s*qkv_stride is sequence s's qkv;
 * results go to out + s*out_stride (out may equal qkv).  max_len bounds every
 * seq_lens[s] (sizes the split plan). */
GQA_API int gqa_decode_batched(gqa_ctx *ctx, gqa_stream_t stream, int n_seq, float *const *k_caches,
                       float *const *v_caches, const float *qkv, long long qkv_stride,
                       const int *seq_lens, int max_len, float *out, long long out_stride);

/* One batched decode step with HOST buffers (the reference's write ->
 * kernels -> read loop, attention_gqa_benchmark.c:531-545, for a batch):
 * copies h_qkv (n_seq rows of qkv_stride floats) into the device buffer d_qkv,
 * runs gqa_decode_batched on it with the other arguments as there, and copies
 * each sequence's n_heads_q*128 output floats (out_stride apart in d_out) into
 * h_out, packed row after row.  d_out may equal d_qkv.  Asynchronous on
 * `stream`; pass page-locked host memory for the copies to run at full rate. */
GQA_API int gqa_decode_batched_host(gqa_ctx *ctx, gqa_stream_t stream, int n_seq,
                            float *const *k_caches, float *const *v_caches, const float *h_qkv,
                            float *d_qkv, long long qkv_stride, const int *seq_lens, int max_len,
                            float *d_out, long long out_stride, float *h_out);

/* Split-KV partial over cache rows [t_begin, t_end) for already-rotated q:
 * per q head h, a reference value m[h] (natural-log units; scores are
 * q.k / sqrt(128)), l[h] = sum exp(s - m) and o[h][:] = sum exp(s - m) v (not
 * normalised).  m is at most the maximum score and trails it by at most
 * 8 ln 2; (m, l, o) is exact up to that common factor, which a log-sum-exp
 * combine removes.  An empty range yields m = -inf, l = 0, o = 0. */
GQA_API int gqa_decode_split_partial(gqa_ctx *ctx, gqa_stream_t stream, const gqa_layer_kv *kv,
                             const float *q_rot, int t_begin, int t_end, float *m, float *l,
                             float *o);

/* One KV-range shard of a decode step (a long sequence split over GPUs by
 * cache rows).  This shard holds global rows [shard_begin, shard_begin +
 * shard_rows) at local rows [0, shard_rows) of kv.  qkv is the new token's
 * row (q|k|v before RoPE, the same on every shard) at global position pos.
 * q is rotated for pos; if pos falls in this shard, its rotated k and raw v
 * are written at local row pos - shard_begin.  Output: the partial (m, l, o)
 * of gqa_decode_split_partial over the shard's rows up to pos (m = -inf,
 * l = 0, o = 0 if none), ready for gqa_lse_combine across shards.  The
 * reference has no multi-GPU path; this replaces its single-queue split-K
 * segments (kernel_attention_gqa.cl:340-397) at the scale of several GPUs. */
GQA_API int gqa_decode_kv_shard(gqa_ctx *ctx, gqa_stream_t stream, const gqa_layer_kv *kv,
                                const float *qkv, int pos, int shard_begin, int shard_rows,
                                float *m, float *l, float *o);

/* Log-sum-exp combine of n_parts partials for n_rows rows (q heads):
 * m, l: [n_parts][n_rows]; o: [n_parts][n_rows][128]; out: [n_rows][128] =
 * sum_p e^(m_p - M) o_p / sum_p e^(m_p - M) l_p, M = max_p m_p.  Parts with
 * l = 0 are ignored. */
GQA_API int gqa_lse_combine(gqa_ctx *ctx, gqa_stream_t stream, int n_parts, int n_rows, const float *m,
                    const float *l, const float *o, float *out);

/* gqa_lse_combine for partials packed one part after another, each part
 * [m (n_rows) | l (n_rows) | o (n_rows*128)] at part_stride floats from the
 * previous: the layout of gqa_decode_kv_shard outputs written to
 * (buf, buf + n_rows, buf + 2*n_rows) and all-gathered across GPUs. */
GQA_API int gqa_lse_combine_packed(gqa_ctx *ctx, gqa_stream_t stream, int n_parts, int n_rows,
                                   const float *packed, long long part_stride, float *out);

/* ---- KV-range split over several GPUs, merged through peer memory ------ */

/* One GPU's member of a group of `world` GPUs (one process or thread each)
 * that decode one sequence with its cache rows split in contiguous ranges.
 * gqa_exchange_create allocates this GPU's inbox and writes its CUDA IPC
 * handle (GQA_IPC_HANDLE_BYTES bytes) to ipc_handle; the caller gathers every
 * rank's handle (in rank order) and passes the array to gqa_exchange_open,
 * which maps the peers' inboxes (a handle equal to the caller's own maps to
 * its own inbox).  The reference runs on one GPU and has no
 * counterpart; the merge it extends is its split-K segment reduce
 * (kernel_attention_gqa.cl:378-397). */
#define GQA_IPC_HANDLE_BYTES 64
typedef struct gqa_exchange gqa_exchange;
GQA_API int gqa_exchange_create(gqa_ctx *ctx, int rank, int world, gqa_exchange **out,
                                void *ipc_handle);
GQA_API int gqa_exchange_open(gqa_exchange *x, const void *handles);
GQA_API int gqa_exchange_destroy(gqa_exchange *x);

/* gqa_decode_kv_shard followed by the cross-GPU merge in one kernel: every
 * rank of the group calls it for the same step (same qkv row and pos) with
 * its own range; each writes its merged (m, l, o) per q head into every
 * rank's inbox over NVLink, waits (bounded, ~1 s) for the others', and
 * writes the complete attention output [n_heads_q][128] to out.  All ranks
 * must make the same sequence of calls; a peer that does not arrive sets the
 * wait-timeout bit (2) of the device status word (gqa_device_status) and
 * leaves out unwritten, and the group must then be destroyed. */
GQA_API int gqa_decode_kv_shard_exchange(gqa_ctx *ctx, gqa_exchange *x, gqa_stream_t stream,
                                         const gqa_layer_kv *kv, const float *qkv, int pos,
                                         int shard_begin, int shard_rows, float *out);

/* ---- the attention half of the decoder layer ---------------------------- */

/* Q4_0 blocks as in the reference (block_q4_0, attention_gqa_benchmark.c:
 * 26-29): 32 weights in 18 bytes, an IEEE fp16 scale d then 16 bytes of
 * 4-bit codes; weight j < 16 = d * ((qs[j] & 15) - 8), weight j + 16 =
 * d * ((qs[j] >> 4) - 8).  A matrix is row-major: rows one after another,
 * each row d_model / 32 blocks. */
#define GQA_Q4_0_BLOCK_BYTES 18

/* The decoder sizes the projections are built for, by the context's shape:
 *   Qwen2.5-1.5B  head_dim 128, 12 q / 2 KV heads: d_model 1536, d_ffn 8960
 *                 (qwen_server.c);
 *   Qwen2.5-0.5B  head_dim 64, 14 q / 2 KV heads:  d_model 896,  d_ffn 4864
 *                 (generate_stream_05b.c:19-26).
 * The block, FFN, embedding and token-step calls report GQA_ERR_UNSUPPORTED
 * for any other shape. */

/* Device pointers of one layer's attention weights (16-byte aligned). */
typedef struct {
    const void *w_qkv;   /* Q4_0 [(n_heads_q + 2 n_heads_kv) * head_dim][d_model / 32] */
    const float *b_qkv;  /* [(n_heads_q + 2 n_heads_kv) * head_dim] */
    const void *w_o;     /* Q4_0 [d_model][d_model / 32] */
    const float *gamma;  /* [d_model] weight of the attention RMSNorm */
} gqa_block_weights;

/* state += W_o * attention(RoPE(W_qkv * rmsnorm(state, gamma) + b_qkv)):
 * the attention half of gpu_decoder_layer_step (qwen_server.c:444-453:
 * k_rmsnorm_attn, k_qkv_gemv, the five attention kernels, k_wo_residual),
 * with the KV append at pos as in gqa_layer_attention.  d_model =
 * n_heads_q * head_dim (1536 or 896, above); the RMSNorm epsilon is the
 * reference's 1e-6 (the 0.5B generator's gpu_decoder_layer_step,
 * generate_stream_05b.c:364-476, is the same chain at its sizes).
 * state: [d_model] device floats, updated in place. */
GQA_API int gqa_attention_block(gqa_ctx *ctx, gqa_stream_t stream, const gqa_block_weights *w,
                                const gqa_layer_kv *kv, float *state, int pos, int seq_len);

/* gqa_attention_block for n_layers layers in a row (one state, the token's
 * position read from device memory d_pos, seq_len = *d_pos + 1), the token
 * loop of qwen_server.c:1021-1023 without the FFN half; with advance != 0 the
 * position is incremented on the device afterwards (wrapping to wrap_lo at
 * wrap_hi when wrap_hi > 0).  Capturable in a CUDA graph. */
GQA_API int gqa_attention_block_layers(gqa_ctx *ctx, gqa_stream_t stream, int n_layers,
                                       const gqa_block_weights *w, const gqa_layer_kv *kv,
                                       float *state, int *d_pos, int advance, int wrap_lo,
                                       int wrap_hi);

/* Device pointers of one layer's FFN weights (16-byte aligned). */
typedef struct {
    const void *w_gate;  /* Q4_0 [d_ffn][d_model / 32] */
    const void *w_up;    /* Q4_0 [d_ffn][d_model / 32] */
    const void *w_down;  /* Q4_0 [d_model][d_ffn / 32] */
    const float *gamma;  /* [d_model] weight of the FFN RMSNorm */
} gqa_ffn_weights;

/* state += W_down * (silu(W_gate * z) * (W_up * z)), z = rmsnorm(state, gamma):
 * the FFN half of gpu_decoder_layer_step (qwen_server.c k_rmsnorm_ffn,
 * k_swiglu_fused, k_down_res; CPU test_28_layers_real.c:298-317), with the
 * reference's stable SiLU.  d_model / d_ffn: 1536 / 8960 or 896 / 4864. */
GQA_API int gqa_ffn_block(gqa_ctx *ctx, gqa_stream_t stream, const gqa_ffn_weights *w,
                          float *state);

/* The whole decoder layer (attention block, then FFN block) for n_layers
 * layers of one token, position on the device as in
 * gqa_attention_block_layers: the reference's per-token loop over
 * gpu_decoder_layer_step (qwen_server.c:1021-1023).  Capturable. */
GQA_API int gqa_decoder_layers(gqa_ctx *ctx, gqa_stream_t stream, int n_layers,
                               const gqa_block_weights *attn, const gqa_ffn_weights *ffn,
                               const gqa_layer_kv *kv, float *state, int *d_pos, int advance,
                               int wrap_lo, int wrap_hi);

/* ---- token embedding, LM head and the whole decode step --------------- */

#define GQA_Q6_K_BLOCK_BYTES 210  /* block_q6_K: 256 weights */

/* Bytes that gqa_lm_head_pack writes for n_rows rows of 1536 inputs: the
 * size of the GGUF tensor itself with the rows rounded up to a multiple of 4,
 * 1260 * ((n_rows + 3) / 4 * 4) (for the 151936-row head exactly its size). */
GQA_API long long gqa_lm_head_packed_bytes(int n_rows);

/* Lays a Q6_K matrix out for gqa_lm_head.  q6k: device, n_rows rows of
 * 1536 / 256 superblocks of 210 bytes (block_q6_K, test_gemv_q6_k.c:21-26),
 * the bytes of the GGUF tensor output.weight that qwen_server.c uploads whole
 * (:586-588, d_W_head); packed: device, 16-byte aligned,
 * gqa_lm_head_packed_bytes(n_rows).  The same bytes in four planes (ql, qh,
 * scales, d) whose rows are aligned, padding rows zero; run once when the
 * weights are loaded. */
GQA_API int gqa_lm_head_pack(gqa_ctx *ctx, gqa_stream_t stream, const void *q6k, int n_rows,
                             void *packed);

/* logits[r] = sum_j W[r][j] * z[j] with z = rmsnorm(state) * gamma (epsilon
 * 1e-6): k_output_norm and the gemv_q6_k LM head of qwen_server.c:1025-1044
 * (CPU: test_full_model_logits.c:944-958).  When token is given, *token
 * (device int) receives the greedy pick of the host loop at
 * qwen_server.c:998-1005: the first row whose logit is the largest one above
 * -1e30 (NaN never wins), 0 if there is none.  logits may be NULL when only
 * the pick is wanted; at least one of logits and token must be given.  A
 * context runs one head at a time (its pick scratch is shared). */
GQA_API int gqa_lm_head(gqa_ctx *ctx, gqa_stream_t stream, const void *packed, int n_rows,
                        const float *gamma, const float *state, float *logits, int *token);

/* state = row *d_token of a Q4_0 embedding table [n_rows][d_model / 32 blocks]
 * (device, the bytes of token_embd.weight): get_token_embedding
 * (qwen_server.c:188-201; generate_stream_05b.c:200-213 with d_model 896)
 * done on the device, so that the token id never
 * leaves it.  An id outside [0, n_rows) sets GQA_STATUS_BAD_TOKEN in the
 * device status word and leaves state unchanged. */
GQA_API int gqa_token_embedding(gqa_ctx *ctx, gqa_stream_t stream, const void *table, int n_rows,
                                const int *d_token, float *state);

/* The Qwen2.5-0.5B head: Q8_0 blocks (block_q8_0, generate_stream_05b.c:
 * 42-45), an IEEE fp16 scale d then 32 int8 codes; weight j = d * qs[j]. */
#define GQA_Q8_0_BLOCK_BYTES 34

/* Bytes that gqa_lm_head_q8_0_pack writes for n_rows rows of 896 inputs:
 * 952 * ((n_rows + 3) / 4 * 4) (for the 151936-row head exactly its size). */
GQA_API long long gqa_lm_head_q8_0_packed_bytes(int n_rows);

/* Lays a Q8_0 matrix out for gqa_lm_head_q8_0.  q8: device, n_rows rows of
 * 28 blocks of 34 bytes (the bytes of output.weight that
 * generate_stream_05b.c uploads whole, :687, d_W_head); packed: device,
 * 16-byte aligned, gqa_lm_head_q8_0_packed_bytes(n_rows).  The same bytes in
 * two planes (codes, scales) whose rows are aligned; run once at load time. */
GQA_API int gqa_lm_head_q8_0_pack(gqa_ctx *ctx, gqa_stream_t stream, const void *q8, int n_rows,
                                  void *packed);

/* gqa_lm_head for the Qwen2.5-0.5B shape (d_model 896): k_output_norm and
 * the gemv_q8_0 LM head (kernel_q8_0.cl:10-61, generate_stream_05b.c:
 * 845-864), logits and/or the greedy pick of the host loop at :872-878
 * (the first row whose logit is the largest one above -1e30). */
GQA_API int gqa_lm_head_q8_0(gqa_ctx *ctx, gqa_stream_t stream, const void *packed, int n_rows,
                             const float *gamma, const float *state, float *logits, int *token);

/* Device status bits (gqa_device_status). */
#define GQA_STATUS_BAD_LENGTH 1   /* a device-side pos / seq_len was out of range */
#define GQA_STATUS_WAIT_TIMEOUT 2 /* a bounded device wait gave up */
#define GQA_STATUS_BAD_TOKEN 8    /* a device-side token id was outside the vocabulary */

/* gqa_model.lm_head_type */
#define GQA_HEAD_Q6_K 0  /* gqa_lm_head_pack layout (Qwen2.5-1.5B, d_model 1536) */
#define GQA_HEAD_Q8_0 1  /* gqa_lm_head_q8_0_pack layout (Qwen2.5-0.5B, d_model 896) */

/* Everything one decode step of the whole model reads (device pointers in
 * host arrays). */
typedef struct {
    int n_layers;
    const gqa_block_weights *attn;  /* [n_layers] */
    const gqa_ffn_weights *ffn;     /* [n_layers] */
    const gqa_layer_kv *kv;         /* [n_layers] */
    const void *token_embd;         /* Q4_0 [vocab][d_model / 32 blocks] */
    const float *gamma_output;      /* [d_model] output_norm.weight */
    const void *lm_head;            /* packed output.weight, layout by lm_head_type */
    int vocab;                      /* rows of token_embd and of the head */
    int lm_head_type;               /* GQA_HEAD_Q6_K or GQA_HEAD_Q8_0 */
} gqa_model;

/* One greedy decode step of the whole model without leaving the device: the
 * token loop of qwen_server.c:1016-1046 -- embedding of *d_token, n_layers
 * decoder layers at position *d_pos, output norm, LM head, greedy pick -- with
 * the pick written back to *d_token and *d_pos advanced (wrapping to wrap_lo
 * at wrap_hi when wrap_hi > 0), so that steps chain on the device and one step
 * can be captured as a graph (the 0.5B generator's loop, generate_stream_05b.c:
 * 823-897, is the same step with the Q8_0 head).  state: [d_model] device
 * workspace; logits: [vocab]
 * device, or NULL.  The end-of-generation check (:1008) and the position
 * limit (:1014) stay with the caller, which reads *d_token. */
GQA_API int gqa_decode_token(gqa_ctx *ctx, gqa_stream_t stream, const gqa_model *model,
                             float *state, int *d_token, int *d_pos, float *logits, int wrap_lo,
                             int wrap_hi);

/* ---- GGUF model files and the server's requests -------------------------- */

/* A GGUF file opened for reading (v2 or v3): the tensor table, the integer
 * metadata, general.alignment and tokenizer.ggml.tokens -- what qwen_server.c
 * gets from parse_gguf_tensors (:113-178) and load_tokenizer_tokens
 * (:203-266).  Unlike the reference, every length is checked against the
 * file size, general.alignment is honoured (the reference assumes 32, the
 * default) and a damaged file is an error, never an exit. */
typedef struct gqa_gguf gqa_gguf;

typedef struct {
    const char *name;            /* owned by the gqa_gguf */
    int n_dims;
    long long ne[4];             /* ne[0] is the innermost dimension */
    int type;                    /* GGUF tensor type: 0 F32, 2 Q4_0, 14 Q6_K, ... */
    unsigned long long offset;   /* absolute file offset of the data */
    unsigned long long bytes;    /* size of the data (0 for a type not sized here) */
} gqa_gguf_tensor;

GQA_API int gqa_gguf_open(const char *path, gqa_gguf **out);
GQA_API int gqa_gguf_close(gqa_gguf *g);
GQA_API int gqa_gguf_tensor_count(const gqa_gguf *g);
GQA_API int gqa_gguf_tensor_at(const gqa_gguf *g, int i, gqa_gguf_tensor *out);
/* get_tensor_offset (:180-186) with an error instead of exit when absent. */
GQA_API int gqa_gguf_find(const gqa_gguf *g, const char *name, gqa_gguf_tensor *out);
/* Reads a tensor's bytes (or any in-file range given as a gqa_gguf_tensor). */
GQA_API int gqa_gguf_read(const gqa_gguf *g, const gqa_gguf_tensor *t, void *host_dst);
GQA_API int gqa_gguf_meta_int(const gqa_gguf *g, const char *key, long long *out);
/* Number of tokenizer.ggml.tokens entries (0 if absent) and one entry's raw
 * string (copied with a terminating NUL; returns its full length). */
GQA_API int gqa_gguf_vocab_size(const gqa_gguf *g);
GQA_API int gqa_gguf_token_string(const gqa_gguf *g, int id, char *out, int cap);

/* Device copies of one model's weights, laid out as the server lays them
 * out (qwen_server.c:525-588): per layer W_qkv = attn_q | attn_k | attn_v rows
 * and b_qkv likewise, attn_output, ffn_gate/up/down and both norm weights;
 * token_embd.weight; output_norm.weight; output.weight through
 * gqa_lm_head_pack.  The sizes come from the context's shape: Qwen2.5-1.5B
 * (Q6_K head) or Qwen2.5-0.5B (Q8_0 head through gqa_lm_head_q8_0_pack, the
 * tensors generate_stream_05b.c:553-615 reads); types and shapes are checked
 * (Q4_0 projections and embedding, the head's type, F32 norms and biases).
 * n_layers <= 0 takes qwen2.block_count from the file.  Allocates on the
 * current device, which must be the context's. */
typedef struct gqa_model_weights gqa_model_weights;
GQA_API int gqa_model_load(gqa_ctx *ctx, const gqa_gguf *g, int n_layers,
                           gqa_model_weights **out);
/* A gqa_model over loaded weights and the caller's KV caches (kv may be NULL
 * for a view without caches). */
GQA_API int gqa_model_view(const gqa_model_weights *w, const gqa_layer_kv *kv, gqa_model *out);
GQA_API int gqa_model_free(gqa_model_weights *w);

/* The server's requests without the socket (qwen_server.c:770-1054): one
 * conversation state over a model whose caches have at least t_max rows.
 * eog_ids / n_eog: the end-of-generation tokens (NULL: the reference's
 * 151643 and 151645).  Errors carry the server's reply text in
 * gqa_last_error_string(): ERR_BAD_REQUEST, ERR_INVALID_TOKEN,
 * ERR_CONTEXT_FULL, ERR_NOT_READY, ERR_RAW_NOT_ALLOWED_WHEN_BASE_ACTIVE,
 * ERR_GPU_FAILURE. */
typedef struct gqa_session gqa_session;
GQA_API int gqa_session_create(gqa_ctx *ctx, const gqa_model *model, int t_max,
                               const int *eog_ids, int n_eog, gqa_session **out);
GQA_API int gqa_session_destroy(gqa_session *s);
/* SET_BASE: the tokens through every layer at positions 0 .. n-1, one token
 * at a time as the server does; then base_pos = n, base_hash = FNV-1a of the
 * ids, base_generation + 1, state READY. */
GQA_API int gqa_session_set_base(gqa_session *s, const int *tokens, int n);
/* QUERY (raw = 0, from base_pos; needs READY) or RAW_QUERY (raw = 1, from
 * position 0; refused while a base is active): the prompt through the layers,
 * the head on its last token, then greedy generation of at most max_new
 * tokens, stopping before an end-of-generation token.  out_tokens receives
 * the generated ids (room for max_new), *n_out their count.  Positions past
 * base_pos are scratch for the next request, as in the server. */
GQA_API int gqa_session_query(gqa_session *s, const int *tokens, int n, int max_new, int raw,
                              int *out_tokens, int *n_out);
/* STATUS: base_pos, base_hash, base_generation and whether the state is
 * READY (any pointer may be NULL). */
GQA_API int gqa_session_status(const gqa_session *s, int *base_pos,
                               unsigned long long *base_hash, int *base_generation,
                               int *ready);

/* ---- prefill ---------------------------------------------------------- */

/* Causal attention over whole prompts on the tensor cores (bf16 operands,
 * fp32 accumulation).  The reference has no prefill: it runs the prompt
 * through the decode layer call one token at a time (qwen_server.c:957-964);
 * this computes the same rows at once.  qkv: [n_seq][seq_len][q|k|v] fp32
 * before RoPE, token s at position s; out: [n_seq][seq_len][n_heads_q*128]
 * fp32.  When k_caches / v_caches (DEVICE arrays of n_seq cache pointers) are
 * given, rows [0, seq_len) of each cache receive the rotated K and raw V in
 * fp32, as the token-by-token path would leave them.  seq_len must be a
 * multiple of 128.  Accuracy: bf16 operands, about 1e-2 of the output RMS. */
GQA_API int gqa_prefill_bf16(gqa_ctx *ctx, gqa_stream_t stream, int n_seq, int seq_len,
                             const float *qkv, float *out, float *const *k_caches,
                             float *const *v_caches);

/* ---- layer call without allocation ------------------------------------ */

/* gqa_layer_attention for callers that cannot allocate device memory when
 * they run (host callbacks, plugins whose framework owns all device memory,
 * allocation-free capture set-ups).  No counterpart in the reference.  It
 * needs no context: it runs on the calling thread's current device, and its
 * split-KV scratch is a static device array inside the library (about
 * 2.03 MiB per device that loads the library, held until exit, room for 4096
 * q-head x split partials; a call needing more is rejected with
 * GQA_ERR_INVALID_ARG).  The first call on a device does a one-time set-up
 * that includes synchronous copies, so make it before any stream capture.  A
 * call whose rope_theta differs from the previous call's writes the new RoPE
 * table with an asynchronous copy on `stream`, ordered like the calls
 * themselves.  Calls share the array: calls on one device that may overlap on
 * the GPU race and must be ordered by the caller (one stream, or events).
 * Errors the kernels detect on the device (a bad length, a wait that ran out)
 * are not in the return value; read them with gqa_static_status.  It calls no
 * cudaMalloc, cudaFree or allocating library routine. */
GQA_API int gqa_layer_attention_static(const gqa_config *cfg, gqa_stream_t stream,
                                       const gqa_layer_kv *kv, float *qkv, int pos,
                                       int seq_len);

/* Device status word of the allocation-free layer calls on `device` (bitmask,
 * 0 = fine; the bits of gqa_device_status); clear != 0 zeroes it.  Waits for
 * all work on that device first.  No counterpart in the reference. */
GQA_API int gqa_static_status(int device, int *status, int clear);

/* ---- utilities -------------------------------------------------------- */

/* Fills dst[0..n) with seeded N(0,1) values (splitmix64 + Box-Muller;
 * element e of stream (seed, stream_id) for e = offset .. offset+n-1). */
GQA_API int gqa_fill_normal(gqa_ctx *ctx, gqa_stream_t stream, float *dst, long long n,
                    unsigned long long seed, unsigned long long stream_id, long long offset);

/* Inverse RoPE frequencies used by the kernels (host copy, head_dim/2
 * floats): powf(theta, -2*i/head_dim) as in attention_gqa_benchmark.c:143. */
GQA_API int gqa_inv_freq(const gqa_ctx *ctx, float *out);

/* Phase trace of the split-KV decode kernel, for profiling (no counterpart in
 * the reference).  Only a library built with -DGQA_PHASE_TRACE records it
 * (build.py --phase-trace writes libgqa_b200_trace.so); the normal build
 * returns GQA_ERR_UNSUPPORTED.  Thread 0 of every CTA records 10 words:
 * {tag = (q pointer << 2) | grid-merged, SM id, globaltimer at start (ns),
 * clock64 at start, clock64 when the dependency wait returned, when q was
 * staged, when warp 0's loop ended, when the partial was stored, when the
 * merged slice's words had all arrived, when the merged slice was stored}
 * (0 = not reached).  Copies up to max_records records of the current device
 * to `records`, sets *n_records to the number recorded since the last reset
 * (at most 65536), and with reset != 0 starts over. */
GQA_API int gqa_phase_trace_read(unsigned long long *records, int max_records, int reset,
                                 int *n_records);

/* Version string of the library. */
GQA_API const char *gqa_version(void);

#ifdef __cplusplus
}
#endif

#endif /* GQA_B200_H */
