/*
 * TEST INFRASTRUCTURE (oracle) -- a CPU restatement of the reference's fp32
 * GQA attention path, used only by tests/, the smoke check and the CPU
 * baseline leg of bench.py.  It is never linked into the product library and
 * the product never calls it.
 *
 * It follows cpu_attention_gqa_pipeline() in
 * compute/attention-gqa-resident/attention_gqa_benchmark.c line by line for the
 * attention slice (RoPE :141-170, scores/softmax/PV :172-208), with the shapes
 * and the cache stride t_max as run-time parameters instead of the reference's
 * compile-time HEAD_DIM=128 / T_MAX=4096, so that caches longer than 4096 can
 * be checked.  Built with the reference's own flags (-O3 -mavx2 -mf16c -mfma,
 * compute/attention-gqa-resident/Makefile:2) it reproduces the compiled
 * reference bit for bit at t_max = 4096 (tests/test_oracle_pin.py).
 *
 * Additions that the reference does not have, each stated in natural-exp
 * form so that tests can check the split-KV protocol:
 *   oracle_attention_partial()  un-normalised (m, l, o) over a token range
 *   oracle_lse_combine()        m = max m_g, o = sum e^(m_g-m) o_g / sum e^(m_g-m) l_g
 *   oracle_*_batched()          the same per-sequence math over many sequences,
 *                               OpenMP-parallel over (sequence, q head); each
 *                               head's arithmetic is identical to the serial loop.
 *
 * And the caller's step around the path where the reference's CPU code cannot
 * be compiled for it: the token embedding, the output RMSNorm and the greedy
 * pick (restated from qwen_server.c / test_full_model_logits.c), and the
 * Qwen2.5-0.5B head oracle_gemv_q8_0() (kernel_q8_0.cl:10-61, which the
 * reference has only as OpenCL; pinned bit for bit to that kernel's source
 * compiled as C and run by a work-group scheduler, oracle/ref_q8_harness.c).
 */
#include <immintrin.h>
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <omp.h>

/* attention_gqa_benchmark.c:143 -- the per-pair inverse frequency, fp32 powf */
void oracle_inv_freq(float rope_base, int head_dim, float *out) {
    for (int tid = 0; tid < head_dim / 2; tid++)
        out[tid] = powf(rope_base, -2.0f * (float)tid / (float)head_dim);
}

/* attention_gqa_benchmark.c:141-170: half-rotation RoPE on every q head (in
 * place) and every k head; rotated k and raw v are written to cache row pos.
 * Cache layout [n_kv][t_max][head_dim].  The body is inlined with the
 * reference's compile-time shape (12 / 2 heads, d = 128) when the shape
 * matches, so that gcc vectorises and contracts (FMA) the loops exactly as it
 * does in the reference and the rotated values agree bit for bit. */
static inline __attribute__((always_inline)) void rope_kv_append_body(
    float *q, const float *k, const float *v, float *k_cache, float *v_cache, int pos, int t_max,
    int n_heads_q, int n_heads_kv, int head_dim, float rope_base) {
    int half = head_dim / 2;
    for (int tid = 0; tid < half; tid++) {
        float theta = (float)pos * powf(rope_base, -2.0f * (float)tid / (float)head_dim);
        float cos_th = cosf(theta);
        float sin_th = sinf(theta);

        for (int h = 0; h < n_heads_q; h++) {
            int base = h * head_dim;
            float q0 = q[base + tid];
            float q1 = q[base + tid + half];
            q[base + tid] = q0 * cos_th - q1 * sin_th;
            q[base + tid + half] = q0 * sin_th + q1 * cos_th;
        }

        for (int h = 0; h < n_heads_kv; h++) {
            int in_base = h * head_dim;
            float k0 = k[in_base + tid];
            float k1 = k[in_base + tid + half];

            float k_rot0 = k0 * cos_th - k1 * sin_th;
            float k_rot1 = k0 * sin_th + k1 * cos_th;

            long out_base = ((long)h * t_max + pos) * head_dim;
            k_cache[out_base + tid] = k_rot0;
            k_cache[out_base + tid + half] = k_rot1;

            v_cache[out_base + tid] = v[in_base + tid];
            v_cache[out_base + tid + half] = v[in_base + tid + half];
        }
    }
}

void oracle_rope_kv_append(float *q, const float *k, const float *v, float *k_cache,
                           float *v_cache, int pos, int t_max, int n_heads_q, int n_heads_kv,
                           int head_dim, float rope_base) {
    if (n_heads_q == 12 && n_heads_kv == 2 && head_dim == 128)
        rope_kv_append_body(q, k, v, k_cache, v_cache, pos, t_max, 12, 2, 128, rope_base);
    else
        rope_kv_append_body(q, k, v, k_cache, v_cache, pos, t_max, n_heads_q, n_heads_kv,
                            head_dim, rope_base);
}

/* attention_gqa_benchmark.c:174-208 for one q head: scores, stable softmax
 * (max initialised to -1e30, normaliser 1/(sum + 1e-12)), then P.V.
 * gcc keeps these loops scalar in the reference; with run-time shapes it
 * would vectorise the P.V loop across d and contract it differently (1-2 ulp
 * apart), so vectorisation is switched off here to stay bit-exact. */
__attribute__((optimize("no-tree-vectorize")))
static void attention_one_head(const float *q, const float *k_cache, const float *v_cache,
                               int h_q, int seq_len, int t_max, int group, int head_dim,
                               float *scores, float *attn_out) {
    float scale_factor = 1.0f / sqrtf((float)head_dim);
    int h_kv = h_q / group;
    float max_s = -1e30f;

    for (int t = 0; t < seq_len; t++) {
        float dot = 0.0f;
        long q_off = (long)h_q * head_dim;
        long k_off = ((long)h_kv * t_max + t) * head_dim;
        for (int d = 0; d < head_dim; d++) {
            dot += q[q_off + d] * k_cache[k_off + d];
        }
        scores[t] = dot * scale_factor;
        if (scores[t] > max_s) max_s = scores[t];
    }

    float sum_exp = 0.0f;
    for (int t = 0; t < seq_len; t++) {
        scores[t] = expf(scores[t] - max_s);
        sum_exp += scores[t];
    }
    float inv_sum = 1.0f / (sum_exp + 1e-12f);
    for (int t = 0; t < seq_len; t++) {
        scores[t] *= inv_sum;
    }

    for (int d = 0; d < head_dim; d++) {
        float acc = 0.0f;
        for (int t = 0; t < seq_len; t++) {
            long v_off = ((long)h_kv * t_max + t) * head_dim + d;
            acc += scores[t] * v_cache[v_off];
        }
        attn_out[(long)h_q * head_dim + d] = acc;
    }
}

void oracle_attention(const float *q, const float *k_cache, const float *v_cache, int seq_len,
                      int t_max, int n_heads_q, int n_heads_kv, int head_dim, float *attn_out) {
    int group = n_heads_q / n_heads_kv;
    float *scores = (float *)malloc(sizeof(float) * (size_t)(seq_len > 0 ? seq_len : 1));
    for (int h_q = 0; h_q < n_heads_q; h_q++)
        attention_one_head(q, k_cache, v_cache, h_q, seq_len, t_max, group, head_dim, scores,
                           attn_out);
    free(scores);
}

/* The whole attention slice of one layer call (qwen_server.c:446-450): qkv is
 * [q (n_heads_q*d) | k (n_kv*d) | v (n_kv*d)]; q is rotated in place, k/v are
 * appended at pos, then attn_out overwrites qkv[0 : n_heads_q*d] as the
 * reference's segment reduce does (qwen_server.c:402-404). */
void oracle_layer_attention(float *qkv, float *k_cache, float *v_cache, int pos, int seq_len,
                            int t_max, int n_heads_q, int n_heads_kv, int head_dim,
                            float rope_base) {
    float *q = qkv;
    const float *k = qkv + (long)n_heads_q * head_dim;
    const float *v = k + (long)n_heads_kv * head_dim;
    oracle_rope_kv_append(q, k, v, k_cache, v_cache, pos, t_max, n_heads_q, n_heads_kv, head_dim,
                          rope_base);
    float *out = (float *)malloc(sizeof(float) * (size_t)n_heads_q * head_dim);
    oracle_attention(q, k_cache, v_cache, seq_len, t_max, n_heads_q, n_heads_kv, head_dim, out);
    memcpy(qkv, out, sizeof(float) * (size_t)n_heads_q * head_dim);
    free(out);
}

/* Many sequences at once (one new token each): per sequence, RoPE + append at
 * pos = seq_lens[s] - 1, then attention over seq_lens[s] tokens; the attention
 * is spread over (sequence, q head) pairs on n_threads threads.  out[s] may
 * alias qkv[s] (then it receives attn_out in its first n_heads_q*d floats). */
void oracle_decode_batched(int n_seq, float *const *qkv, float *const *k_caches,
                           float *const *v_caches, const int *seq_lens, int t_max, int n_heads_q,
                           int n_heads_kv, int head_dim, float rope_base, float *const *out,
                           int n_threads) {
    int hd = n_heads_q * head_dim;
    float **qrot = (float **)malloc(sizeof(float *) * (size_t)n_seq);
    #pragma omp parallel for schedule(dynamic, 1) num_threads(n_threads)
    for (int s = 0; s < n_seq; s++) {
        qrot[s] = (float *)malloc(sizeof(float) * (size_t)hd);
        memcpy(qrot[s], qkv[s], sizeof(float) * (size_t)hd);
        const float *k = qkv[s] + hd;
        const float *v = k + (long)n_heads_kv * head_dim;
        oracle_rope_kv_append(qrot[s], k, v, k_caches[s], v_caches[s], seq_lens[s] - 1, t_max,
                              n_heads_q, n_heads_kv, head_dim, rope_base);
    }
    int group = n_heads_q / n_heads_kv;
    long n_items = (long)n_seq * n_heads_q;
    #pragma omp parallel num_threads(n_threads)
    {
        int max_len = 1;
        for (int s = 0; s < n_seq; s++) if (seq_lens[s] > max_len) max_len = seq_lens[s];
        float *scores = (float *)malloc(sizeof(float) * (size_t)max_len);
        #pragma omp for schedule(dynamic, 1)
        for (long it = 0; it < n_items; it++) {
            int s = (int)(it / n_heads_q), h = (int)(it % n_heads_q);
            attention_one_head(qrot[s], k_caches[s], v_caches[s], h, seq_lens[s], t_max, group,
                               head_dim, scores, out[s]);
        }
        free(scores);
    }
    for (int s = 0; s < n_seq; s++) free(qrot[s]);
    free(qrot);
}

/* Attention only (q already rotated, nothing appended) for many sequences;
 * the CPU baseline of the batched and long-context workloads. */
void oracle_attention_batched(int n_seq, const float *const *q, const float *const *k_caches,
                              const float *const *v_caches, const int *seq_lens, int t_max,
                              int n_heads_q, int n_heads_kv, int head_dim, float *const *out,
                              int n_threads) {
    int group = n_heads_q / n_heads_kv;
    long n_items = (long)n_seq * n_heads_q;
    #pragma omp parallel num_threads(n_threads)
    {
        int max_len = 1;
        for (int s = 0; s < n_seq; s++) if (seq_lens[s] > max_len) max_len = seq_lens[s];
        float *scores = (float *)malloc(sizeof(float) * (size_t)max_len);
        #pragma omp for schedule(dynamic, 1)
        for (long it = 0; it < n_items; it++) {
            int s = (int)(it / n_heads_q), h = (int)(it % n_heads_q);
            attention_one_head(q[s], k_caches[s], v_caches[s], h, seq_lens[s], t_max, group,
                               head_dim, scores, out[s]);
        }
        free(scores);
    }
}

/* Split-KV partial over tokens [t_begin, t_end) of one sequence, natural-exp
 * domain: m[h] = max_t s_t, l[h] = sum_t e^(s_t - m), o[h][:] = sum_t e^(s_t - m) v_t
 * with s_t = (q.k_t) / sqrt(d).  An empty range gives m = -inf, l = 0, o = 0. */
void oracle_attention_partial(const float *q, const float *k_cache, const float *v_cache,
                              int t_begin, int t_end, int t_max, int n_heads_q, int n_heads_kv,
                              int head_dim, float *m, float *l, float *o) {
    int group = n_heads_q / n_heads_kv;
    float scale_factor = 1.0f / sqrtf((float)head_dim);
    int n = t_end - t_begin;
    float *scores = (float *)malloc(sizeof(float) * (size_t)(n > 0 ? n : 1));
    for (int h_q = 0; h_q < n_heads_q; h_q++) {
        int h_kv = h_q / group;
        float max_s = -INFINITY;
        for (int t = t_begin; t < t_end; t++) {
            float dot = 0.0f;
            long k_off = ((long)h_kv * t_max + t) * head_dim;
            for (int d = 0; d < head_dim; d++) dot += q[(long)h_q * head_dim + d] * k_cache[k_off + d];
            scores[t - t_begin] = dot * scale_factor;
            if (scores[t - t_begin] > max_s) max_s = scores[t - t_begin];
        }
        float sum = 0.0f;
        for (int i = 0; i < n; i++) { scores[i] = expf(scores[i] - max_s); sum += scores[i]; }
        for (int d = 0; d < head_dim; d++) {
            float acc = 0.0f;
            for (int t = t_begin; t < t_end; t++)
                acc += scores[t - t_begin] * v_cache[((long)h_kv * t_max + t) * head_dim + d];
            o[(long)h_q * head_dim + d] = acc;
        }
        m[h_q] = max_s;
        l[h_q] = sum;
    }
    free(scores);
}

/* Log-sum-exp combine of n_parts partials laid out [part][n_heads_q](m, l) and
 * [part][n_heads_q][head_dim] (o) into out[n_heads_q][head_dim]. */
void oracle_lse_combine(int n_parts, const float *m, const float *l, const float *o,
                        int n_heads_q, int head_dim, float *out) {
    for (int h = 0; h < n_heads_q; h++) {
        float mx = -INFINITY;
        for (int p = 0; p < n_parts; p++) if (m[p * n_heads_q + h] > mx) mx = m[p * n_heads_q + h];
        float den = 0.0f;
        float *w = (float *)malloc(sizeof(float) * (size_t)n_parts);
        for (int p = 0; p < n_parts; p++) {
            float mp = m[p * n_heads_q + h];
            w[p] = (mp == -INFINITY) ? 0.0f : expf(mp - mx);
            den += w[p] * l[p * n_heads_q + h];
        }
        for (int d = 0; d < head_dim; d++) {
            float acc = 0.0f;
            for (int p = 0; p < n_parts; p++)
                acc += w[p] * o[((long)p * n_heads_q + h) * head_dim + d];
            out[(long)h * head_dim + d] = den > 0.0f ? acc / den : 0.0f;
        }
        free(w);
    }
}

/* Causal prefill of one sequence of S tokens stated as the reference's own
 * token-by-token decode (qwen_server.c:957-964: pos = p, seq_len = p + 1):
 * q/k/v are [S][n_heads*d] (pre-RoPE); every k/v row is rotated and appended
 * first (k_cache/v_cache [n_kv][t_max][d], t_max >= S), then attention is
 * evaluated only for the n_rows query positions in rows[] (the others are not
 * needed by the tests and would make the check slow).  out: [n_rows][n_heads_q*d]. */
void oracle_prefill_rows(const float *q, const float *k, const float *v, int S, int t_max,
                         int n_heads_q, int n_heads_kv, int head_dim, float rope_base,
                         float *k_cache, float *v_cache, const int *rows, int n_rows,
                         float *out, int n_threads) {
    int hq = n_heads_q * head_dim, hk = n_heads_kv * head_dim;
    float *qrot = (float *)malloc(sizeof(float) * (size_t)n_rows * hq);
    float *scratch_q = (float *)malloc(sizeof(float) * (size_t)hq);
    for (int p = 0; p < S; p++) {
        memcpy(scratch_q, q + (long)p * hq, sizeof(float) * (size_t)hq);
        oracle_rope_kv_append(scratch_q, k + (long)p * hk, v + (long)p * hk, k_cache, v_cache, p,
                              t_max, n_heads_q, n_heads_kv, head_dim, rope_base);
        for (int r = 0; r < n_rows; r++)
            if (rows[r] == p) memcpy(qrot + (long)r * hq, scratch_q, sizeof(float) * (size_t)hq);
    }
    free(scratch_q);
    int group = n_heads_q / n_heads_kv;
    long n_items = (long)n_rows * n_heads_q;
    #pragma omp parallel num_threads(n_threads)
    {
        float *scores = (float *)malloc(sizeof(float) * (size_t)S);
        #pragma omp for schedule(dynamic, 1)
        for (long it = 0; it < n_items; it++) {
            int r = (int)(it / n_heads_q), h = (int)(it % n_heads_q);
            attention_one_head(qrot + (long)r * hq, k_cache, v_cache, h, rows[r] + 1, t_max, group,
                               head_dim, scores, out + (long)r * hq);
        }
        free(scores);
    }
    free(qrot);
}

/* ---- around the decoder layers: embedding, output norm, greedy pick ---- */

/* fp16 -> fp32 as the reference converts it (fp16_to_float,
 * qwen_server.c:66-68: _cvtsh_ss, F16C). */
static float oracle_fp16_to_float(uint16_t h) { return _cvtsh_ss(h); }

/* get_token_embedding (qwen_server.c:188-201): row `token` of a Q4_0 table of
 * d_model / 32 blocks of 18 bytes, x[32b + j] = ((qs[j] & 15) - 8) * d and
 * x[32b + j + 16] = ((qs[j] >> 4) - 8) * d. */
void oracle_token_embedding(const uint8_t *table, int d_model, int token, float *x) {
    int nb = d_model / 32;
    const uint8_t *row = table + (size_t)token * nb * 18;
    for (int b = 0; b < nb; b++) {
        const uint8_t *blk = row + 18 * b;
        float d = oracle_fp16_to_float((uint16_t)(blk[0] | (blk[1] << 8)));
        for (int j = 0; j < 16; j++) {
            uint8_t q = blk[2 + j];
            x[b * 32 + j] = (float)((int)(q & 0x0F) - 8) * d;
            x[b * 32 + j + 16] = (float)((int)(q >> 4) - 8) * d;
        }
    }
}

/* The output RMSNorm of the whole-model check (test_full_model_logits.c:
 * 944-948): fp32 sum of squares in index order, scale = 1 / sqrtf(sum / n +
 * eps), z = x * scale * gamma. */
void oracle_output_norm(const float *x, const float *gamma, int n, float eps, float *z) {
    float sum_sq = 0.0f;
    for (int i = 0; i < n; i++) sum_sq += x[i] * x[i];
    float scale = 1.0f / sqrtf((sum_sq / (float)n) + eps);
    for (int i = 0; i < n; i++) z[i] = x[i] * scale * gamma[i];
}

/* The Qwen2.5-0.5B LM head, gemv_q8_0 (kernel_q8_0.cl:10-61), restated on
 * the CPU (the reference has no CPU path for it).  For each row, lane l of
 * the kernel's 32-lane group accumulates d_b * q_bl * x[32b + l] over the row's
 * k / 32 blocks in block order (:30-37); the 32 lane sums then meet by the
 * kernel's tree, halves 16, 8, 4, 2, 1 (:40-53).  w: n_rows rows of k / 32
 * block_q8_0 (fp16 d, 32 int8 codes; 34 bytes each).  Pinned bit for bit to
 * the kernel's own source run on the CPU (oracle/ref_q8_harness.c). */
__attribute__((optimize("fp-contract=off")))  /* each product rounded, then added, as the
                                                kernel's source reads (no fused multiply-add) */
void oracle_gemv_q8_0(const uint8_t *w, const float *x, int n_rows, int k, float *y) {
    const int nb = k / 32;
    for (int r = 0; r < n_rows; r++) {
        const uint8_t *row = w + (size_t)r * nb * 34;
        float acc[32];
        for (int l = 0; l < 32; l++) acc[l] = 0.0f;
        for (int b = 0; b < nb; b++) {
            const uint8_t *blk = row + b * 34;
            const float d = oracle_fp16_to_float((uint16_t)(blk[0] | (blk[1] << 8)));
            for (int l = 0; l < 32; l++)
                acc[l] += d * (float)(int8_t)blk[2 + l] * x[b * 32 + l];
        }
        for (int s = 16; s > 0; s >>= 1)
            for (int l = 0; l < s; l++) acc[l] += acc[l + s];
        y[r] = acc[0];
    }
}

/* The server's greedy pick (qwen_server.c:998-1005): best_val starts at
 * -1e30, a logit replaces it only when strictly larger, so the first row of
 * the maximum wins, NaN never does, and 0 comes back when nothing beats -1e30. */
int oracle_greedy_pick(const float *logits, int n) {
    int best_tok = 0;
    float best_val = -1e30f;
    for (int i = 0; i < n; i++) {
        if (logits[i] > best_val) {
            best_val = logits[i];
            best_tok = i;
        }
    }
    return best_tok;
}
