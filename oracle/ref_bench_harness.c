/*
 * TEST INFRASTRUCTURE (oracle) -- never linked into the product library.
 *
 * Compiles the reference's own CPU attention block,
 * cpu_attention_gqa_pipeline() at compute/attention-gqa-resident/
 * attention_gqa_benchmark.c:109-216, unmodified: the Makefile in this folder
 * passes the reference file's path as REF_BENCH_SRC and this unit #includes it
 * with its main() renamed (the OpenCL host program is then dropped by
 * --gc-sections).
 *
 * The reference function starts from the residual stream x (RMSNorm, then a
 * Q4_0 QKV GEMV plus bias).  To feed it a chosen q/k/v we give it all-zero
 * Q4_0 weights (fp16 scale 1.0, every nibble 8, i.e. weight 0) and put the
 * wanted [q | k | v] into the bias, exactly as cpu_gemv_q4_0_bias()
 * (attention_gqa_benchmark.c:86-106) then yields qkv = bias bit for bit.  The
 * attention output attn_out (:206) is what we return; r_out is discarded.
 *
 * Cache layout is the reference's: [N_HEADS_KV=2][T_MAX=4096][HEAD_DIM=128]
 * fp32, so callers must pass caches of exactly that shape.
 */
#include <pthread.h>

#define main gqa_reference_bench_main_unused
#include REF_BENCH_SRC
#undef main

static block_q4_0 *g_zero_wqkv;
static block_q4_0 *g_zero_wo;
static float g_gamma[D_MODEL];
static float g_x[D_MODEL];
static pthread_once_t g_once = PTHREAD_ONCE_INIT;

static void init_zero_weights(void) {
    size_t nb = D_MODEL / QK4_0;
    g_zero_wqkv = (block_q4_0 *)malloc(sizeof(block_q4_0) * (size_t)D_QKV * nb);
    g_zero_wo = (block_q4_0 *)malloc(sizeof(block_q4_0) * (size_t)D_MODEL * nb);
    for (size_t i = 0; i < (size_t)D_QKV * nb; i++) {
        g_zero_wqkv[i].d = 0x3C00; /* fp16 1.0 */
        memset(g_zero_wqkv[i].qs, 0x88, sizeof(g_zero_wqkv[i].qs));
    }
    for (size_t i = 0; i < (size_t)D_MODEL * nb; i++) {
        g_zero_wo[i].d = 0x3C00;
        memset(g_zero_wo[i].qs, 0x88, sizeof(g_zero_wo[i].qs));
    }
    for (int i = 0; i < D_MODEL; i++) { g_gamma[i] = 1.0f; g_x[i] = 0.0f; }
}

int ref_bench_t_max(void) { return T_MAX; }

/* One call of the reference attention block.  qkv_in: [2048] = q[1536] | k[256]
 * | v[256] (pre-RoPE).  k_cache/v_cache: [2][4096][128], updated in place at
 * row pos.  attn_out: [1536]. */
int ref_bench_attention(const float *qkv_in, float *k_cache, float *v_cache,
                        int pos, int seq_len, float *attn_out) {
    if (pos < 0 || pos >= T_MAX || seq_len < 1 || seq_len > T_MAX) return -1;
    pthread_once(&g_once, init_zero_weights);
    float r_out[D_MODEL];
    cpu_attention_gqa_pipeline(g_x, g_gamma, g_zero_wqkv, qkv_in, g_zero_wo,
                               k_cache, v_cache, pos, seq_len, attn_out, r_out);
    return 0;
}

/* Many independent calls (e.g. the layers of one decode step, whose inputs are
 * all known up front in the synthetic workload) spread over n_threads host
 * threads.  Each call is the unmodified reference function; the reference's
 * inner OpenMP GEMV regions run single-threaded inside (nested parallelism is
 * off by default). */
int ref_bench_attention_many(int n, const float *const *qkv_in, float *const *k_cache,
                             float *const *v_cache, const int *pos, const int *seq_len,
                             float *const *attn_out, int n_threads) {
    pthread_once(&g_once, init_zero_weights);
    int bad = 0;
    #pragma omp parallel for schedule(dynamic, 1) num_threads(n_threads) reduction(|:bad)
    for (int i = 0; i < n; i++) {
        bad |= ref_bench_attention(qkv_in[i], k_cache[i], v_cache[i], pos[i], seq_len[i],
                                   attn_out[i]) != 0;
    }
    return bad ? -1 : 0;
}
