/*
 * TEST INFRASTRUCTURE (oracle) -- never linked into the product library.
 *
 * Compiles the reference's Q6_K LM-head check,
 * compute/gguf-real-weights-loader/test_gemv_q6_k.c, unmodified (the Makefile
 * passes the file's path as REF_HEAD_SRC) and exports its CPU path:
 *   ref_gemv_q6_k     cpu_gemv_q6_k_ref (:77-94): each row dequantised by
 *                     dequantize_row_q6_k_ref (the GGML order, :46-74), then an
 *                     fp32 dot product in index order; OpenMP over rows.
 *   ref_dequant_q6_k  dequantize_row_q6_k_ref of one 1536-wide row.
 * The same routines appear verbatim in test_full_model_logits.c (:146-176,
 * :950-958), where they form the CPU LM head of the whole-model check.
 */
#define main gqa_reference_q6k_main_unused
#include REF_HEAD_SRC
#undef main

int ref_head_d_model(void) { return D_MODEL; }

void ref_gemv_q6_k(const uint8_t *W, const float *x, float *y, int M) {
    cpu_gemv_q6_k_ref(W, x, y, M, D_MODEL);
}

void ref_dequant_q6_k(const uint8_t *row, float *y) { dequantize_row_q6_k_ref(row, y, D_MODEL); }
