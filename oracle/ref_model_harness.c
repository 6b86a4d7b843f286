/*
 * TEST INFRASTRUCTURE (oracle) -- never linked into the product library.
 *
 * Compiles the reference's whole-model check,
 * compute/gguf-real-weights-loader/test_full_model_logits.c, unmodified (the
 * Makefile passes the file's path as REF_MODEL_SRC) and exports its token
 * embedding lookup:
 *   ref_token_embedding  get_token_embedding (:584-597; the same function as
 *                        qwen_server.c:188-201): pread of the token's 48 Q4_0
 *                        blocks from the model file, dequantised on the host.
 * The function reads a file descriptor, so the table is handed to it through
 * an anonymous in-memory file.
 */
#define main gqa_reference_model_main_unused
#include REF_MODEL_SRC
#undef main

#include <sys/mman.h>

/* table: n_bytes of Q4_0 rows (48 blocks of 18 bytes each); returns 0 on success. */
int ref_token_embedding(const uint8_t *table, long long n_bytes, int token, float *x_out) {
    if (token < 0 || (long long)(token + 1) * 48 * (long long)sizeof(block_q4_0) > n_bytes) return -1;
    int fd = memfd_create("gqa_oracle_embd", 0);
    if (fd < 0) return -2;
    long long done = 0;
    while (done < n_bytes) {
        ssize_t w = write(fd, table + done, (size_t)(n_bytes - done));
        if (w <= 0) { close(fd); return -3; }
        done += w;
    }
    get_token_embedding(fd, 0, token, x_out);
    close(fd);
    return 0;
}
