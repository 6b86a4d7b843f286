/*
 * TEST INFRASTRUCTURE (oracle) -- never linked into the product library.
 *
 * Compiles the reference's resident server,
 * compute/gguf-real-weights-loader/qwen_server.c, unmodified (the Makefile
 * passes the file's path as REF_SERVER_SRC) and exports its GGUF reading:
 *   ref_gguf_parse   parse_gguf_tensors (:113-178): header, metadata skipped
 *                    by value type, the tensor table, data start rounded up
 *                    to 32 bytes, absolute offsets;
 *   ref_gguf_token   load_tokenizer_tokens (:203-266): the string of one
 *                    token id of tokenizer.ggml.tokens.
 * The socket daemon (its main) and the OpenCL set-up are discarded by the
 * linker with the rest of main.
 */
#define main gqa_reference_server_main_unused
#include REF_SERVER_SRC
#undef main

/* Parses the file at path.  Per tensor i < return value: names[64 i ..]
 * (NUL-terminated), n_dims[i], ne[4 i ..], types[i], abs_offsets[i].
 * Returns the tensor count, or a negative value on failure. */
int ref_gguf_parse(const char *path, int max_tensors, char *names, uint32_t *n_dims, uint64_t *ne,
                   uint32_t *types, uint64_t *abs_offsets, uint64_t *data_start) {
    int fd = open(path, O_RDONLY);
    if (fd < 0) return -1;
    uint64_t header[3];
    /* parse_gguf_tensors writes one entry per tensor of the file without a
     * bound: refuse files with more tensors than the caller has room for */
    if (pread(fd, header, sizeof(header), 0) != (ssize_t)sizeof(header) ||
        (uint64_t)max_tensors < header[1]) {
        close(fd);
        return -2;
    }
    GGUFTensor *t = (GGUFTensor *)calloc((size_t)max_tensors, sizeof(GGUFTensor));
    int n = parse_gguf_tensors(fd, t, max_tensors, data_start);
    close(fd);
    for (int i = 0; i < n; i++) {
        memcpy(names + 64 * i, t[i].name, 64);
        n_dims[i] = t[i].n_dims;
        for (int d = 0; d < 4; d++) ne[4 * i + d] = t[i].ne[d];
        types[i] = t[i].type;
        abs_offsets[i] = t[i].abs_offset;
    }
    free(t);
    return n;
}

/* Copies the string of token `id` (at most cap - 1 bytes) into out; returns
 * the vocabulary size, or a negative value on failure. */
int ref_gguf_token(const char *path, int id, char *out, int cap) {
    int fd = open(path, O_RDONLY);
    if (fd < 0) return -1;
    int count = 0;
    char **tokens = load_tokenizer_tokens(fd, &count);
    close(fd);
    if (!tokens) return -2;
    int rc = count;
    if (id >= 0 && id < count) {
        strncpy(out, tokens[id], (size_t)cap - 1);
        out[cap - 1] = '\0';
    } else {
        rc = -3;
    }
    for (int i = 0; i < count; i++) free(tokens[i]);
    free(tokens);
    return rc;
}
