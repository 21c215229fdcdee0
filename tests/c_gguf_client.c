/* c_gguf_client.c — a plain C99 client of the GGUF part of include/ti_b200.h,
 * which needs no GPU (test infrastructure).
 *
 *     c_gguf_client model.gguf
 *
 * Prints the model description, every token of tokenizer.ggml.tokens (one per
 * line, as "token <i> <bytes>"), and for each tensor its name, ggml type, the
 * reference name it maps to and a checksum of its bf16 conversion (the sum of
 * the bf16 bit patterns).  Exit status 0, or 1 with the library's message. */
#include <stdio.h>
#include <stdlib.h>

#include "ti_b200.h"

#define CHECK(call)                                                                  \
    do {                                                                             \
        ti_status st_ = (call);                                                      \
        if (st_ != TI_OK) {                                                          \
            fprintf(stderr, "%s: status %d: %s\n", #call, (int)st_, ti_last_error()); \
            if (g) ti_gguf_close(g);                                                 \
            return 1;                                                                \
        }                                                                            \
    } while (0)

int main(int argc, char** argv) {
    ti_gguf* g = NULL;
    if (argc < 2) {
        fprintf(stderr, "usage: %s model.gguf\n", argv[0]);
        return 2;
    }
    CHECK(ti_gguf_open(argv[1], &g));
    ti_model_desc d;
    CHECK(ti_gguf_model_desc(g, &d));
    printf("desc arch %d hidden %d layers %d heads %d kv %d head_dim %d inter %d vocab %d wfmt %d\n", d.arch,
           d.hidden, d.n_layers, d.n_heads, d.n_kv_heads, d.head_dim, d.intermediate, d.vocab, d.weight_format);
    int64_t n_tok = 0;
    CHECK(ti_gguf_meta_array_len(g, "tokenizer.ggml.tokens", &n_tok));
    for (int64_t i = 0; i < n_tok; ++i) {
        const char* s = NULL;
        size_t len = 0;
        CHECK(ti_gguf_meta_array_string(g, "tokenizer.ggml.tokens", i, &s, &len));
        printf("token %lld %.*s\n", (long long)i, (int)len, s);
    }
    int n = 0;
    CHECK(ti_gguf_tensor_count(g, &n));
    for (int i = 0; i < n; ++i) {
        const char* name = NULL;
        int type = 0, nd = 0;
        int64_t dims[4] = {1, 1, 1, 1};
        const void* data = NULL;
        size_t bytes = 0;
        CHECK(ti_gguf_tensor_info(g, i, &name, &type, &nd, dims, &data, &bytes));
        char ref[256];
        if (ti_gguf_reference_name(g, i, ref, sizeof ref) != TI_OK) ref[0] = 0;
        size_t elems = 1;
        for (int k = 0; k < nd; ++k) elems *= (size_t)dims[k];
        uint16_t* bf = (uint16_t*)malloc(elems * 2);
        if (!bf) return 1;
        unsigned long long sum = 0;
        if (ti_gguf_read(g, i, TI_DTYPE_BF16, bf, elems * 2) == TI_OK)
            for (size_t k = 0; k < elems; ++k) sum += bf[k];
        free(bf);
        printf("tensor %s type %d ref %s bf16sum %llu\n", name, type, ref[0] ? ref : "-", sum);
    }
    CHECK(ti_gguf_close(g));
    return 0;
}
