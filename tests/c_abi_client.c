/* c_abi_client.c — a plain C99 client of include/ti_b200.h, as a C or FFI binding
 * of the reference side would use it (test infrastructure).
 *
 *     c_abi_client [steps] [p]
 *
 * Checks the hardware (ti_init), builds a 2-layer Llama-shape engine with
 * synthetic weights, prefills a 6-token prompt and decodes `steps` tokens,
 * greedy or, with a second argument "p", top-p 0.9 at temperature 0.8 with
 * seed 7.  Prints the ids on one line.  Exit status: 0 done; 2 the library
 * reports the hardware unsupported (no B200); 1 any other error. */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "ti_b200.h"

#define CHECK(call)                                                                          \
    do {                                                                                     \
        ti_status st_ = (call);                                                              \
        if (st_ != TI_OK) {                                                                  \
            fprintf(stderr, "%s: status %d: %s\n", #call, (int)st_, ti_last_error());        \
            if (eng) ti_engine_destroy(eng);                                                 \
            return st_ == TI_ERR_UNSUPPORTED ? 2 : 1;                                        \
        }                                                                                    \
    } while (0)

int main(int argc, char** argv) {
    ti_engine* eng = NULL;
    const int steps = argc > 1 ? atoi(argv[1]) : 4;
    const int top_p = argc > 2 && argv[2][0] == 'p';
    int n_devices = 0;
    CHECK(ti_init(&n_devices));

    ti_model_desc d;
    memset(&d, 0, sizeof d);
    d.arch = TI_ARCH_LLAMA;
    d.hidden = 256;
    d.n_layers = 2;
    d.n_heads = 4;
    d.n_kv_heads = 2;
    d.head_dim = 64;
    d.intermediate = 512;
    d.vocab = 1000;
    d.rms_eps = 1e-5f;
    d.rope_theta = 10000.0f;
    d.weight_format = TI_WFMT_BF16;

    ti_engine_opts o;
    memset(&o, 0, sizeof o);
    o.max_batch = 1;
    o.max_seqs = 1;
    o.max_seq_len = 64;
    o.tp_size = 1;
    CHECK(ti_engine_create(&d, &o, &eng));
    CHECK(ti_engine_init_synthetic(eng, 0, 0.02f));

    int seq = -1;
    CHECK(ti_seq_create(eng, &seq));
    if (top_p) {
        ti_sampling s;
        memset(&s, 0, sizeof s);
        s.kind = TI_SAMPLE_TOP_P;
        s.temperature = 0.8f;
        s.p = 0.9f;
        s.seeded = 1;
        s.seed = 7;
        CHECK(ti_engine_seq_set_sampler(eng, seq, &s));
    }
    const int32_t prompt[6] = {1, 17, 256, 42, 999, 3};
    int32_t tok = 0;
    CHECK(ti_engine_prefill(eng, seq, prompt, 6, -1, &tok, TI_LOGITS_NONE, NULL));
    printf("%d", (int)tok);
    for (int i = 0; i < steps; ++i) {
        int32_t next = 0;
        CHECK(ti_engine_decode(eng, 1, &seq, &tok, NULL, &next, TI_LOGITS_NONE, NULL, NULL));
        tok = next;
        printf(" %d", (int)tok);
    }
    printf("\n");
    CHECK(ti_engine_check(eng));
    CHECK(ti_engine_destroy(eng));
    eng = NULL;
    CHECK(ti_shutdown());
    return 0;
}
