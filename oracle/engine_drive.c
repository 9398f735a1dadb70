/*
 * engine_drive.c -- drives the reference engine's own transformer forward
 * (src/transformer/transformer.c, src/model/model.c, src/gguf/gguf.c,
 * compiled unmodified from the reference tree by oracle/Makefile) over a
 * GGUF model: n_tokens greedy-free steps, token i = (7 i + 3) mod n_vocab at
 * position i, the logits of every step written to a file as fp32.  Linked
 * once against the reference's kv_cache.c and once against this
 * repository's library (the drop-in check of the KV interface inside the
 * engine's own loop, transformer.c:183-214).  Test infrastructure only.
 *
 *   engine_drive <model.gguf> <n_tokens> <logits.out>
 */
#include "transformer/transformer.h"

#include <stdio.h>
#include <stdlib.h>

int main(int argc, char **argv) {
    if (argc != 4) { fprintf(stderr, "usage: %s model.gguf n_tokens out\n", argv[0]); return 2; }
    const int n = atoi(argv[2]);
    ct_model_t *m = ct_model_load(argv[1]);
    if (!m || !ct_model_is_loaded(m)) { fprintf(stderr, "model did not load\n"); return 1; }
    ct_transformer_t *t = ct_transformer_create(m, ct_model_n_ctx(m));
    if (!t) { fprintf(stderr, "transformer_create failed\n"); return 1; }
    const uint32_t V = ct_model_n_vocab(m);
    FILE *f = fopen(argv[3], "wb");
    if (!f) return 1;
    for (int i = 0; i < n; i++) {
        const float *lg = ct_transformer_forward(t, (int32_t)((7 * i + 3) % V), (uint32_t)i);
        if (!lg || fwrite(lg, sizeof(float), V, f) != V) { fclose(f); return 1; }
    }
    fclose(f);
    printf("kv_len %u\n", ct_kv_len(ct_transformer_kv(t)));
    ct_transformer_free(t);
    ct_model_free(m);
    return 0;
}
