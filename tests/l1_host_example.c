/* l1_host_example.c -- the registration a host program adds to use the B200 backend through the
 * reference's own L1 session (the code INTEGRATION.md shows), as a program: compiled against the
 * reference's frozen headers (sp/sp_l1.h) and linked with the reference's library and
 * libspb200_l1.so. Used by tests/test_l1_host_example.py.
 *
 *   l1_host_example MODEL.sp-model TOKENIZER.sp-tokenizer N_PROMPT OUT.f32
 *
 * Prefills N_PROMPT tokens (1, 2, ...) through section 6, opens a section-6b cache on the same
 * model, feeds it the prompt and takes one decode step; prints one "step rc" line per call and
 * writes the decode step's logits to OUT.f32 when every call succeeded. Without a usable GPU the
 * device calls must return a status (and the reference session its SP_EBADSTATE with the
 * backend's detail), never crash. */
#include "sp/sp_l1.h"
#include "spb200_l1.h"

#include <stdio.h>
#include <stdlib.h>

int main(int argc, char **argv) {
    if (argc != 5) {
        fprintf(stderr, "usage: %s MODEL TOKENIZER N_PROMPT OUT\n", argv[0]);
        return 2;
    }
    const int n = atoi(argv[3]);
    sp_model *m = NULL;
    if (sp_model_load(argv[1], argv[2], &m) != SP_OK) {
        printf("load %s\n", sp_last_error());
        return 3;
    }
    sp_arch_info ai;
    if (sp_model_arch(m, &ai) != SP_OK) return 4;
    sp_session_config cfg = {0};
    cfg.max_context = (size_t)n + 8;
    sp_session *s = NULL;
    if (sp_session_create(m, &cfg, NULL, &s) != SP_OK) {
        printf("create %s\n", sp_last_error());
        return 5;
    }
    int32_t *toks = malloc(sizeof(int32_t) * (size_t)n);
    float *lg = malloc(sizeof(float) * ai.vocab_size);
    for (int i = 0; i < n; i++) toks[i] = 1 + i;
    int failed = 0;

    /* section 6: the prefill runs on the GPU */
    sp_status rc = sp_session_register_forward_backend(s, spb_l1_backend(), spb_l1_forward);
    printf("register6 %d\n", (int)rc);
    rc = sp_prefill_chunk(s, toks, (size_t)n, lg, ai.vocab_size);
    printf("prefill6 %d %s\n", (int)rc, rc ? sp_last_error() : "");
    failed |= rc != SP_OK;

    /* section 6b: a resident cache on the GPU, fed the prompt, one decode step */
    const sp_kvdecode_dispatch_fn *dt = spb_l1_kvdecode_table();
    sp_kvdecode_handle *h = NULL;
    const void *qm = sp_session_qwen3_model(s);
    int orc = dt->open(qm, (int)cfg.max_context, &h);
    printf("open6b %d %s\n", orc, orc ? sp_last_error() : "");
    failed |= orc != 0;
    if (orc == 0) {
        int prc = dt->prefill(h, toks, n);
        printf("prefill6b %d\n", prc);
        failed |= prc != 0;
        int drc = dt->decode_step(h, toks[n - 1], lg);
        printf("decode6b %d position %d\n", drc, dt->position(h));
        failed |= drc != 0;
        dt->close(h);
    }
    if (!failed) {
        FILE *f = fopen(argv[4], "wb");
        if (!f || fwrite(lg, sizeof(float), ai.vocab_size, f) != ai.vocab_size) return 6;
        fclose(f);
    }
    spb_l1_release_model(qm);   /* before the model goes */
    sp_session_destroy(s);
    sp_model_unload(m);
    free(lg);
    free(toks);
    printf("done %d\n", failed);
    return 0;
}
