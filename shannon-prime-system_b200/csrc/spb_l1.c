/* spb_l1.c -- section-6 / section-6b backend of libshannonprime on the B200 forward.
 *
 * Compiled against the reference's frozen L1 headers; the only reference symbols it
 * calls are resolved from the host process (libshannonprime): sp_arena_find
 * (arena.c:143-148), sp_as_f32 (forward_dispatch.c:182-188) and sp_set_error
 * (sp_error.c:22). It walks the borrowed qwen3_model (model.h:150-182) the session
 * hands to the hooks, checks every matmul weight is an OK_Q4B arena tensor (bscale
 * set, all rows Q4, row_off == r * ceil(cols/2): the layout sp_model_bridge.c:114-148
 * builds), and passes plain pointers to spb_model_upload.
 */
#include "sp/sp_l1.h"
#include "sp/model.h"
#include "sp/arena.h"
#include "sp/forward_dispatch.h"
#include "sp/sp_error.h"

#include "../../include/spb200.h"
#include "../../include/spb200_l1.h"

#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define SPB_L1_MAX_MODELS 32

static unsigned g_kv_flags = 0;   /* spb_session_open_ex flags of section-6b caches */
static pthread_mutex_t g_mu = PTHREAD_MUTEX_INITIALIZER;
static struct { const void *qm; uint64_t fp; spb_model *m; spb_kvpool *pool; } g_models[SPB_L1_MAX_MODELS];
static int g_device = 0;
static int g_pool_pg = 0, g_pool_pages = 0;   /* spb_l1_set_kv_pool: 0 = unpaged caches */
static int g_backend_tag;

static int fail(const char *what) {
    char buf[640];
    snprintf(buf, sizeof buf, "spb200: %s: %s", what, spb_last_error());
    sp_set_error(buf);
    return 1;
}

static const sp_frob_packed_tensor *packed_of(const qwen3_model *qm, const gguf_tensor *t) {
    if (!t || !qm->arena) return NULL;
    const sp_arena_tensor *at = sp_arena_find(qm->arena, t->name);
    return at ? &at->pt : NULL;
}

static int q4b_of(const qwen3_model *qm, const gguf_tensor *t, spb_q4b *out) {
    const sp_frob_packed_tensor *pt = packed_of(qm, t);
    if (!pt) return 0;
    if (!pt->bscale || !pt->codes || pt->bs_nblk != (pt->cols + 31) / 32) return 0;
    const size_t nib = (size_t)(pt->cols + 1) / 2;
    for (int r = 0; r < pt->rows; r++)
        if (pt->row_prec[r] != 4 || pt->row_off[r] != (size_t)r * nib) return 0;
    out->codes = pt->codes;
    out->bscale = pt->bscale;
    out->rows = pt->rows;
    out->cols = pt->cols;
    return 1;
}

static spb_model *upload(const qwen3_model *qm) {
    const qwen3_config *c = &qm->cfg;
    if (c->arch != SP_ARCH_GEMMA3 && c->arch != SP_ARCH_QWEN3) {
        sp_set_error("spb200: only the Gemma3 and Qwen3 forwards are on the B200 path");
        return NULL;
    }
    spb_layer_desc *ly = (spb_layer_desc *)calloc(c->n_layers, sizeof *ly);
    if (!ly) { sp_set_error("spb200: out of memory"); return NULL; }
    spb_model_desc d;
    memset(&d, 0, sizeof d);
    d.cfg.arch = c->arch == SP_ARCH_GEMMA3 ? SPB_ARCH_GEMMA3 : SPB_ARCH_QWEN3;
    d.cfg.n_layers = (int32_t)c->n_layers;
    d.cfg.n_embd = (int32_t)c->n_embd;
    d.cfg.n_ff = (int32_t)c->n_ff;
    d.cfg.n_head = (int32_t)c->n_head;
    d.cfg.n_head_kv = (int32_t)c->n_head_kv;
    d.cfg.head_dim = (int32_t)c->head_dim;
    d.cfg.n_vocab = (int32_t)c->n_vocab;
    d.cfg.sliding_window = (int32_t)c->sliding_window;
    d.cfg.rope_base = c->rope_freq_base;
    d.cfg.rope_base_local = 10000.0f;            /* local-layer base, sp_session.c:397 */
    d.cfg.swa_period = 6;                        /* L % 6 == 5 is global, sp_session.c:396 */
    d.cfg.has_qk_norm = c->has_qk_norm;
    d.layers = ly;
    int ok = 1;
    for (uint32_t L = 0; L < c->n_layers && ok; L++) {
        const qwen3_layer *s = &qm->layers[L];
        ok = q4b_of(qm, s->attn_q, &ly[L].wq) && q4b_of(qm, s->attn_k, &ly[L].wk) &&
             q4b_of(qm, s->attn_v, &ly[L].wv) && q4b_of(qm, s->attn_output, &ly[L].wo) &&
             q4b_of(qm, s->ffn_gate, &ly[L].wg) && q4b_of(qm, s->ffn_up, &ly[L].wu) &&
             q4b_of(qm, s->ffn_down, &ly[L].wd);
        ly[L].attn_norm = sp_as_f32(qm, s->attn_norm);
        ly[L].ffn_norm = sp_as_f32(qm, s->ffn_norm);
        ly[L].q_norm = s->attn_q_norm ? sp_as_f32(qm, s->attn_q_norm) : NULL;
        ly[L].k_norm = s->attn_k_norm ? sp_as_f32(qm, s->attn_k_norm) : NULL;
        ly[L].post_attn_norm = s->post_attn_norm ? sp_as_f32(qm, s->post_attn_norm) : NULL;
        ly[L].post_ffw_norm = s->post_ffw_norm ? sp_as_f32(qm, s->post_ffw_norm) : NULL;
    }
    ok = ok && q4b_of(qm, qm->token_embd, &d.token_embd) && q4b_of(qm, qm->output, &d.output);
    d.output_norm = sp_as_f32(qm, qm->output_norm);
    spb_model *m = NULL;
    if (!ok) {
        sp_set_error("spb200: a matmul weight is not an OK_Q4B arena tensor (only OK_Q4B models run on the B200 path)");
    } else if (spb_model_upload(&d, g_device, &m) != SPB_OK) {
        fail("model upload");
        m = NULL;
    }
    free(ly);
    return m;
}

static uint64_t fnv1a(uint64_t h, const void *p, size_t n) {
    const unsigned char *b = (const unsigned char *)p;
    for (size_t i = 0; i < n; i++) { h ^= b[i]; h *= 1099511628211ull; }
    return h;
}

/* The identity of a borrowed model beyond its address (a model unloaded without
 * spb_l1_release_model and another loaded at the same address must not find the first one's
 * device copy): FNV-1a over the config, the arena pointer, and the pointers and first bytes of
 * the embedding's and the first layer's Q codes and block scales. */
static uint64_t fingerprint(const qwen3_model *qm) {
    uint64_t h = 14695981039346656037ull;
    h = fnv1a(h, &qm->cfg, sizeof qm->cfg);
    h = fnv1a(h, &qm->arena, sizeof qm->arena);
    const gguf_tensor *ts[2] = {qm->token_embd, qm->cfg.n_layers > 0 ? qm->layers[0].attn_q : NULL};
    for (int i = 0; i < 2; i++) {
        const sp_frob_packed_tensor *pt = packed_of(qm, ts[i]);   /* (no per-row walk: pointers and bytes) */
        if (!pt || !pt->codes || !pt->bscale || pt->rows <= 0 || pt->cols <= 0) continue;
        const size_t row = (size_t)(pt->cols + 1) / 2, nblk = (size_t)(pt->cols + 31) / 32;
        h = fnv1a(h, &pt->codes, sizeof pt->codes);
        h = fnv1a(h, &pt->bscale, sizeof pt->bscale);
        h = fnv1a(h, pt->codes, row < 64 ? row : 64);
        h = fnv1a(h, pt->bscale, (nblk < 16 ? nblk : 16) * 2);
    }
    return h;
}

static spb_model *model_for(const void *qm_opaque, spb_kvpool **pool) {
    if (!qm_opaque) { sp_set_error("spb200: null model"); return NULL; }
    spb_model *m = NULL;
    if (pool) *pool = NULL;
    const uint64_t fp = fingerprint((const qwen3_model *)qm_opaque);
    pthread_mutex_lock(&g_mu);
    int slot = -1;
    for (int i = 0; i < SPB_L1_MAX_MODELS; i++)
        if (g_models[i].qm == qm_opaque) {
            if (g_models[i].fp == fp) { m = g_models[i].m; slot = i; break; }
            /* another model now lives at this address: drop the stale device copy */
            spb_kvpool_free(g_models[i].pool);
            spb_model_free(g_models[i].m);
            g_models[i].qm = NULL;
            g_models[i].m = NULL;
            g_models[i].pool = NULL;
        }
    if (!m) {
        for (int i = 0; i < SPB_L1_MAX_MODELS; i++)
            if (!g_models[i].qm) { slot = i; break; }
        if (slot < 0) sp_set_error("spb200: too many resident models");
        else if ((m = upload((const qwen3_model *)qm_opaque)) != NULL) {
            g_models[slot].qm = qm_opaque;
            g_models[slot].fp = fp;
            g_models[slot].m = m;
            g_models[slot].pool = NULL;
            if (g_pool_pg > 0 && spb_kvpool_create(m, g_pool_pg, g_pool_pages, &g_models[slot].pool) != SPB_OK) {
                fail("kv pool");
                spb_model_free(m);
                g_models[slot].qm = NULL;
                g_models[slot].m = m = NULL;
            }
        }
    }
    if (m && pool) *pool = g_models[slot].pool;
    pthread_mutex_unlock(&g_mu);
    return m;
}

int spb_l1_set_kv_pool(int page_positions, int n_pages) {
    if (page_positions < 0 || n_pages < 0 || (page_positions > 0 && (page_positions % 128 || n_pages == 0)))
        return SPB_EBADARG;
    g_pool_pg = page_positions;
    g_pool_pages = n_pages;
    return SPB_OK;
}

int spb_l1_set_device(int device) {
    if (device < 0) return SPB_EBADARG;
    g_device = device;
    return SPB_OK;
}

void spb_l1_release_model(const void *qm_opaque) {
    pthread_mutex_lock(&g_mu);
    for (int i = 0; i < SPB_L1_MAX_MODELS; i++)
        if (g_models[i].qm == qm_opaque) {
            spb_kvpool_free(g_models[i].pool);
            spb_model_free(g_models[i].m);
            g_models[i].qm = NULL;
            g_models[i].m = NULL;
            g_models[i].pool = NULL;
        }
    pthread_mutex_unlock(&g_mu);
}

void *spb_l1_backend(void) { return &g_backend_tag; }

/* K/V kept as Spinor blocks (SPB_KV_SPINOR) for caches opened after this call; the engine-side
 * counterpart of the reference's SP_KV_SPINOR session flag (sp_l1.h:156), which the frozen
 * section-6b open row cannot carry. Unpaged caches only (a page pool takes precedence). */
int spb_l1_set_kv_flags(unsigned flags) {
    if (flags & ~(unsigned)SPB_KV_SPINOR) { sp_set_error("spb200: set_kv_flags: unknown flags"); return 1; }
    __atomic_store_n(&g_kv_flags, flags, __ATOMIC_RELAXED);
    return 0;
}

int spb_l1_forward(void *handle, const void *qm_opaque, const int32_t *tokens, int n_tok, float *logits) {
    (void)handle;
    spb_model *m = model_for(qm_opaque, NULL);
    if (!m) return 1;
    if (spb_forward(m, tokens, n_tok, logits) != SPB_OK) return fail("forward");
    return 0;
}

/* ---- section-6b table ---- */
static int kv_open(const void *qm_opaque, int pmax, sp_kvdecode_handle **out) {
    if (!out) { sp_set_error("spb200: open: null out"); return 1; }
    *out = NULL;
    spb_kvpool *pool = NULL;
    spb_model *m = model_for(qm_opaque, &pool);
    if (!m) return 1;
    spb_session *s = NULL;
    const unsigned flags = __atomic_load_n(&g_kv_flags, __ATOMIC_RELAXED);
    const int rc = pool ? spb_session_open_paged(pool, pmax, &s) : spb_session_open_ex(m, pmax, flags, &s);
    if (rc != SPB_OK) return fail("open");
    *out = (sp_kvdecode_handle *)s;
    return 0;
}

static int kv_prefill(sp_kvdecode_handle *h, const int32_t *tokens, int n_tok) {
    if (spb_session_prefill((spb_session *)h, tokens, n_tok, NULL) != SPB_OK) return fail("prefill");
    return 0;
}

static int kv_decode_step(sp_kvdecode_handle *h, int32_t token, float *logits) {
    if (spb_session_decode_step((spb_session *)h, token, logits) != SPB_OK) return fail("decode_step");
    return 0;
}

static int kv_rewind(sp_kvdecode_handle *h, int n) {
    if (spb_session_rewind((spb_session *)h, n) != SPB_OK) return fail("rewind");
    return 0;
}

static int kv_position(const sp_kvdecode_handle *h) {
    return h ? spb_session_position((const spb_session *)h) : -1;
}

static void kv_close(sp_kvdecode_handle *h) { spb_session_close((spb_session *)h); }

int spb_l1_kvdecode_clone(const struct sp_kvdecode_handle *h, struct sp_kvdecode_handle **out) {
    spb_session *c = NULL;
    if (!h || !out) { sp_set_error("spb200: clone: null arg"); return 1; }
    if (spb_session_clone((const spb_session *)h, &c) != SPB_OK) return fail("clone");
    *out = (sp_kvdecode_handle *)c;
    return 0;
}

/* the frozen six rows (sp_l1.h:403-410) followed by the appended clone row */
static const struct spb_kvdecode_dispatch_ext g_table = {
    {kv_open, kv_prefill, kv_decode_step, kv_rewind, kv_position, kv_close}, spb_l1_kvdecode_clone};

const struct sp_kvdecode_dispatch_fn *spb_l1_kvdecode_table(void) { return &g_table.base; }
const struct spb_kvdecode_dispatch_ext *spb_l1_kvdecode_table_ext(void) { return &g_table; }
