/* xref_forward.c -- the XREF exact-integer forward (checker; test infrastructure).
 *
 * Orchestration restated from the reference's per-token decode paths:
 *   Gemma3: kv_step_gemma3 (sp_session.c:380-464) / gemma3_forward (gemma3.c:39-148)
 *     embed * sqrtf(E) -> per layer [attn_norm -> Q,K,V -> QK-norm -> RoPE (global
 *     layers base=rope_base, local base=rope_base_local) -> attention (local layers:
 *     sliding window, s0 = pos - win + 1, forward_kernels.c:62) -> O -> sandwich
 *     post_attn_norm + residual -> ffn_norm -> GeGLU (gelu(gate) * up) -> down ->
 *     post_ffw_norm + residual] -> output_norm -> LM head (tied to token_embd).
 *     Layer L is global iff L % 6 == 5 (gemma3.c:79, sp_session.c:396).
 *   Qwen3: kv_step (sp_session.c:274-363): no embedding scale, plain residuals,
 *     SwiGLU (silu(gate) * up), QK-norm, full causal attention, untied LM head.
 * with every float island replaced by its exact-integer rule:
 *   RMSNorm -> xref_rmsnorm_exact; matvec -> xref_matvec (int64 block-scale
 *   accumulation); RoPE -> CORDIC; attention score -> exact int64 <q,k> on the 2^16
 *   grid (forward.c:232-246 convention); softmax -> island integer exponentials;
 *   V-sum -> exact integer sum of e_t * v_t (128-bit) with one floor division;
 *   GELU/SiLU -> islands.
 * The residual adds, the sqrtf(E) embedding scale and gate*up stay single IEEE f32
 * ops (compiled with -ffp-contract=off).
 *
 * Prefill is defined as sequential decode over the tokens (position t sees
 * positions [0, t]); every position's logits are produced, as the reference's
 * section-6 forward hook requires (sp_l1.h:312-318).
 */
#include "xref.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#define ONE (INT64_C(1) << 30)
typedef __int128 i128;

struct xref_session {
    const xref_model *m;
    int max_ctx, pos;
    int32_t *kc, *vc;          /* [n_layers][max_ctx][n_head_kv*head_dim], 2^16 grid */
    unsigned flags;            /* XREF_KV_SPINOR: the rows above are the decoded Spinor blocks */
    uint8_t *kb, *vb;          /* spinor: [n_layers][max_ctx][n_head_kv][nblk * 63] */
    uint64_t *wg, *wl;         /* RoPE turn tables, [head_dim/2] */
    float *x, *nx, *q, *k, *v, *ao, *ap, *g, *u, *dn, *t;
    int32_t *qi;
};

static int rms_ok(const float *x, int n) {
    i128 ss = 0;
    for (int i = 0; i < n; i++) {
        if (!(fabsf(x[i]) < 32768.0f)) return 0;
        int64_t xi = xref_llround((double)x[i] * 65536.0);
        ss += (i128)xi * xi;
    }
    return ss < ((i128)1 << 63);
}

static int act_ok(const float *x, int n) {
    for (int i = 0; i < n; i++) if (!(fabsf(x[i]) < 2048.0f)) return 0;
    return 1;
}

/* floor(a / b), b > 0 */
static int64_t floordiv128(i128 a, int64_t b) {
    i128 q = a / b;
    if ((a % b) != 0 && a < 0) q -= 1;
    return (int64_t)q;
}

int xref_attn_head(const int32_t *q, const int32_t *K, const int32_t *V, int stride,
                   int s0, int pos, int hd, float ascale, float *out) {
    const int m = pos - s0 + 1;
    int64_t *zi = (int64_t *)malloc((size_t)m * sizeof(int64_t));
    if (!zi) return XREF_ENOMEM;
    int64_t mx = INT64_MIN;
    int rc = XREF_OK;
    for (int t = s0; t <= pos; t++) {
        const int32_t *kt = K + (size_t)t * stride;
        int64_t s = 0;
        for (int i = 0; i < hd; i++) s += (int64_t)q[i] * (int64_t)kt[i];
        float z = (float)((double)s / 4294967296.0) * ascale;
        if (!(fabsf(z) < 131072.0f)) { rc = XREF_ERANGE; z = 0.0f; }
        int64_t v = xref_llround((double)z * 16384.0);
        zi[t - s0] = v;
        if (v > mx) mx = v;
    }
    int64_t S = 0;
    for (int t = 0; t < m; t++) {
        zi[t] = xref_exp_fixed(((zi[t] - mx) * ONE) >> 14);
        S += zi[t];
    }
    for (int d = 0; d < hd; d++) {
        i128 N = 0;
        for (int t = s0; t <= pos; t++) N += (i128)zi[t - s0] * V[(size_t)t * stride + d];
        int64_t qd = floordiv128(N * 65536, S);
        out[d] = (float)((double)qd * 0x1p-32);
    }
    free(zi);
    return rc;
}

static size_t spin_row_bytes(const xref_config *c) {
    return (size_t)c->n_head_kv * (size_t)xref_spinor_blocks_for(c->head_dim) * XREF_SPINOR_BYTES;
}

int xref_session_create(const xref_model *m, int max_ctx, xref_session **out) {
    return xref_session_create_ex(m, max_ctx, 0u, out);
}

int xref_session_create_ex(const xref_model *m, int max_ctx, unsigned flags, xref_session **out) {
    if (!m || !out || max_ctx <= 0 || (flags & ~XREF_KV_SPINOR)) return XREF_EBADARG;
    const xref_config *c = &m->cfg;
    const int E = c->n_embd, HD = c->head_dim, KVD = c->n_head_kv * HD, QD = c->n_head * HD;
    const int FF = c->n_ff;
    if (c->n_head % c->n_head_kv) return XREF_EBADARG;
    xref_session *s = (xref_session *)calloc(1, sizeof *s);
    if (!s) return XREF_ENOMEM;
    s->m = m; s->max_ctx = max_ctx; s->flags = flags;
    if (flags & XREF_KV_SPINOR) {
        const size_t nb = (size_t)c->n_layers * (size_t)max_ctx * spin_row_bytes(c);
        s->kb = (uint8_t *)calloc(nb, 1);
        s->vb = (uint8_t *)calloc(nb, 1);
        if (!s->kb || !s->vb) { xref_session_destroy(s); return XREF_ENOMEM; }
    }
    size_t kvn = (size_t)c->n_layers * (size_t)max_ctx * (size_t)KVD;
    s->kc = (int32_t *)calloc(kvn, sizeof(int32_t));
    s->vc = (int32_t *)calloc(kvn, sizeof(int32_t));
    s->wg = (uint64_t *)malloc((size_t)HD / 2 * sizeof(uint64_t));
    s->wl = (uint64_t *)malloc((size_t)HD / 2 * sizeof(uint64_t));
    int big = E > FF ? E : FF; if (QD > big) big = QD;
    s->x = malloc((size_t)E * 4); s->nx = malloc((size_t)big * 4); s->q = malloc((size_t)QD * 4);
    s->k = malloc((size_t)KVD * 4); s->v = malloc((size_t)KVD * 4); s->ao = malloc((size_t)QD * 4);
    s->ap = malloc((size_t)E * 4); s->g = malloc((size_t)FF * 4); s->u = malloc((size_t)FF * 4);
    s->dn = malloc((size_t)E * 4); s->t = malloc((size_t)big * 4);
    s->qi = malloc((size_t)QD * 4);
    if (!s->kc || !s->vc || !s->wg || !s->wl || !s->x || !s->nx || !s->q || !s->k || !s->v ||
        !s->ao || !s->ap || !s->g || !s->u || !s->dn || !s->t || !s->qi) {
        xref_session_destroy(s); return XREF_ENOMEM;
    }
    if (xref_rope_freq_table(c->rope_base, HD, s->wg) ||
        xref_rope_freq_table(c->arch == XREF_ARCH_GEMMA3 ? c->rope_base_local : c->rope_base, HD, s->wl)) {
        xref_session_destroy(s); return XREF_EBADARG;
    }
    *out = s;
    return XREF_OK;
}

void xref_session_destroy(xref_session *s) {
    if (!s) return;
    free(s->kc); free(s->vc); free(s->kb); free(s->vb); free(s->wg); free(s->wl);
    free(s->x); free(s->nx); free(s->q); free(s->k); free(s->v); free(s->ao); free(s->ap);
    free(s->g); free(s->u); free(s->dn); free(s->t); free(s->qi);
    free(s);
}

#define CHK(e) do { int rc_ = (e); if (rc_) return rc_; } while (0)

static int norm(const float *x, const float *w, int n, float *out) {
    if (!rms_ok(x, n)) return XREF_ERANGE;
    for (int i = 0; i < n; i++) if (!(fabsf(w[i]) < 32768.0f)) return XREF_ERANGE;
    xref_rmsnorm_exact(x, w, n, out);
    return XREF_OK;
}

int xref_decode_step(xref_session *s, int32_t tok, float *logits) {
    const xref_model *m = s->m;
    const xref_config *c = &m->cfg;
    const int E = c->n_embd, FF = c->n_ff, HD = c->head_dim, NH = c->n_head, NKV = c->n_head_kv;
    const int KVD = NKV * HD, group = NH / NKV, P = s->max_ctx;
    const int gem = c->arch == XREF_ARCH_GEMMA3;
    const int pos = s->pos;
    const float ascale = 1.0f / sqrtf((float)HD);
    if (pos >= P) return XREF_EBADARG;
    if (tok < 0 || tok >= c->n_vocab) return XREF_EBADARG;

    xref_dequant_row(&m->token_embd, tok, s->x);
    if (gem) { const float es = sqrtf((float)E); for (int i = 0; i < E; i++) s->x[i] = s->x[i] * es; }

    for (int L = 0; L < c->n_layers; L++) {
        const xref_layer *ly = &m->layers[L];
        const int period = c->swa_period > 0 ? c->swa_period : 6;
        const int global = !gem || (L % period) == period - 1;
        const uint64_t *W = global ? s->wg : s->wl;
        const int win = (gem && !global && c->sliding_window > 0) ? c->sliding_window : -1;

        CHK(norm(s->x, ly->attn_norm, E, s->nx));
        CHK(xref_matvec(&ly->wq, s->nx, 1, s->q));
        CHK(xref_matvec(&ly->wk, s->nx, 1, s->k));
        CHK(xref_matvec(&ly->wv, s->nx, 1, s->v));

        int32_t *kcl = s->kc + (size_t)L * P * KVD, *vcl = s->vc + (size_t)L * P * KVD;
        for (int h = 0; h < NH; h++) {
            float *qh = s->q + (size_t)h * HD;
            if (c->has_qk_norm) { CHK(norm(qh, ly->q_norm, HD, s->t)); memcpy(qh, s->t, (size_t)HD * 4); }
            CHK(xref_rope_cordic(qh, HD, pos, W, s->qi + (size_t)h * HD));
        }
        for (int h = 0; h < NKV; h++) {
            float *kh = s->k + (size_t)h * HD;
            if (c->has_qk_norm) { CHK(norm(kh, ly->k_norm, HD, s->t)); memcpy(kh, s->t, (size_t)HD * 4); }
            CHK(xref_rope_cordic(kh, HD, pos, W, kcl + (size_t)pos * KVD + (size_t)h * HD));
        }
        if (s->flags & XREF_KV_SPINOR) {   /* K/V rows through the Spinor codec (sp_session.c:298-313) */
            const size_t rbh = (size_t)xref_spinor_blocks_for(HD) * XREF_SPINOR_BYTES, rb = spin_row_bytes(c);
            uint8_t *kb = s->kb + ((size_t)L * P + pos) * rb, *vb = s->vb + ((size_t)L * P + pos) * rb;
            for (int h = 0; h < NKV; h++) {
                int32_t *kr = kcl + (size_t)pos * KVD + (size_t)h * HD;
                CHK(xref_spinor_kv_row(kr, NULL, HD, kb + h * rbh, kr));
                CHK(xref_spinor_kv_row(NULL, s->v + (size_t)h * HD, HD, vb + h * rbh,
                                       vcl + (size_t)pos * KVD + (size_t)h * HD));
            }
        } else {
            for (int i = 0; i < KVD; i++) {
                if (!(fabsf(s->v[i]) < 16384.0f)) return XREF_ERANGE;
                vcl[(size_t)pos * KVD + i] = (int32_t)lrintf(s->v[i] * 65536.0f);
            }
        }
        for (int h = 0; h < NH; h++) {
            const int g = h / group;
            const int s0 = (win >= 0 && pos - win + 1 > 0) ? pos - win + 1 : 0;
            CHK(xref_attn_head(s->qi + (size_t)h * HD, kcl + (size_t)g * HD, vcl + (size_t)g * HD,
                               KVD, s0, pos, HD, ascale, s->ao + (size_t)h * HD));
        }
        CHK(xref_matvec(&ly->wo, s->ao, 1, s->ap));
        if (gem) {
            CHK(norm(s->ap, ly->post_attn_norm, E, s->t));
            for (int i = 0; i < E; i++) s->x[i] = s->x[i] + s->t[i];
        } else {
            for (int i = 0; i < E; i++) s->x[i] = s->x[i] + s->ap[i];
        }

        CHK(norm(s->x, ly->ffn_norm, E, s->nx));
        CHK(xref_matvec(&ly->wg, s->nx, 1, s->g));
        CHK(xref_matvec(&ly->wu, s->nx, 1, s->u));
        if (!act_ok(s->g, FF)) return XREF_ERANGE;
        if (gem) xref_gelu_exact(s->g, FF, s->t); else xref_silu_exact(s->g, FF, s->t);
        for (int i = 0; i < FF; i++) s->g[i] = s->t[i] * s->u[i];
        CHK(xref_matvec(&ly->wd, s->g, 1, s->dn));
        if (gem) {
            CHK(norm(s->dn, ly->post_ffw_norm, E, s->t));
            for (int i = 0; i < E; i++) s->x[i] = s->x[i] + s->t[i];
        } else {
            for (int i = 0; i < E; i++) s->x[i] = s->x[i] + s->dn[i];
        }
    }
    if (logits) {
        CHK(norm(s->x, m->output_norm, E, s->nx));
        CHK(xref_matvec(&m->output, s->nx, 1, logits));
    }
    s->pos = pos + 1;
    return XREF_OK;
}

int xref_prefill(xref_session *s, const int32_t *tokens, int n, float *logits) {
    const int V = s->m->cfg.n_vocab;
    for (int i = 0; i < n; i++)
        CHK(xref_decode_step(s, tokens[i], logits ? logits + (size_t)i * V : NULL));
    return XREF_OK;
}

int xref_rewind(xref_session *s, int n) {
    if (n < 0 || n > s->pos) return XREF_EBADARG;
    s->pos -= n;
    return XREF_OK;
}

int xref_position(const xref_session *s) { return s ? s->pos : -1; }

int xref_clone(const xref_session *s, xref_session **out) {
    CHK(xref_session_create_ex(s->m, s->max_ctx, s->flags, out));
    const xref_config *c = &s->m->cfg;
    size_t kvn = (size_t)c->n_layers * (size_t)s->max_ctx * (size_t)(c->n_head_kv * c->head_dim);
    memcpy((*out)->kc, s->kc, kvn * sizeof(int32_t));
    memcpy((*out)->vc, s->vc, kvn * sizeof(int32_t));
    if (s->flags & XREF_KV_SPINOR) {
        const size_t nb = (size_t)c->n_layers * (size_t)s->max_ctx * spin_row_bytes(c);
        memcpy((*out)->kb, s->kb, nb);
        memcpy((*out)->vb, s->vb, nb);
    }
    (*out)->pos = s->pos;
    return XREF_OK;
}

int xref_kv_read(const xref_session *s, int layer, int pos, int which, int32_t *out) {
    const xref_config *c = &s->m->cfg;
    const int KVD = c->n_head_kv * c->head_dim;
    if (layer < 0 || layer >= c->n_layers || pos < 0 || pos >= s->max_ctx) return XREF_EBADARG;
    const int32_t *src = (which ? s->vc : s->kc) + ((size_t)layer * s->max_ctx + pos) * KVD;
    memcpy(out, src, (size_t)KVD * sizeof(int32_t));
    return XREF_OK;
}

int xref_kv_bytes(const xref_session *s, int layer, int pos, int which, uint8_t *out) {
    const xref_config *c = &s->m->cfg;
    if (!(s->flags & XREF_KV_SPINOR) || layer < 0 || layer >= c->n_layers || pos < 0 || pos >= s->max_ctx)
        return XREF_EBADARG;
    const size_t rb = spin_row_bytes(c);
    memcpy(out, (which ? s->vb : s->kb) + ((size_t)layer * s->max_ctx + pos) * rb, rb);
    return XREF_OK;
}
