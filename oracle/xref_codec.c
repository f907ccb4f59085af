/* xref_codec.c -- OK_Q4B codec + exact-integer matvec (checker; test infrastructure).
 *
 * Restates:
 *   - f16 -> f32                      weight_dtype.c:9-28
 *   - 4-bit nibble unpack             frobenius_lift.c:102-107 (low nibble = even col,
 *                                     two's-complement sign extension)
 *   - OK_Q4B row dequant              frobenius_lift.c:200-209 (w = code * f16(bscale))
 *   - activation quantizer quant1     frobenius_lift.c:27-35 (v/s*127, round half away,
 *                                     clamp +-127)
 * and defines the exact matvec that replaces matmul_arena's Q4B branch
 * (forward_dispatch.c:69-86):
 *   isum_jb = sum_{i in block b} code_ji * q_i             (int32, |isum| < 2^15)
 *   k_jb    = f16 block scale as an integer, value = k * 2^-24  (|k| < 2^40)
 *   acc_j   = sum_b k_jb * isum_jb                         (int64, exact; bound checked)
 *   y_j     = (float)((double)acc_j * (((double)s / 127.0) * 2^-24))
 * where s is the activation row's max |u| and q its quant1 codes.
 */
#include "xref.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

float xref_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) & 1u;
    uint32_t e = (h >> 10) & 0x1Fu, m = h & 0x3FFu;
    float v;
    if (e == 0)        v = ldexpf((float)m, -24);              /* subnormal/zero: m * 2^-24 */
    else if (e == 31)  v = m ? NAN : INFINITY;
    else               v = ldexpf((float)(1024u + m), (int)e - 25);
    return sign ? -v : v;
}

int xref_f16_to_k(uint16_t h, int64_t *k) {
    uint32_t sign = (uint32_t)(h >> 15) & 1u;
    uint32_t e = (h >> 10) & 0x1Fu, m = h & 0x3FFu;
    int64_t v;
    if (e == 31) return -1;
    if (e == 0) v = (int64_t)m;
    else        v = (int64_t)(1024u + m) << (e - 1u);
    *k = sign ? -v : v;
    return 0;
}

int8_t xref_quant1(float v, float scale) {
    if (scale == 0.0f) return 0;
    float x = v / scale * 127.0f;
    float r = (x >= 0.0f) ? floorf(x + 0.5f) : ceilf(x - 0.5f);
    if (r > 127.0f) r = 127.0f;
    if (r < -127.0f) r = -127.0f;
    return (int8_t)r;
}

void xref_unpack_q4(const uint8_t *nib, int n, int8_t *codes) {
    for (int i = 0; i < n; i++) {
        unsigned b = (i & 1) ? (unsigned)(nib[i >> 1] >> 4) : (unsigned)(nib[i >> 1] & 0xF);
        codes[i] = (int8_t)(b >= 8 ? (int)b - 16 : (int)b);
    }
}

void xref_dequant_row(const xref_q4b *w, int r, float *dst) {
    const int nib = (w->cols + 1) / 2, nblk = (w->cols + 31) / 32;
    const uint8_t *rc = w->codes + (size_t)r * (size_t)nib;
    const uint16_t *bs = w->bscale + (size_t)r * (size_t)nblk;
    for (int i = 0; i < w->cols; i++) {
        unsigned b = (i & 1) ? (unsigned)(rc[i >> 1] >> 4) : (unsigned)(rc[i >> 1] & 0xF);
        int c = b >= 8 ? (int)b - 16 : (int)b;
        dst[i] = (float)c * xref_f16_to_f32(bs[i >> 5]);
    }
}

/* The int64 accumulator of one row is exact when sum_b |k_jb| * 32 * 8 * 127 < 2^63. */
int xref_q4b_check(const xref_q4b *w) {
    const int nblk = (w->cols + 31) / 32;
    const uint64_t lim = (UINT64_C(1) << 63) / (32u * 8u * 127u);
    for (int r = 0; r < w->rows; r++) {
        uint64_t sum = 0;
        for (int b = 0; b < nblk; b++) {
            int64_t k;
            if (xref_f16_to_k(w->bscale[(size_t)r * nblk + b], &k)) return -1;
            sum += (uint64_t)(k < 0 ? -k : k);
            if (sum >= lim) return -1;
        }
    }
    return 0;
}

void xref_quant_vec(const float *u, int n, int8_t *q, float *s) {
    float m = 0.0f;
    for (int i = 0; i < n; i++) { float a = fabsf(u[i]); if (a > m) m = a; }
    for (int i = 0; i < n; i++) q[i] = xref_quant1(u[i], m);
    *s = m;
}

/* Rows are independent, so large matvecs are split over host threads (XREF_THREADS, default the
 * online cores, at most 64); every output is the same integer whatever the split. */
typedef struct {
    const xref_q4b *w; const int8_t *q; const float *s; int n_tok; float *Y; int r0, r1;
} mv_part;

static void *matvec_rows(void *arg) {
    const mv_part *p = (const mv_part *)arg;
    const xref_q4b *w = p->w;
    const int K = w->cols, nib = (K + 1) / 2, nblk = (K + 31) / 32;
    int8_t *c = (int8_t *)malloc((size_t)K);
    int64_t *kk = (int64_t *)malloc((size_t)nblk * sizeof(int64_t));
    if (c && kk) {
        for (int j = p->r0; j < p->r1; j++) {
            xref_unpack_q4(w->codes + (size_t)j * nib, K, c);
            for (int b = 0; b < nblk; b++) (void)xref_f16_to_k(w->bscale[(size_t)j * nblk + b], &kk[b]);
            for (int t = 0; t < p->n_tok; t++) {
                const int8_t *x = p->q + (size_t)t * K;
                int64_t acc = 0;
                for (int b = 0; b < nblk; b++) {
                    int i0 = b * 32, i1 = i0 + 32 < K ? i0 + 32 : K;
                    int32_t isum = 0;
                    for (int i = i0; i < i1; i++) isum += (int32_t)c[i] * (int32_t)x[i];
                    acc += kk[b] * (int64_t)isum;
                }
                double dsc = ((double)p->s[t] / 127.0) * 0x1p-24;
                p->Y[(size_t)t * w->rows + j] = (float)((double)acc * dsc);
            }
        }
    }
    free(c); free(kk);
    return NULL;
}

static int mv_threads(void) {
    static int n = 0;
    if (!n) {
        const char *e = getenv("XREF_THREADS");
        long v = e ? strtol(e, NULL, 10) : sysconf(_SC_NPROCESSORS_ONLN);
        n = v < 1 ? 1 : v > 64 ? 64 : (int)v;
    }
    return n;
}

void xref_matvec_q(const xref_q4b *w, const int8_t *q, const float *s, int n_tok, float *Y) {
    int nt = mv_threads();
    if ((int64_t)w->rows * w->cols * n_tok < (INT64_C(1) << 22)) nt = 1;
    if (nt > w->rows) nt = w->rows;
    mv_part parts[64];
    pthread_t th[64];
    int started[64] = {0};
    for (int i = 0; i < nt; i++) {
        parts[i] = (mv_part){w, q, s, n_tok, Y, (int)((int64_t)w->rows * i / nt),
                             (int)((int64_t)w->rows * (i + 1) / nt)};
        if (i > 0) started[i] = pthread_create(&th[i], NULL, matvec_rows, &parts[i]) == 0;
    }
    matvec_rows(&parts[0]);
    for (int i = 1; i < nt; i++) {
        if (started[i]) pthread_join(th[i], NULL);
        else matvec_rows(&parts[i]);   /* no thread: this caller does the part */
    }
}

int xref_matvec(const xref_q4b *w, const float *X, int n_tok, float *Y) {
    const int K = w->cols;
    int8_t *q = (int8_t *)malloc((size_t)n_tok * K);
    float *s = (float *)malloc((size_t)n_tok * sizeof(float));
    if (!q || !s) { free(q); free(s); return XREF_ENOMEM; }
    for (int t = 0; t < n_tok; t++) {
        const float *u = X + (size_t)t * K;
        for (int i = 0; i < K; i++) if (!isfinite(u[i])) { free(q); free(s); return XREF_ERANGE; }
        xref_quant_vec(u, K, q + (size_t)t * K, &s[t]);
    }
    xref_matvec_q(w, q, s, n_tok, Y);
    free(q); free(s);
    return XREF_OK;
}

int xref_argmax(const float *v, int n) {
    int best = 0;
    for (int i = 1; i < n; i++) if (v[i] > v[best]) best = i;
    return best;
}
