/* xref_islands.c -- exact-integer islands (checker; test infrastructure).
 *
 * A C restatement of the reference's exact islands (exact_islands.c), used by the
 * XREF forward and pinned against the reference's own compiled islands and the
 * golden vectors under tests/golden/. Fixed-point layout (exact_islands.h:16-19):
 *   RMSNorm Q=16 input, IB=20 inverse-rms, Qw=16 weight; softmax Z=2^14 grid;
 *   GELU Z=2^16 grid; exp/tanh in FB=30 fixed point.
 * Signed right shifts are arithmetic (floor), as the reference relies on
 * (exact_islands.c:7-12). 128-bit products use unsigned __int128 wrapping so that
 * the truncation to int64 matches the reference's (int64_t) casts bit for bit.
 *
 * Builder-defined (no reference code): exact SiLU on the same exp primitive.
 */
#include "xref.h"

#include <math.h>

#define FB 30
#define ONE (INT64_C(1) << FB)

typedef __int128 i128;

/* round(log2(e) * 2^30) and round((ln 2)^k / k! * 2^30), k = 0..6 (exact_islands.c:21-27) */
static const int64_t K_LOG2E = INT64_C(1549082005);
static const int64_t K_EXP2[7] = {
    INT64_C(1073741824), INT64_C(744261118), INT64_C(257941248), INT64_C(59597083),
    INT64_C(10327387),   INT64_C(1431680),   INT64_C(165394)
};
/* round(sqrt(2/pi) * 2^30), round(0.044715 * 2^30) (exact_islands.c:100-101) */
static const int64_t K_GELU_K = INT64_C(856722024);
static const int64_t K_GELU_A = INT64_C(48012366);

int64_t xref_llround(double v) { return (int64_t)llround(v); }

/* floor((a*b) / 2^FB) truncated to int64, a and b any int64 (exact_islands.c uses
 * ((__int128)a*b) >> FB followed by an (int64_t) cast). */
static int64_t mulshr(int64_t a, int64_t b) {
    i128 p = (i128)a * (i128)b;
    return (int64_t)(p >> FB);
}

/* 2^(r/2^FB) for r in [0, ONE]: degree-6 Horner in FB fixed point (exact_islands.c:30-34) */
static int64_t exp2_frac(int64_t r) {
    int64_t acc = K_EXP2[6];
    for (int k = 5; k >= 0; k--) acc = ((acc * r) >> FB) + K_EXP2[k];
    return acc;
}

/* e^(d/2^FB) for d <= 0, FB fixed point (exact_islands.c:38-45) */
int64_t xref_exp_fixed(int64_t d) {
    int64_t g = -mulshr(d, K_LOG2E);             /* -d*log2(e) >= 0 */
    int64_t n = g >> FB, r = g - (n << FB);
    if (n >= 32) return 0;
    if (r != 0) return exp2_frac(ONE - r) >> (n + 1);
    return ONE >> n;
}

/* floor(sqrt(v)) (exact_islands.c:49-58 computes the same integer) */
static uint64_t isqrt64(uint64_t v) {
    uint64_t res = 0, bit = UINT64_C(1) << 62;
    while (bit > v) bit >>= 2;
    while (bit) {
        if (v >= res + bit) { v -= res + bit; res = (res >> 1) + bit; }
        else res >>= 1;
        bit >>= 2;
    }
    return res;
}

/* Island 1, exact_islands.c:60-79: out_i = x_i * sqrt(n / sum x^2) * w_i with
 * xi = llround(x_i * 2^16), inv = isqrt(floor(n * 2^72 / sum xi^2)) (the quotient
 * truncated to 64 bits as the reference's uint64_t cast does), and
 * out_i = (float)((double)(int64)(xi*inv*wi) / 2^52). */
void xref_rmsnorm_exact(const float *x, const float *w, int n, float *out) {
    int64_t ss = 0;
    for (int i = 0; i < n; i++) {
        int64_t xi = xref_llround((double)x[i] * 65536.0);
        ss += xi * xi;
    }
    if (ss == 0) { for (int i = 0; i < n; i++) out[i] = 0.0f; return; }
    unsigned __int128 num = (unsigned __int128)(uint64_t)n << 72;
    uint64_t q = (uint64_t)(num / (unsigned __int128)(uint64_t)ss);
    uint64_t inv = isqrt64(q);
    for (int i = 0; i < n; i++) {
        int64_t xi = xref_llround((double)x[i] * 65536.0);
        int64_t wi = xref_llround((double)w[i] * 65536.0);
        int64_t yi = (int64_t)((uint64_t)xi * inv * (uint64_t)wi);
        out[i] = (float)((double)yi / 4503599627370496.0);   /* 2^52 */
    }
}

/* Island 2, exact_islands.c:82-97 */
void xref_softmax_exact(const float *z, int m, double *p) {
    int64_t mx = INT64_MIN, S = 0;
    for (int i = 0; i < m; i++) {
        int64_t zi = xref_llround((double)z[i] * 16384.0);
        if (zi > mx) mx = zi;
    }
    for (int i = 0; i < m; i++) {
        int64_t zi = xref_llround((double)z[i] * 16384.0);
        int64_t e = xref_exp_fixed(((zi - mx) * ONE) >> 14);
        p[i] = (double)e;
        S += e;
    }
    for (int i = 0; i < m; i++) p[i] /= (double)S;
}

/* tanh(t), FB fixed point, via the exp primitive (exact_islands.c:104-110) */
static int64_t tanh_fixed(int64_t t) {
    int64_t a = t >= 0 ? t : -t;
    int64_t e2 = xref_exp_fixed(-(2 * a));
    int64_t th = ONE - ((2 * e2) << FB) / (ONE + e2);
    return t >= 0 ? th : -th;
}

/* Island 3, exact_islands.c:112-124: 0.5*x*(1+tanh(sqrt(2/pi)*(x+0.044715x^3))) */
void xref_gelu_exact(const float *x, int n, float *out) {
    for (int i = 0; i < n; i++) {
        int64_t xq = xref_llround((double)x[i] * 65536.0);
        int64_t X = (xq * ONE) >> 16;
        int64_t X2 = mulshr(X, X);
        int64_t X3 = mulshr(X2, X);
        int64_t inner = mulshr(K_GELU_K, X + mulshr(K_GELU_A, X3));
        int64_t t = tanh_fixed(inner);
        int64_t g = mulshr(X >> 1, ONE + t);
        out[i] = (float)((double)g / 1073741824.0);          /* 2^30 */
    }
}

/* Exact SiLU (builder-defined; no reference island exists -- forward.c:269-273 and
 * sp_session.c:354 use float expf). Same Z=2^16 input grid and FB=30 exp primitive
 * as the GELU island:
 *   X   = llround(x * 2^16) * 2^14
 *   sig = X >= 0 ? floor(2^60 / (ONE + e^-X)) : floor(e^X * ONE / (ONE + e^X))
 *   out = (float)((double)floor(X * sig / 2^30) / 2^30)
 */
void xref_silu_exact(const float *x, int n, float *out) {
    for (int i = 0; i < n; i++) {
        int64_t xq = xref_llround((double)x[i] * 65536.0);
        int64_t X = (xq * ONE) >> 16;
        int64_t sig;
        if (X >= 0) {
            int64_t e = xref_exp_fixed(-X);
            sig = (ONE << FB) / (ONE + e);
        } else {
            int64_t e = xref_exp_fixed(X);
            sig = (e << FB) / (ONE + e);
        }
        int64_t g = mulshr(X, sig);
        out[i] = (float)((double)g / 1073741824.0);
    }
}
