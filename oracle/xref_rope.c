/* xref_rope.c -- CORDIC-RoPE (checker; test infrastructure).
 *
 * The reference claims a CORDIC-RoPE island but has no code for it; its RoPE is
 * float NEOX (forward_kernels.c:31-41: pairs (i, i+d/2) rotated counter-clockwise by
 * p * base^(-2i/d) with powf/cosf/sinf). This file defines the exact replacement
 * (builder-defined; method: J. E. Volder, "The CORDIC Trigonometric Computing
 * Technique", 1959), using integer arithmetic only -- no libm anywhere:
 *
 *   angles are in TURNS as unsigned Q64 (a full turn == 2^64), so "mod 2*pi" is
 *   plain 64-bit wraparound;
 *   W_i  = round(base^(-2i/d) / (2*pi) * 2^64)   turns per position (table, integer
 *          algorithms: bit-by-bit log2, a 2^(-2^-j) square-root ladder, pi from
 *          Machin's formula with an integer arctan series);
 *   phi  = p * W_i  (mod 2^64);
 *   A,B  = llround(a * 2^30), llround(b * 2^30)       (|a|,|b| < 2^8)
 *   quadrant: phi + 1/8 turn, top 2 bits pick a multiple of 90 degrees (exact swap/
 *   negate), residual z in [-1/8, 1/8) turn;
 *   30 CORDIC micro-rotations X -= d*(Y>>k), Y += d*(X>>k), z -= d*T_k with
 *   T_k = round(atan(2^-k) / (2*pi) * 2^64) (T_0 = 2^61 exactly);
 *   out = floor((X * G + 2^75) / 2^76) with G = round(2^62 / prod sqrt(1+2^-2k)),
 *   i.e. the rotated pair rounded (half up) onto the 2^16 attention grid.
 * |out| < 2^24 is part of the contract (the int64 score bound); violations are
 * reported as XREF_ERANGE.
 */
#include "xref.h"

#include <math.h>
#include <string.h>

typedef unsigned __int128 u128;
typedef __int128 i128;

/* atan(1/m) * 2^124 by the alternating series, m >= 2 */
static u128 atan_inv_q124(uint32_t m) {
    u128 p = ((u128)1 << 124) / m, m2 = (u128)m * m, sum = 0;
    int add = 1;
    for (uint32_t k = 1; p != 0; k += 2) {
        u128 t = p / k;
        if (add) sum += t; else sum -= t;
        add = !add;
        p /= m2;
    }
    return sum;
}

/* 2*pi * 2^124 (Machin: pi = 16 atan(1/5) - 4 atan(1/239)) */
static u128 two_pi_q124(void) {
    return 2 * (16 * atan_inv_q124(5) - 4 * atan_inv_q124(239));
}

/* atan(2^-k) * 2^124, k >= 1 */
static u128 atan_pow2_q124(int k) {
    u128 p = (u128)1 << (124 - k), sum = 0;
    int add = 1;
    for (uint32_t n = 1; p != 0; n += 2) {
        u128 t = p / n;
        if (add) sum += t; else sum -= t;
        add = !add;
        p >>= 2 * k;
    }
    return sum;
}

/* floor(num * 2^shift / den) rounded half up; num < den < 2^127 */
static u128 ratio_shift(u128 num, u128 den, int shift) {
    u128 r = num, q = 0;
    for (int i = 0; i < shift; i++) {
        r <<= 1; q <<= 1;
        if (r >= den) { r -= den; q |= 1; }
    }
    if ((r << 1) >= den) q++;
    return q;
}

static u128 isqrt128(u128 v) {
    u128 res = 0, bit = (u128)1 << 126;
    while (bit > v) bit >>= 2;
    while (bit) {
        if (v >= res + bit) { v -= res + bit; res = (res >> 1) + bit; }
        else res >>= 1;
        bit >>= 2;
    }
    return res;
}

void xref_cordic_atan_table(uint64_t tab[XREF_CORDIC_ITERS]) {
    const u128 P = two_pi_q124();
    tab[0] = UINT64_C(1) << 61;                       /* atan(1) = 1/8 turn */
    for (int k = 1; k < XREF_CORDIC_ITERS; k++)
        tab[k] = (uint64_t)ratio_shift(atan_pow2_q124(k), P, 64);
}

uint64_t xref_cordic_gain_q62(void) {
    u128 g = (u128)1 << 62;
    for (int k = 0; k < XREF_CORDIC_ITERS; k++) {
        u128 s = isqrt128(((u128)1 << 124) + ((u128)1 << (124 - 2 * k)));   /* sqrt(1+2^-2k) Q62 */
        g = (g << 62) / s;
    }
    return (uint64_t)g;
}

int xref_rope_freq_table(float base, int d, uint64_t *W) {
    uint32_t bits; memcpy(&bits, &base, 4);
    uint32_t e8 = (bits >> 23) & 0xFFu, mant = bits & 0x7FFFFFu;
    if ((bits >> 31) || e8 < 127u || e8 == 255u || d <= 0 || (d & 1)) return XREF_EBADARG;
    /* log2(base) in Q62: integer part from the exponent, fraction bit by bit */
    u128 y = (u128)(mant | 0x800000u) << 39;          /* mantissa in [1,2), Q62 */
    u128 L = 0;
    for (int j = 1; j <= 62; j++) {
        y = (y * y) >> 62;
        if (y >= ((u128)1 << 63)) { y >>= 1; L |= (u128)1 << (62 - j); }
    }
    L += (u128)(e8 - 127u) << 62;
    /* c_j = 2^(-2^-j) in Q62 */
    u128 c[63];
    c[1] = isqrt128((u128)1 << 123);
    for (int j = 2; j <= 62; j++) c[j] = isqrt128(c[j - 1] << 62);
    const u128 P = two_pi_q124();
    for (int i = 0; i < d / 2; i++) {
        u128 t = ((u128)(2 * i) * L) / (u128)d;       /* -exponent, Q62 */
        u128 n = t >> 62, f = t & (((u128)1 << 62) - 1);
        u128 r = (u128)1 << 62;
        for (int j = 1; j <= 62; j++)
            if ((f >> (62 - j)) & 1) r = (r * c[j]) >> 62;
        W[i] = (n > 126) ? 0 : (uint64_t)ratio_shift(r, P, 126 - (int)n);
    }
    return XREF_OK;
}

int xref_rope_cordic(const float *v, int d, int64_t p, const uint64_t *W, int32_t *out) {
    static uint64_t T[XREF_CORDIC_ITERS];
    static uint64_t G;
    static int init = 0;
    if (!init) { xref_cordic_atan_table(T); G = xref_cordic_gain_q62(); init = 1; }
    const int half = d / 2;
    int rc = XREF_OK;
    for (int i = 0; i < half; i++) {
        float a = v[i], b = v[i + half];
        if (!(fabsf(a) < 256.0f) || !(fabsf(b) < 256.0f)) { rc = XREF_ERANGE; a = 0.0f; b = 0.0f; }
        int64_t A = xref_llround((double)a * 1073741824.0);
        int64_t B = xref_llround((double)b * 1073741824.0);
        uint64_t ph = (uint64_t)p * W[i] + (UINT64_C(1) << 61);
        unsigned quad = (unsigned)(ph >> 62);
        int64_t z = (int64_t)(ph & ((UINT64_C(1) << 62) - 1)) - (INT64_C(1) << 61);
        int64_t X, Y;
        switch (quad) {
            case 0:  X = A;  Y = B;  break;
            case 1:  X = -B; Y = A;  break;
            case 2:  X = -A; Y = -B; break;
            default: X = B;  Y = -A; break;
        }
        for (int k = 0; k < XREF_CORDIC_ITERS; k++) {
            int64_t xs = X >> k, ys = Y >> k;
            if (z >= 0) { X -= ys; Y += xs; z -= (int64_t)T[k]; }
            else        { X += ys; Y -= xs; z += (int64_t)T[k]; }
        }
        i128 rx = ((i128)X * (i128)G + ((i128)1 << 75)) >> 76;
        i128 ry = ((i128)Y * (i128)G + ((i128)1 << 75)) >> 76;
        if (rx >= (1 << 24) || rx <= -(1 << 24) || ry >= (1 << 24) || ry <= -(1 << 24)) {
            rc = XREF_ERANGE; rx = 0; ry = 0;
        }
        out[i] = (int32_t)rx;
        out[i + half] = (int32_t)ry;
    }
    return rc;
}
