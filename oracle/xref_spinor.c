/* xref_spinor.c -- XREF restatement of the reference's 63-byte Spinor KV block codec.
 *
 * TEST INFRASTRUCTURE ONLY (see xref.h): the checker the CUDA path's compressed KV cache is
 * compared against, itself pinned to the reference's compiled codec by the tests.
 *
 * The reference codec (frozen v1):
 *   - block = header[7] || body[55] || crc8, 63 bytes (include/sp/spinor_block.h:93-97)
 *       header: f32 scale little-endian [0..3], exponent int8 [4] (v1: 0), basis [5] (0), 0 [6]
 *   - encode (vht2.c:58-84, spinor_block.c:56-75): scale = max |v| over the chunk (1 when the
 *     max is 0), coefficient = saturate to +-127 of round-half-away(f32(v / scale) * 127) with
 *     round-half-away(x) = floorf(x + 0.5f) for x >= 0, ceilf(x - 0.5f) otherwise (f32 ops);
 *     coordinates past the chunk are 0; body[(17 i) mod 55] = coefficient i (mobius_reorder.c:41-46)
 *   - CRC-8/SMBus (poly 0x07, init 0, no reflection, xorout 0) over header || body (vht2.c:29-47)
 *   - decode (spinor_block.c:77-97, vht2.c:86-98): coefficient i = body[(17 i) mod 55],
 *     mul = f32(scale * 2^exp) / 127.0f, v_i = (float)coefficient_i * mul; the CRC result is
 *     reported but the session's window decode ignores it (sp_session.c:306-310)
 *   - a head of k > 55 coordinates: nblk = ceil(k / 55) contiguous chunks, the first k % nblk
 *     of them one longer (spinor_block.c:121-149)
 *
 * The KV-cache transform of the exact path (builder-defined, no reference counterpart): a K
 * row on the 2^16 score grid is encoded from kf_i = kg_i * 2^-16 (exact in f32), a V row from
 * its float projections; the grid value attention uses is lrintf(decoded * 65536).
 */
#include "xref.h"

#include <math.h>
#include <string.h>

uint8_t xref_crc8(const uint8_t *data, int len) {
    unsigned crc = 0u;
    for (int i = 0; i < len; i++) {
        crc ^= data[i];
        for (int b = 0; b < 8; b++) crc = (crc & 0x80u) ? ((crc << 1) ^ 0x07u) & 0xFFu : (crc << 1) & 0xFFu;
    }
    return (uint8_t)crc;
}

int xref_spinor_blocks_for(int k) { return k <= XREF_SPINOR_BODY ? 1 : (k + XREF_SPINOR_BODY - 1) / XREF_SPINOR_BODY; }

static int32_t round_half_away_f(float x) {
    const float r = (x >= 0.0f) ? floorf(x + 0.5f) : ceilf(x - 0.5f);
    return (int32_t)r;
}

void xref_spinor_encode(const float *v, int len, uint8_t out[XREF_SPINOR_BYTES]) {
    const int lim = len < 0 ? 0 : (len < XREF_SPINOR_BODY ? len : XREF_SPINOR_BODY);
    float mx = 0.0f;
    for (int i = 0; i < lim; i++) {
        const float a = fabsf(v[i]);
        if (a > mx) mx = a;
    }
    const float scale = mx > 0.0f ? mx : 1.0f;
    memset(out, 0, XREF_SPINOR_BYTES);
    uint32_t u;
    memcpy(&u, &scale, 4);
    for (int b = 0; b < 4; b++) out[b] = (uint8_t)(u >> (8 * b));
    for (int i = 0; i < lim; i++) {
        int32_t q = round_half_away_f((v[i] / scale) * 127.0f);
        if (q > 127) q = 127;
        if (q < -127) q = -127;
        out[7 + (17 * i) % XREF_SPINOR_BODY] = (uint8_t)(int8_t)q;
    }
    out[XREF_SPINOR_BYTES - 1] = xref_crc8(out, XREF_SPINOR_BYTES - 1);
}

int xref_spinor_decode(const uint8_t in[XREF_SPINOR_BYTES], float *v, int len) {
    const int bad = xref_crc8(in, XREF_SPINOR_BYTES - 1) != in[XREF_SPINOR_BYTES - 1];
    uint32_t u = (uint32_t)in[0] | ((uint32_t)in[1] << 8) | ((uint32_t)in[2] << 16) | ((uint32_t)in[3] << 24);
    float scale;
    memcpy(&scale, &u, 4);
    const float mul = scale * ldexpf(1.0f, (int)(int8_t)in[4]) / 127.0f;
    const int lim = len < 0 ? 0 : (len < XREF_SPINOR_BODY ? len : XREF_SPINOR_BODY);
    for (int i = 0; i < lim; i++) v[i] = (float)(int8_t)in[7 + (17 * i) % XREF_SPINOR_BODY] * mul;
    for (int i = XREF_SPINOR_BODY; i < len; i++) v[i] = 0.0f;
    return bad;
}

void xref_spinor_encode_vec(const float *v, int k, uint8_t *blocks) {
    const int nb = xref_spinor_blocks_for(k), base = k / nb, extra = k % nb;
    for (int b = 0, off = 0; b < nb; b++) {
        const int len = base + (b < extra ? 1 : 0);
        xref_spinor_encode(v + off, len, blocks + (size_t)b * XREF_SPINOR_BYTES);
        off += len;
    }
}

int xref_spinor_decode_vec(const uint8_t *blocks, int k, float *v) {
    const int nb = xref_spinor_blocks_for(k), base = k / nb, extra = k % nb;
    int rc = 0;
    for (int b = 0, off = 0; b < nb; b++) {
        const int len = base + (b < extra ? 1 : 0);
        rc |= xref_spinor_decode(blocks + (size_t)b * XREF_SPINOR_BYTES, v + off, len);
        off += len;
    }
    return rc;
}

/* One head row of the compressed cache: kg != NULL: a K row on the 2^16 grid (encoded from
 * kg * 2^-16); else a V row from its float values vf (|v| < 16384 before and after the round
 * trip). Writes the blocks and the grid values attention reads; XREF_ERANGE on a V range break. */
int xref_spinor_kv_row(const int32_t *kg, const float *vf, int hd, uint8_t *blocks, int32_t *grid) {
    float f[1024], d[1024];
    if (hd <= 0 || hd > 1024) return XREF_EBADARG;
    for (int i = 0; i < hd; i++) {
        if (kg) f[i] = (float)kg[i] * (1.0f / 65536.0f);
        else {
            if (!(fabsf(vf[i]) < 16384.0f)) return XREF_ERANGE;
            f[i] = vf[i];
        }
    }
    xref_spinor_encode_vec(f, hd, blocks);
    (void)xref_spinor_decode_vec(blocks, hd, d);
    for (int i = 0; i < hd; i++) {
        if (!kg && !(fabsf(d[i]) < 16384.0f)) return XREF_ERANGE;
        grid[i] = (int32_t)lrintf(d[i] * 65536.0f);
    }
    return XREF_OK;
}
