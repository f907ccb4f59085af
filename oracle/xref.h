/* xref.h -- XREF: the exact-integer CPU checker for the byte-exact OK_Q4B forward.
 *
 * TEST INFRASTRUCTURE ONLY. Nothing in the product library links, loads or calls
 * this code; only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg
 * use it, and only as the checker the CUDA path is compared against.
 *
 * XREF restates, in plain C, the reference's exact pieces:
 *   - OK_Q4B codec: nibble unpack (frobenius_lift.c:102-107, 200-209), f16->f32
 *     (weight_dtype.c:9-28), activation quantizer sp_frob_quant1 (frobenius_lift.c:27-35)
 *   - the exact islands: RMSNorm / softmax / GELU-tanh (exact_islands.c:20-124)
 *   - the exact attention-score convention of the NTT overlay (forward.c:232-246:
 *     q,k on a 2^16 grid, <q,k> exact, d = (float)((double)ip/2^32) * ascale)
 * and fixes the pieces the reference does not define (the "numeric contract"):
 *   - int64 block-scale accumulation of the OK_Q4B matvec and its one rounding
 *   - CORDIC-RoPE (Volder 1959) with integer-only angle tables
 *   - exact SiLU on the island's exp primitive
 *   - the integer V-sum of the attention
 * Every function documents the rule it implements; the CUDA kernels implement the
 * same rules and must agree byte for byte.
 */
#ifndef XREF_H
#define XREF_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- model descriptor (host pointers; same field order as spb_model_desc) ---- */
typedef struct {
    const uint8_t  *codes;   /* [rows][ceil(cols/2)] nibbles, low nibble = even column */
    const uint16_t *bscale;  /* [rows][ceil(cols/32)] f16 block scales */
    int32_t rows, cols;
} xref_q4b;

typedef struct {
    const float *attn_norm, *q_norm, *k_norm, *post_attn_norm, *ffn_norm, *post_ffw_norm;
    xref_q4b wq, wk, wv, wo, wg, wu, wd;
} xref_layer;

enum { XREF_ARCH_QWEN3 = 0, XREF_ARCH_GEMMA3 = 1 };

typedef struct {
    int32_t arch;            /* XREF_ARCH_* */
    int32_t n_layers, n_embd, n_ff, n_head, n_head_kv, head_dim, n_vocab;
    int32_t sliding_window;  /* gemma3 local layers; <= 0 = none */
    float   rope_base;       /* global layers (gemma3) / all layers (qwen3) */
    float   rope_base_local; /* gemma3 local (sliding-window) layers */
    int32_t swa_period;      /* gemma3: layer L is global iff L % period == period-1 */
    int32_t has_qk_norm;
} xref_config;

typedef struct {
    xref_config       cfg;
    const xref_layer *layers;       /* [n_layers] */
    xref_q4b          token_embd;   /* [n_vocab][n_embd] */
    xref_q4b          output;       /* LM head [n_vocab][n_embd] (== token_embd when tied) */
    const float      *output_norm;  /* [n_embd] */
} xref_model;

/* status codes (mirror the product's error classes) */
enum {
    XREF_OK = 0,
    XREF_EBADARG = -3,
    XREF_ERANGE = -50,      /* a value left the exact-arithmetic range of the contract */
    XREF_ENOMEM = -1,
};

/* ---- codec ---- */
float   xref_f16_to_f32(uint16_t h);
int     xref_f16_to_k(uint16_t h, int64_t *k);      /* value == k * 2^-24; -1 on inf/nan */
int8_t  xref_quant1(float v, float scale);
void    xref_unpack_q4(const uint8_t *nib, int n, int8_t *codes);
void    xref_dequant_row(const xref_q4b *w, int r, float *dst);
int     xref_q4b_check(const xref_q4b *w);          /* int64 accumulation bound; 0 = ok */
/* activation quantization of one vector: s = max|u|, q = quant1(u, s). */
void    xref_quant_vec(const float *u, int n, int8_t *q, float *s);
/* exact matvec over n_tok token rows: Y[t][j] for W [rows][cols]; X [n_tok][cols] f32. */
int     xref_matvec(const xref_q4b *w, const float *X, int n_tok, float *Y);
/* same, from already-quantized activations (q [n_tok][cols], s [n_tok]) */
void    xref_matvec_q(const xref_q4b *w, const int8_t *q, const float *s, int n_tok, float *Y);

/* ---- islands (exact_islands.c restated) + builder-defined SiLU ---- */
int64_t xref_llround(double v);
void    xref_rmsnorm_exact(const float *x, const float *w, int n, float *out);
void    xref_softmax_exact(const float *z, int m, double *p);
void    xref_gelu_exact(const float *x, int n, float *out);
void    xref_silu_exact(const float *x, int n, float *out);
int64_t xref_exp_fixed(int64_t d);

/* ---- CORDIC-RoPE ---- */
#define XREF_CORDIC_ITERS 30
void    xref_cordic_atan_table(uint64_t tab[XREF_CORDIC_ITERS]);
uint64_t xref_cordic_gain_q62(void);
/* turns-per-position table W[i] = base^(-2i/d)/(2*pi) * 2^64, i in [0, d/2) */
int     xref_rope_freq_table(float base, int d, uint64_t *W);
/* rotate one head vector (NEOX pairs (i, i+d/2)) at position p; out on the 2^16 grid */
int     xref_rope_cordic(const float *v, int d, int64_t p, const uint64_t *W, int32_t *out);

/* ---- attention (one query head over positions [s0, pos]) ---- */
int     xref_attn_head(const int32_t *q, const int32_t *K, const int32_t *V, int stride,
                       int s0, int pos, int hd, float ascale, float *out);

/* ---- session: persistent exact KV, prefill == sequential decode ---- */
typedef struct xref_session xref_session;
int     xref_session_create(const xref_model *m, int max_ctx, xref_session **out);
void    xref_session_destroy(xref_session *s);
/* one token at the live position; writes [n_vocab] logits if logits != NULL */
int     xref_decode_step(xref_session *s, int32_t token, float *logits);
/* n tokens; writes [n][n_vocab] logits when logits != NULL (every position) */
int     xref_prefill(xref_session *s, const int32_t *tokens, int n, float *logits);
int     xref_rewind(xref_session *s, int n);
int     xref_position(const xref_session *s);
int     xref_clone(const xref_session *s, xref_session **out);
/* read back the cached K or V of one layer at one position ([n_head_kv*head_dim] int32) */
int     xref_kv_read(const xref_session *s, int layer, int pos, int which, int32_t *out);
int     xref_argmax(const float *v, int n);

/* ---- Spinor KV blocks (xref_spinor.c; the reference's frozen 63-byte codec) ---- */
#define XREF_SPINOR_BODY 55
#define XREF_SPINOR_BYTES 63
#define XREF_KV_SPINOR 1u        /* session flag: K/V rows kept as Spinor blocks (SP_KV_SPINOR) */
uint8_t xref_crc8(const uint8_t *data, int len);
int     xref_spinor_blocks_for(int k);
void    xref_spinor_encode(const float *v, int len, uint8_t out[XREF_SPINOR_BYTES]);
int     xref_spinor_decode(const uint8_t in[XREF_SPINOR_BYTES], float *v, int len);
void    xref_spinor_encode_vec(const float *v, int k, uint8_t *blocks);
int     xref_spinor_decode_vec(const uint8_t *blocks, int k, float *v);
int     xref_spinor_kv_row(const int32_t *kg, const float *vf, int hd, uint8_t *blocks, int32_t *grid);
/* a session whose cache holds Spinor blocks (flags = XREF_KV_SPINOR; 0 = xref_session_create) */
int     xref_session_create_ex(const xref_model *m, int max_ctx, unsigned flags, xref_session **out);
/* the cached blocks of one layer at one position: n_head_kv * blocks_for(head_dim) * 63 bytes */
int     xref_kv_bytes(const xref_session *s, int layer, int pos, int which, uint8_t *out);

#ifdef __cplusplus
}
#endif
#endif /* XREF_H */
