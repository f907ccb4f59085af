/* spb200.h -- C ABI of the B200-native byte-exact OK_Q4B forward (libspb200.so).
 *
 * Plain pointers and sizes only. This is the device-side library the reference's
 * L1 backend hooks bind to (the binding itself is libspb200_l1.so, declared in
 * spb200_l1.h). Every entry point returns 0 or a negative status whose values are
 * the reference's sp_status codes (sp_status.h:19-56) where one exists; detail goes
 * to the thread-local spb_last_error().
 *
 * Exactness: every result is byte-identical to the exact-integer CPU restatement
 * of the forward (the checker under oracle/), because every reduction is an integer
 * sum and every rounding is a single IEEE operation; sharding or reordering the
 * work cannot change a byte. Values outside the contract's exact range are reported
 * as SPB_ERANGE instead of being silently wrapped.
 */
#ifndef SPB200_H
#define SPB200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    SPB_OK = 0,
    SPB_ENOMEM = -1,          /* SP_ENOMEM        (host allocation)                  */
    SPB_EBADARG = -3,         /* SP_EBADARG                                          */
    SPB_EBADSTATE = -4,       /* SP_EBADSTATE                                        */
    SPB_EUNSUPPORTED = -5,    /* SP_EUNSUPPORTED  (shape outside the kernels' set)   */
    SPB_ECONTEXT_FULL = -33,  /* SP_ECONTEXT_FULL                                    */
    SPB_ECUDA = -40,          /* SP_ECUDA         (any cudaError_t; detail in text)  */
    SPB_EOOM = -43,           /* SP_EBACKEND_OOM  (device allocation)                */
    SPB_ERANGE = -50          /* a value left the exact-arithmetic range             */
};

/* One OK_Q4B matrix in host memory: the arena layout v2 of frobenius_lift.h:160-173
 * restricted to all-Q4B rows: codes [rows][ceil(cols/2)] (low nibble = even column,
 * 4-bit two's complement), bscale [rows][ceil(cols/32)] f16. */
typedef struct {
    const uint8_t  *codes;
    const uint16_t *bscale;
    int32_t rows, cols;
} spb_q4b;

/* Per-layer tensors; the fields mirror qwen3_layer (model.h:97-113). Norm pointers
 * are f32; post_* are the Gemma3 sandwich norms (NULL for Qwen3). */
typedef struct {
    const float *attn_norm, *q_norm, *k_norm, *post_attn_norm, *ffn_norm, *post_ffw_norm;
    spb_q4b wq, wk, wv, wo, wg, wu, wd;
} spb_layer_desc;

enum { SPB_ARCH_QWEN3 = 0, SPB_ARCH_GEMMA3 = 1 };   /* sp_arch_t values (model.h:24) */

/* Model geometry; mirrors the qwen3_config fields the forward reads (model.h:28-43). */
typedef struct {
    int32_t arch;
    int32_t n_layers, n_embd, n_ff, n_head, n_head_kv, head_dim, n_vocab;
    int32_t sliding_window;   /* Gemma3 local layers; <= 0 = none                 */
    float   rope_base;        /* global layers (Gemma3) / every layer (Qwen3)     */
    float   rope_base_local;  /* Gemma3 local layers (10000, sp_session.c:397)    */
    int32_t swa_period;       /* Gemma3: layer L global iff L % period == period-1 */
    int32_t has_qk_norm;
} spb_config;

typedef struct {
    spb_config            cfg;
    const spb_layer_desc *layers;       /* [n_layers] */
    spb_q4b               token_embd;   /* [n_vocab][n_embd] */
    spb_q4b               output;       /* LM head; == token_embd when tied */
    const float          *output_norm;  /* [n_embd] */
} spb_model_desc;

typedef struct spb_model spb_model;       /* weights resident in one GPU's HBM     */
typedef struct spb_session spb_session;   /* one resident exact KV cache + state   */

const char *spb_last_error(void);
int         spb_device_count(void);

/* ---- model ------------------------------------------------------------------
 * Upload (replaces reading the arena per call, sp_model_bridge.c:114-148 +
 * forward_dispatch.c:100-106): codes/scales/norms copied once into HBM; Q|K|V rows
 * stored contiguously so one launch streams all three. Shapes: n_embd, n_head*head_dim
 * and n_ff multiples of 32; head_dim in {64,128,256}; n_head/n_head_kv <= 8. */
int     spb_model_upload(const spb_model_desc *desc, int device, spb_model **out);
/* Same geometry filled on the device by the counter-based generator of the test
 * fixtures (seeded; identical bytes to the host generator). */
int     spb_model_synthetic(const spb_config *cfg, uint64_t seed, int device, spb_model **out);
void    spb_model_free(spb_model *m);   /* also frees the closed sessions' kept buffers */
int64_t spb_model_weight_bytes(const spb_model *m);   /* OK_Q4B bytes streamed per token */

/* ---- resident KV session (the section-6b verbs, sp_l1.h:386-410) ------------ */
int  spb_session_open(spb_model *m, int pmax, spb_session **out);
/* Compressed K/V (sp_l1.h:156 SP_KV_SPINOR; the reference's kv_mode 1, sp_session.c:233-244,
 * 298-313): every K and V head row is kept as ceil(head_dim / 55) frozen 63-byte Spinor blocks
 * (include/sp/spinor_block.h:93-97), 315 bytes per row at head_dim 256 against 1024 for the
 * int32 grid. A K row is encoded from its 2^16-grid values times 2^-16, a V row from its float
 * projections; attention reads lrintf(decoded * 65536). Unpaged sessions with head_dim 64,
 * 128 or 256 (else SPB_EUNSUPPORTED); not in spb_batch_decode_step. Clone, rewind and prefill
 * keep their meaning. */
#define SPB_KV_SPINOR 1u
int  spb_session_open_ex(spb_model *m, int pmax, unsigned flags, spb_session **out);
/* ingest n_tok tokens at the live position; logits [n_tok][n_vocab] (host) or NULL */
int  spb_session_prefill(spb_session *s, const int32_t *tokens, int n_tok, float *logits);
/* one token; writes the next position's full-vocab logits (host buffer) */
int  spb_session_decode_step(spb_session *s, int32_t token, float *logits);
/* like decode_step, and also returns the greedy argmax (first max index) */
int  spb_session_decode_step_argmax(spb_session *s, int32_t token, float *logits, int32_t *argmax);
/* n_steps greedy steps entirely on the device (no host sync between steps): feeds
 * `token`, then each step's argmax; writes the n_steps argmaxes (host). */
int  spb_session_decode_greedy(spb_session *s, int32_t token, int n_steps, int32_t *tokens_out);
/* One decode step for B (1..64) sessions of one model at once, each at its own position:
 * tokens[B] in, full-vocab logits [B][n_vocab] (host, or NULL) and the greedy argmaxes [B]
 * (host, or NULL) out, every position advanced by one. Same bytes as B separate
 * spb_session_decode_step calls; the weights are streamed once for all B rows. ss[0] runs
 * the step on its stream; the sessions must be distinct. */
int  spb_batch_decode_step(spb_session *const *ss, int B, const int32_t *tokens, float *logits,
                           int32_t *argmax);
int  spb_session_rewind(spb_session *s, int n);          /* O(1): position -= n */
int  spb_session_position(const spb_session *s);         /* -1 on NULL */
/* sp_session_clone (sp_session.c:773-816): a session at the same position with the same cache.
 * A paged session's clone shares its pages (no K/V copied: O(pages) host work); a page is
 * copied only when one of the sessions holding it writes into it. An unpaged session's clone
 * is a deep copy of its cache on the device. */
int  spb_session_clone(const spb_session *s, spb_session **out);

/* ---- paged, copy-on-write K/V (for forks: speculative decode, beam search) --------------
 * A pool of pages on the model's device, each holding page_positions (a multiple of 128)
 * positions of every layer's K and V rows: n_pages * page_positions * n_layers * n_head_kv *
 * head_dim * 8 bytes in all. Paged sessions take pages as they write positions; a page two
 * sessions share (after a clone) is copied before either writes into it. SPB_EOOM when the
 * pool has no free page left. Close every session of a pool before freeing it. */
typedef struct spb_kvpool spb_kvpool;
int  spb_kvpool_create(spb_model *m, int page_positions, int n_pages, spb_kvpool **out);
void spb_kvpool_free(spb_kvpool *p);
int  spb_kvpool_free_pages(spb_kvpool *p);                 /* pages not held by any session */
/* spb_session_open with the K/V rows in pool pages (same verbs and bytes as an unpaged session) */
int  spb_session_open_paged(spb_kvpool *p, int pmax, spb_session **out);
/* Ends a session. Its device buffer (at most 1 GiB), stream and pinned staging stay with the model
 * for the next open of the same size (at most 16 buffers and 4 GiB per model, oldest dropped
 * first); spb_model_free releases them. Environment SPB_SESSION_REUSE=0 frees them at once. */
void spb_session_close(spb_session *s);
/* readback of one cached K (which=0) or V (which=1) row: [n_head_kv*head_dim] int32
 * (SPB_EUNSUPPORTED for a Spinor session) */
int  spb_session_kv_read(const spb_session *s, int layer, int pos, int which, int32_t *out);
/* a Spinor session's cached K or V blocks of one layer and position: n_head_kv rows of
 * ceil(head_dim / 55) * 63 bytes */
int  spb_session_kv_bytes(const spb_session *s, int layer, int pos, int which, uint8_t *out);
/* device stream the session enqueues on (cudaStream_t) */
void *spb_session_stream(spb_session *s);

/* ---- full forward (the section-6 hook, sp_l1.h:319-321) ----------------------
 * n_tok tokens from position 0; writes all n_tok x n_vocab logits (host). */
int  spb_forward(spb_model *m, const int32_t *tokens, int n_tok, float *logits);

/* ---- isolated kernels over device buffers (parity + the dequant-GEMV sweep) --
 * stream: a cudaStream_t (NULL = legacy default stream). */
/* y[t][j] = exact OK_Q4B matvec of the f32 rows x[t] (quantized by sp_frob_quant1
 * over each row's max|x|); n_tok in {1,2,4,8,16}; cols % 32 == 0. Uses a per-device
 * workspace allocated on first use. */
int spb_gemv_q4b(const uint8_t *codes, const uint16_t *bscale, int rows, int cols,
                 const float *x, int n_tok, float *y, void *stream);
/* spb_gemv_q4b without any device allocation (no counterpart in the reference; it exists for
 * callers that may not call cudaMalloc, e.g. when the device memory is already owned by
 * another pool or a latency-critical path must avoid the allocator's implicit device sync).
 * Same arguments and bytes as spb_gemv_q4b. Its scratch is one fixed array inside the
 * library (about 288 KB per GPU, held until the process exits): cols must be at most 16384
 * (the GEMV's widest row) and n_tok * cols at most 262144, else SPB_EBADARG before anything
 * is launched. All calls on a device share that scratch, so calls that can overlap on the
 * GPU race; serialise them. The first call on a device (and in each new context on it) sets
 * up the scratch's device address and should come before any stream capture. Inputs must be
 * finite: spb_gemv_q4b's range-error bits live in an allocated word (read by
 * spb_take_device_errors), so this variant records none. */
int spb_gemv_q4b_noalloc(const uint8_t *codes, const uint16_t *bscale, int rows, int cols,
                         const float *x, int n_tok, float *y, void *stream);
/* A prepared OK_Q4B matrix in device memory (codes and bscale stay the caller's and must
 * outlive the handle). Preparing replaces what matmul_arena redoes on every call
 * (forward_dispatch.c:69-86: sp_arena_find, the per-row unpack) and the arena freeze
 * (arena.c:28-31) with one pass over the block scales: the exact int64 accumulation bound
 * is checked per row (SPB_ERANGE when a row breaks it, the test xref_q4b_check restates),
 * and the scales are described for the kernels (the small-scale flag of the token-batch
 * GEMM; per-row exponent shifts and the digit planes of the tensor-core GEMM). Stream-ordered
 * on `stream`, then synchronises it. cols a multiple of 32, at most 16384; codes 16-byte
 * aligned. */
typedef struct spb_q4b_mat spb_q4b_mat;
int  spb_q4b_prepare(const uint8_t *codes, const uint16_t *bscale, int rows, int cols, void *stream,
                     spb_q4b_mat **out);
void spb_q4b_release(spb_q4b_mat *m);
/* out = {rows, cols, small-scale flag, digit planes (0: the tensor-core GEMM does not cover it)} */
int  spb_q4b_info(const spb_q4b_mat *m, int32_t out[4]);
/* y [n_tok][rows] = the exact OK_Q4B matmul of the f32 rows x [n_tok][cols] (device pointers), any
 * n_tok >= 1: the sp_matmul of forward_dispatch.c:100-106 over the Q4B branch. Rows are quantized
 * by sp_frob_quant1 over each row's max|x|; batches of 16 and more run the token-batch GEMM,
 * fewer the dequant-GEMV; the bytes are the same either way. Uses the per-device workspace. */
int  spb_q4b_matmul(const spb_q4b_mat *m, const float *x, int n_tok, float *y, void *stream);
/* The activation quantizer alone: n_tok rows of cols floats -> the GEMV's input form:
 * q [n_tok][cols] int8 (per 8 columns: the 4 even then the 4 odd), bsum [n_tok][cols/32]
 * int32 block sums of q, scale [n_tok] f32 (max|x|). All device pointers. */
int spb_quantize_rows(const float *x, int cols, int n_tok, int8_t *q, int32_t *bsum, float *scale,
                      void *stream);
/* The dequant-GEMV alone over pre-quantized activations (the form above). */
int spb_gemv_q4b_q(const uint8_t *codes, const uint16_t *bscale, int rows, int cols, const int8_t *q,
                   const int32_t *bsum, const float *scale, int n_tok, float *y, void *stream);
/* Gated pair: y = act(W_gate x) * (W_up x), act 0 = exact GELU (Gemma3), 1 = exact SiLU. */
int spb_gemv_q4b_gated_q(const uint8_t *codes_g, const uint16_t *bscale_g, const uint8_t *codes_u,
                         const uint16_t *bscale_u, int rows, int cols, const int8_t *q,
                         const int32_t *bsum, const float *scale, int n_tok, int act, float *y,
                         void *stream);
int spb_rmsnorm_exact_dev(const float *x, const float *w, int n, int rows, float *out, void *stream);
int spb_gelu_exact_dev(const float *x, int n, float *out, void *stream);
int spb_silu_exact_dev(const float *x, int n, float *out, void *stream);
/* CORDIC-RoPE of `rows` head vectors of length d at positions pos[r] (device) */
int spb_rope_cordic_dev(const float *v, int d, int rows, const int32_t *pos, float base,
                        int32_t *out, void *stream);
/* error bits raised by the last isolated-kernel call on this thread's device */
int spb_take_device_errors(void);

/* Record the spb_* kernel calls a caller makes on `stream` between begin and end into
 * one instantiated CUDA graph, replayed by spb_graph_launch without per-call host cost. */
int  spb_graph_begin(void *stream);
int  spb_graph_end(void *stream, void **graph_exec);
int  spb_graph_launch(void *graph_exec, void *stream);
void spb_graph_free(void *graph_exec);

/* ---- tensor parallel: one process per GPU ----------------------------------
 * Sharding of the per-layer orchestration (gemma3_forward, gemma3.c:39-148; qwen3_forward_ex2,
 * forward.c:87-291) over a group of GPUs. Rank r holds query heads [h0, h0+nh) and their KV
 * heads (Q/K/V rows), the FFN columns [f0, f0+nff) (gate/up rows, down columns), the attention
 * output projection's columns of its heads and the LM-head rows [v0, v0+nv); norms, tables
 * and the embedding are whole on every rank. The two K-split matrices per layer end in an
 * all-reduce of their int64 partial sums (exact in any order); the quantizer's row max of a
 * split producer is all-reduced first; the LM head all-reduces its greedy-argmax keys and
 * all-gathers its logits, so every rank returns the full-vocabulary logits and the argmax of
 * the unsplit model, byte for byte. Exchanges run on NCCL (loaded at run time). */
typedef struct spb_tp spb_tp;
#define SPB_TP_ID_BYTES 128
/* out = {h0, nh, kv0, nkv, f0, nff, v0, nv} of `rank`; no device needed. Requires n_head_kv,
 * n_vocab divisible by world and n_ff by 32 * world. */
int  spb_tp_shard(const spb_config *cfg, int rank, int world, int32_t out[8]);
int  spb_tp_unique_id(uint8_t id[SPB_TP_ID_BYTES]);   /* on one rank; every rank opens with it */
int  spb_tp_open(const uint8_t id[SPB_TP_ID_BYTES], int rank, int world, int device, spb_tp **out);
void spb_tp_close(spb_tp *tp);
int  spb_tp_rank(const spb_tp *tp);
int  spb_tp_world(const spb_tp *tp);
/* Optional, collective: a mailbox of `cap` 8-byte values per rank and exchange parity in this
 * rank's HBM, mapped into every rank through CUDA IPC; afterwards every exchange of at most cap
 * values (the decode step's) runs as one kernel over peer memory (stores over NVLink, a system
 * fence, a flag per rank, a wait bounded at 2 s that reports SPB_ECUDA "timeout" when a rank
 * does not arrive) instead of NCCL. init returns this rank's blob; connect takes all ranks'
 * blobs in rank order (SPB_TP_P2P_BLOB_BYTES each) and refuses two ranks on one GPU. */
#define SPB_TP_P2P_BLOB_BYTES 80
int  spb_tp_p2p_init(spb_tp *tp, int cap, uint8_t blob[SPB_TP_P2P_BLOB_BYTES]);
int  spb_tp_p2p_connect(spb_tp *tp, const uint8_t *blobs);
/* Diagnostics of the exchange kernel's bounded wait (no group needed): one exchange of n
 * (<= 4096) int64 values through that kernel as rank 0 of a loopback group of `world` (2..8)
 * mailboxes that all live on the current device. The sources outside absent_mask have arrived
 * before the launch; those in it (never bit 0) never do, so the wait runs out after timeout_ms
 * (1..10000) and the call returns SPB_ECUDA with "timeout" in spb_last_error(), the device and
 * context staying usable. With absent_mask 0 it returns SPB_OK once the exact sum is checked.
 * This is the failure contract of sp_status (SP_ECUDA, sp_status.h:19-56) for a peer that never
 * arrives; a decode step whose exchange times out reports the same SPB_ECUDA. */
int  spb_tp_p2p_loopback(int world, uint32_t absent_mask, int timeout_ms, int n);
/* The rank's shard of the counter-generated model of spb_model_synthetic (same bytes as the
 * corresponding slices of the unsplit model), on the group's device. */
int  spb_model_synthetic_tp(const spb_config *cfg, uint64_t seed, spb_tp *tp, spb_model **out);
/* The rank's shard of a whole host model (the same descriptor spb_model_upload takes): only
 * the rank's rows and columns are copied to its device. */
int  spb_model_upload_tp(const spb_model_desc *desc, spb_tp *tp, spb_model **out);

/* ---- host-side tables (no device needed) ------------------------------------ */
int      spb_rope_freq_table(float base, int d, uint64_t *W);      /* [d/2] turns Q64 */
void     spb_cordic_tables(uint64_t T[30], uint64_t *gain_q62);

#ifdef __cplusplus
}
#endif
#endif /* SPB200_H */
