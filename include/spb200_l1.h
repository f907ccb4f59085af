/* spb200_l1.h -- the reference-facing drop-in: L1 backend hooks of libshannonprime
 * implemented on the B200 byte-exact forward (libspb200_l1.so).
 *
 * Built against the reference's own frozen headers (sp/sp_l1.h, sp/model.h,
 * sp/arena.h); loaded into a process that already links libshannonprime, whose
 * sp_arena_find / sp_as_f32 / sp_set_error it calls. Registration is the caller's
 * (the L2 daemon's) job, exactly as for the engine backends:
 *
 *   sp_session_register_forward_backend(s, spb_l1_backend(), spb_l1_forward);
 *   sp_kvdecode_handle *h;  const sp_kvdecode_dispatch_fn *dt = spb_l1_kvdecode_table();
 *   dt->open(sp_session_qwen3_model(s), pmax, &h);
 *   sp_session_register_kvdecode_backend(s, h, dt);
 *
 * Device weights are uploaded once per model (keyed by the qwen3_model pointer) and
 * shared by every session on that model.
 */
#ifndef SPB200_L1_H
#define SPB200_L1_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

struct sp_kvdecode_dispatch_fn;
struct sp_kvdecode_handle;

/* Replaces the engine's per-backend full-forward (gemma3_forward_cuda) behind the
 * section-6 hook: same signature as sp_forward_dispatch_fn (sp_l1.h:319-321). Writes
 * all n_tok x n_vocab logits of the full history (sp_l1.h:312-318); nonzero on error
 * with the detail in sp_set_error. `handle` is spb_l1_backend() (or NULL). */
int spb_l1_forward(void *handle, const void *qm_opaque, const int32_t *tokens, int n_tok,
                   float *logits);

/* Opaque handle to pass with spb_l1_forward (selects the device). */
void *spb_l1_backend(void);

/* The section-6b dispatch table (sp_l1.h:403-410): open uploads the model on first use
 * and allocates an exact resident KV cache of pmax positions; prefill ingests history;
 * decode_step writes the next position's full-vocab logits; rewind is O(1); position
 * reports dpos; close frees the cache. Replaces the engine's gemma4_kv_* resident
 * decode (sp_l1.h:381-384, 436-441). */
const struct sp_kvdecode_dispatch_fn *spb_l1_kvdecode_table(void);

/* Append-only extension of the section-6b table (sp_l1.h:450-452 allows new rows at the
 * end): fork a resident cache, the missing piece for speculative decode --
 * sp_session_clone drops section-6b (sp_session.c:792-799). With a page pool (below) the
 * fork shares the cache's pages and copies a page only when one side writes into it; without
 * one it is a deep copy of the cache on the device. */
int spb_l1_kvdecode_clone(const struct sp_kvdecode_handle *h, struct sp_kvdecode_handle **out);

/* The table with that row appended: its first member is the frozen table, so a caller that
 * knows only sp_l1.h reads the same six rows; one that knows the extension finds `clone`
 * after `close`. spb_l1_kvdecode_table() returns &spb_l1_kvdecode_table_ext()->base.
 * (Complete type only where sp/sp_l1.h is included before this header.) */
#ifdef SP_L1_H
struct spb_kvdecode_dispatch_ext {
    struct sp_kvdecode_dispatch_fn base;
    int (*clone)(const struct sp_kvdecode_handle *h, struct sp_kvdecode_handle **out);
};
#else
struct spb_kvdecode_dispatch_ext;
#endif
const struct spb_kvdecode_dispatch_ext *spb_l1_kvdecode_table_ext(void);

/* Caches of models uploaded after this call live in a per-model page pool of n_pages pages of
 * page_positions (a multiple of 128) positions, so forks are O(1); 0, 0 (default) = each
 * cache its own allocation. */
int spb_l1_set_kv_pool(int page_positions, int n_pages);

/* spb_session_open_ex flags of the section-6b caches opened after this call: SPB_KV_SPINOR keeps
 * their K/V rows as the reference's 63-byte Spinor blocks (its SP_KV_SPINOR session flag,
 * sp_l1.h:156-157, which the frozen open row cannot carry); 0 (default) = int32 rows. A page pool
 * set with spb_l1_set_kv_pool takes precedence. No reference counterpart beyond that flag. */
int spb_l1_set_kv_flags(unsigned flags);

/* Device used for models uploaded after this call (default 0). */
int spb_l1_set_device(int device);

/* Drop the cached device copy of one model (call before sp_model_unload). The cache is keyed by
 * the model's address and a fingerprint of its config, arena and first weight bytes, so a model
 * loaded later at the address of one that was never released is uploaded afresh; releasing
 * still frees the old copy's device memory at once. */
void spb_l1_release_model(const void *qm_opaque);

#ifdef __cplusplus
}
#endif
#endif /* SPB200_L1_H */
