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

/* Append-only extension proposed for the section-6b table (sp_l1.h:450-452 allows new
 * rows at the end): fork a resident cache (deep KV copy on the device), the missing
 * piece for speculative decode -- sp_session_clone drops section-6b (sp_session.c:792-799). */
int spb_l1_kvdecode_clone(const struct sp_kvdecode_handle *h, struct sp_kvdecode_handle **out);

/* Device used for models uploaded after this call (default 0). */
int spb_l1_set_device(int device);

/* Drop the cached device copy of one model (call before sp_model_unload). */
void spb_l1_release_model(const void *qm_opaque);

#ifdef __cplusplus
}
#endif
#endif /* SPB200_L1_H */
