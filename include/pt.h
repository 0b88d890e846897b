#ifndef PITORCH_PT_H
#define PITORCH_PT_H

/*
 * Top-level context API -- drop-in for pitorch/pt.h, backed by a B200.
 *
 * pt_context_t keeps every field of the reference (pitorch/pt.h:23-44) with
 * the same meaning; this build appends device fields at the end. One call to
 * pt_pi_init / pt_host_init uploads the weights once into a device arena,
 * allocates all decode (and, with max_T > 0, training) state on the GPU and
 * captures the decode step as a CUDA graph. Every call is synchronous on
 * return, as in the reference.
 *
 * Differences a caller can observe:
 *  - ctx->w still points into the caller's blob; training updates the
 *    DEVICE weights. pt_sync_weights() copies them back into the blob.
 *  - ctx->state.logits is refreshed after each pt_forward_step only while
 *    ctx->sync_logits is non-zero (the default); the argmax is computed on
 *    the GPU either way.
 *  - training activations/gradients are device-resident; pt_sync_grads()
 *    fills ctx->grads._mem.
 */

#include "llama2.h"
#include "pt_train.h"
#include "pt_shard.h"
#include "trace.h"

struct pt_device;

typedef struct {
    pt_config_t       cfg;
    pt_weights_t      w;
    int               shared_weights;
    pt_matvec_fn      matvec;

    /* inference */
    pt_state_t        state;
    int               pos;

    /* training (zeroed when max_T == 0) */
    pt_activations_t  acts;
    pt_grads_t        grads;
    pt_backward_buf_t bb;
    int               max_T;

    /* profiling -- NULL means disabled */
    pt_trace_t       *trace;

    /* on the Pi: QPU count; here: the CUDA device ordinal in use */
    int               num_qpus;

    /* ---- pitorch_b200 additions ---- */
    struct pt_device *dev;          /* device-side context (opaque) */
    int               sync_logits;  /* copy logits to state.logits each step (default 1) */
} pt_context_t;

/* pitorch/pt.h:50-51 (host build) -- here: device 0 (or $PT_DEVICE), arena
 * sized automatically. */
void pt_host_init(pt_context_t *ctx, void *weight_data, int max_T);
void pt_free(pt_context_t *ctx);

/* pitorch/pt.h:62-63. num_qpus has no QPU meaning here: a value >= 0 that
 * names a visible CUDA device selects it, anything else means device 0
 * (or $PT_DEVICE). arena_bytes is the initial device arena size; it is
 * raised to what the model needs. */
void pt_pi_init(pt_context_t *ctx, void *weight_data,
                int num_qpus, int max_T, unsigned arena_bytes);

/* pitorch/pt.h:72-74. Loads a SHRD shard: only the owned layers
 * (cfg.n_layers = n_local) and, when present, embedding + head. */
void pt_pi_init_shard(pt_context_t *ctx, pt_shard_info_t *shard_out,
                      void *shard_data, int num_qpus, int max_T,
                      unsigned arena_bytes);

/* pitorch/pt.h:83: forward at ctx->pos, ++pos, returns the greedy token. */
int pt_forward_step(pt_context_t *ctx, int token);

/* pitorch/pt.h:86 */
void pt_reset_kv(pt_context_t *ctx);

/* pitorch/pt.h:89 */
void pt_print_config(const pt_context_t *ctx);

/* pitorch/pt.h:95 */
void *pt_read_file(const char *path, long *out_size);

/* pitorch/pt.h:104: zero_grads -> forward_train -> backward -> sgd. */
float pt_train_step(pt_context_t *ctx, const int *tokens, int T, float lr);

/* pitorch/pt.h:108-109 */
void pt_enable_trace(pt_context_t *ctx, pt_trace_t *preallocated);
void pt_disable_trace(pt_context_t *ctx);

/* ---- pitorch_b200 additions ---- */

/* Greedy decode of n_pos positions entirely on the device: prompt tokens
 * are teacher-forced, then each argmax feeds the next position. Resets the
 * KV cache first and leaves ctx->pos = n_pos. out_tokens[p] is the token
 * emitted at position p (the next input). */
void pt_generate_greedy(pt_context_t *ctx, const int *prompt, int n_prompt,
                        int n_pos, int *out_tokens);

/* Copy device weights back into the caller's blob (after training). */
void pt_sync_weights(pt_context_t *ctx);
/* Fill ctx->grads._mem from the device gradients of the last step. */
void pt_sync_grads(pt_context_t *ctx);
/* Checkpoint (no reference counterpart: the Pi build keeps weights only in
 * RAM): bring the device weights back (pt_sync_weights) and write the
 * context's model image -- the llama2.c .bin, or the SHRD shard for a
 * pt_pi_init_shard context -- to path, loadable again with pt_read_file +
 * pt_pi_init / pt_pi_init_shard. Returns 0, or -1 when the file cannot be
 * written. */
int pt_save_weights(pt_context_t *ctx, const char *path);

/* The device context's C-ABI handles (see ptc.h). */
struct ptc_ctx *pt_ptc_ctx(pt_context_t *ctx);
struct ptc_decoder *pt_ptc_decoder(pt_context_t *ctx);
struct ptc_trainer *pt_ptc_trainer(pt_context_t *ctx);   /* NULL without max_T > 0 */

#endif
