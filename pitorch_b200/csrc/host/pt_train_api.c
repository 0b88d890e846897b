/*
 * pt_train_api.c -- training entry points of pitorch/pt.c:339-364 and
 * pitorch/train/pt_train.h on the device trainer (ptc_trainer_*).
 *
 * A context created with max_T > 0 owns a trainer whose activations,
 * backward buffers and gradients live on the GPU. The host structs keep
 * their meaning as handles: the staged functions find the owning context
 * from the pt_activations_t / pt_grads_t / pt_backward_buf_t address.
 * ctx->grads._mem is a host mirror filled by pt_sync_grads().
 */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "pt_device.h"

#define PT_MAX_TRAIN_CTX 64
static pt_context_t *g_train_ctx[PT_MAX_TRAIN_CTX];

static void reg_ctx(pt_context_t *ctx) {
    for (int i = 0; i < PT_MAX_TRAIN_CTX; i++)
        if (!g_train_ctx[i]) { g_train_ctx[i] = ctx; return; }
    pt_fatal("too many training contexts (max %d)", PT_MAX_TRAIN_CTX);
}

static void unreg_ctx(pt_context_t *ctx) {
    for (int i = 0; i < PT_MAX_TRAIN_CTX; i++)
        if (g_train_ctx[i] == ctx) g_train_ctx[i] = NULL;
}

static pt_context_t *ctx_of(const void *member, const char *what) {
    for (int i = 0; i < PT_MAX_TRAIN_CTX; i++) {
        pt_context_t *c = g_train_ctx[i];
        if (c && (member == (const void *)&c->acts || member == (const void *)&c->grads ||
                  member == (const void *)&c->bb || member == (const void *)&c->w))
            return c;
    }
    pt_fatal("%s was not created by pt_pi_init / pt_host_init with max_T > 0", what);
    return NULL;
}

static ptc_trainer *trainer(pt_context_t *ctx) {
    if (!ctx->dev || !ctx->dev->trainer) pt_fatal("context has no trainer (initialise with max_T > 0)");
    return ctx->dev->trainer;
}

/* Host-mirror gradient layout of pt_train.c:334-371 (absent parts empty). */
static void carve_host_grads(pt_context_t *ctx, size_t n) {
    pt_grads_t *g = &ctx->grads;
    const pt_config_t *c = &ctx->cfg;
    size_t D = c->dim, H = c->hidden_dim, L = c->n_layers;
    size_t K = (size_t)c->n_kv_heads * (c->dim / c->n_heads);
    size_t Ve = ctx->dev->has_embed ? (size_t)c->vocab_size : 0;
    g->_mem = (float *)calloc(n ? n : 1, sizeof(float));
    g->_n_params = (int)n;
    float *p = g->_mem;
    g->token_embedding = Ve ? p : NULL; p += Ve * D;
    g->rms_att_weight = p; p += L * D;
    g->wq = p; p += L * D * D;
    g->wk = p; p += L * K * D;
    g->wv = p; p += L * K * D;
    g->wo = p; p += L * D * D;
    g->rms_ffn_weight = p; p += L * D;
    g->w1 = p; p += L * H * D;
    g->w2 = p; p += L * D * H;
    g->w3 = p; p += L * H * D;
    g->rms_final_weight = ctx->dev->has_head ? p : NULL;
    p += ctx->dev->has_head ? D : 0;
    if (ctx->dev->has_head)
        g->wcls = ctx->shared_weights ? g->token_embedding : p;
}

void pt_train_init(pt_context_t *ctx, int max_T) {
    struct pt_device *d = ctx->dev;
    d->trainer = ptc_trainer_create(d->ctx, &d->cfg, &d->dw, max_T, d->has_embed, d->has_head);
    carve_host_grads(ctx, ptc_trainer_n_params(d->trainer));
    ctx->acts.T = max_T;
    reg_ctx(ctx);
}

void pt_train_free(pt_context_t *ctx) {
    unreg_ctx(ctx);
    if (ctx->dev && ctx->dev->trainer) ptc_trainer_destroy(ctx->dev->trainer);
    if (ctx->dev) ctx->dev->trainer = NULL;
    free(ctx->grads._mem);
    memset(&ctx->grads, 0, sizeof(ctx->grads));
}

/* pt.c:339-364 */
float pt_train_step(pt_context_t *ctx, const int *tokens, int T, float lr) {
    pt_trace_t *tr = ctx->trace;
    pt_trace_begin(tr, "train_step", "train", -1);
    float loss = ptc_trainer_step(trainer(ctx), tokens, T, lr);
    ptc_decoder_weights_updated(ctx->dev->dec);
    ctx->acts.T = T;
    pt_trace_end(tr);
    return loss;
}

void pt_sync_weights(pt_context_t *ctx) {
    struct pt_device *d = ctx->dev;
    if (!d) return;
    /* everything after the header: tensors are updated in place on the device */
    size_t hdr = d->is_shard ? 56 : 28;
    ptc_d2h(d->ctx, (char *)d->host_image + hdr, d->dev_image + hdr, d->image_bytes - hdr);
}

int pt_save_weights(pt_context_t *ctx, const char *path) {
    struct pt_device *d = ctx->dev;
    if (!d || !d->host_image) return -1;
    pt_sync_weights(ctx);
    FILE *f = fopen(path, "wb");
    if (!f) return -1;
    const size_t n = fwrite(d->host_image, 1, d->image_bytes, f);
    const int rc = fclose(f);
    return (n == d->image_bytes && rc == 0) ? 0 : -1;
}

void pt_sync_grads(pt_context_t *ctx) {
    ptc_trainer *t = trainer(ctx);
    ptc_trainer_sync(t);
    ptc_d2h(ctx->dev->ctx, ctx->grads._mem, ptc_trainer_grads(t), (size_t)ctx->grads._n_params * 4);
}

/* ---- pt_train.h allocation API (host structs; bind to a device context
 *      through pt_pi_init / pt_host_init with max_T > 0) ------------------- */

void pt_alloc_activations(pt_activations_t *a, const pt_config_t *cfg, int T) {
    (void)cfg;
    memset(a, 0, sizeof(*a));
    a->T = T;
}
void pt_free_activations(pt_activations_t *a) { memset(a, 0, sizeof(*a)); }
void pt_alloc_grads(pt_grads_t *g, const pt_config_t *cfg, int shared_weights) {
    (void)cfg; (void)shared_weights;
    memset(g, 0, sizeof(*g));
}
void pt_free_grads(pt_grads_t *g) { memset(g, 0, sizeof(*g)); }
void pt_alloc_backward_buf(pt_backward_buf_t *b, const pt_config_t *cfg, int T) {
    (void)cfg; (void)T;
    memset(b, 0, sizeof(*b));
}
void pt_free_backward_buf(pt_backward_buf_t *b) { memset(b, 0, sizeof(*b)); }

void pt_zero_grads(pt_grads_t *g) {
    pt_context_t *ctx = ctx_of(g, "pt_grads_t");
    ptc_trainer_zero_grads(trainer(ctx));
    if (g->_mem) memset(g->_mem, 0, (size_t)g->_n_params * 4);
}

/* ---- whole-model passes (pt_train.h:66-159) -------------------------------- */

float pt_forward_train(const pt_config_t *cfg, const pt_weights_t *w, pt_activations_t *a,
                       const int *tokens, int T, pt_matvec_fn matvec, pt_trace_t *trace) {
    (void)cfg; (void)w; (void)matvec;
    pt_context_t *ctx = ctx_of(a, "pt_activations_t");
    ptc_trainer *t = trainer(ctx);
    pt_trace_begin(trace, "forward", "fwd", -1);
    ptc_trainer_set_tokens(t, tokens, T);
    ptc_trainer_fwd_embed(t);
    ptc_trainer_fwd_layers(t, 0, ctx->cfg.n_layers);
    float loss = ptc_trainer_fwd_head(t);
    pt_trace_end(trace);
    a->T = T;
    return loss;
}

void pt_backward(const pt_config_t *cfg, const pt_weights_t *w, pt_grads_t *g, const pt_activations_t *a,
                 pt_backward_buf_t *b, const int *tokens, int T, pt_matvec_fn matvec, pt_trace_t *trace) {
    (void)cfg; (void)w; (void)g; (void)b; (void)matvec;
    pt_context_t *ctx = ctx_of(a, "pt_activations_t");
    ptc_trainer *t = trainer(ctx);
    pt_trace_begin(trace, "backward", "bwd", -1);
    ptc_trainer_set_tokens(t, tokens, T);
    ptc_trainer_bwd_head(t);
    ptc_trainer_bwd_layers(t, 0, ctx->cfg.n_layers);
    ptc_trainer_bwd_embed(t);
    ptc_trainer_sync(t);
    pt_trace_end(trace);
}

void pt_sgd_update(pt_weights_t *w, const pt_grads_t *g, float lr, const pt_config_t *cfg) {
    (void)w; (void)cfg;
    pt_context_t *ctx = ctx_of(g, "pt_grads_t");
    ptc_trainer *t = trainer(ctx);
    ptc_trainer_sgd_head(t, lr);
    ptc_trainer_sgd_layers(t, lr, 0, ctx->cfg.n_layers);
    ptc_trainer_sync(t);
    ptc_decoder_weights_updated(ctx->dev->dec);
}

void pt_sgd_update_layers(pt_weights_t *w, const pt_grads_t *g, float lr, const pt_config_t *cfg,
                          int l_start, int l_end) {
    (void)w; (void)cfg;
    pt_context_t *ctx = ctx_of(g, "pt_grads_t");
    ptc_trainer_sgd_layers(trainer(ctx), lr, l_start, l_end);
    ptc_trainer_sync(trainer(ctx));
    ptc_decoder_weights_updated(ctx->dev->dec);
}

void pt_sgd_update_head(pt_weights_t *w, const pt_grads_t *g, float lr, const pt_config_t *cfg) {
    (void)w; (void)cfg;
    pt_context_t *ctx = ctx_of(g, "pt_grads_t");
    ptc_trainer_sgd_head(trainer(ctx), lr);
    ptc_trainer_sync(trainer(ctx));
}

/* ---- staged passes for pipeline parallelism (pt_train.h:174-224) ---------- */

void pt_forward_train_embed(const pt_weights_t *w, pt_activations_t *a, const int *tokens, int T, int dim) {
    (void)w; (void)dim;
    pt_context_t *ctx = ctx_of(a, "pt_activations_t");
    ptc_trainer *t = trainer(ctx);
    ptc_trainer_set_tokens(t, tokens, T);
    ptc_trainer_fwd_embed(t);
    ptc_trainer_sync(t);
    a->T = T;
}

void pt_forward_train_layers_range(const pt_config_t *cfg, const pt_weights_t *w, pt_activations_t *a, int T,
                                   int l_start, int l_end, pt_matvec_fn matvec, pt_trace_t *trace) {
    (void)cfg; (void)w; (void)matvec; (void)trace;
    pt_context_t *ctx = ctx_of(a, "pt_activations_t");
    ptc_trainer *t = trainer(ctx);
    if (T != a->T) pt_fatal("pt_forward_train_layers_range: T=%d but activations hold T=%d", T, a->T);
    ptc_trainer_fwd_layers(t, l_start, l_end);
    ptc_trainer_sync(t);
}

float pt_forward_train_head(const pt_config_t *cfg, const pt_weights_t *w, pt_activations_t *a,
                            const int *tokens, int T, pt_matvec_fn matvec, pt_trace_t *trace) {
    (void)cfg; (void)w; (void)matvec; (void)trace;
    pt_context_t *ctx = ctx_of(a, "pt_activations_t");
    ptc_trainer *t = trainer(ctx);
    ptc_trainer_set_tokens(t, tokens, T);
    a->T = T;
    return ptc_trainer_fwd_head(t);
}

void pt_backward_head(const pt_config_t *cfg, const pt_weights_t *w, pt_grads_t *g, const pt_activations_t *a,
                      pt_backward_buf_t *b, const int *tokens, int T, pt_matvec_fn matvec, pt_trace_t *trace) {
    (void)cfg; (void)w; (void)g; (void)b; (void)matvec; (void)trace;
    pt_context_t *ctx = ctx_of(a, "pt_activations_t");
    ptc_trainer *t = trainer(ctx);
    ptc_trainer_set_tokens(t, tokens, T);
    ptc_trainer_bwd_head(t);
    ptc_trainer_sync(t);
}

void pt_backward_layers_range(const pt_config_t *cfg, const pt_weights_t *w, pt_grads_t *g,
                              const pt_activations_t *a, pt_backward_buf_t *b, int T, int l_start, int l_end,
                              pt_matvec_fn matvec, pt_trace_t *trace) {
    (void)cfg; (void)w; (void)g; (void)b; (void)T; (void)matvec; (void)trace;
    pt_context_t *ctx = ctx_of(a, "pt_activations_t");
    ptc_trainer_bwd_layers(trainer(ctx), l_start, l_end);
    ptc_trainer_sync(trainer(ctx));
}

void pt_backward_embed(pt_grads_t *g, const pt_backward_buf_t *b, const int *tokens, int T, int dim) {
    (void)b; (void)dim;
    pt_context_t *ctx = ctx_of(g, "pt_grads_t");
    ptc_trainer *t = trainer(ctx);
    ptc_trainer_set_tokens(t, tokens, T);
    ptc_trainer_bwd_embed(t);
    ptc_trainer_sync(t);
}
