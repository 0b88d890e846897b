/*
 * pt_train_api.c -- training entry points of pitorch/pt.c:339-364 and
 * pitorch/train/pt_train.h on the device trainer (ptc_trainer_*).
 *
 * A context created with max_T > 0 owns a trainer whose activations,
 * backward buffers and gradients live on the GPU. Its member structs keep
 * their meaning as handles: the staged functions find the owning context
 * from the pt_activations_t / pt_grads_t / pt_backward_buf_t address, and
 * ctx->grads._mem is a host mirror filled by pt_sync_grads(). Structs a
 * caller allocates with pt_alloc_* work too (below).
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

/* ---- caller-owned training structs (pt_train.h allocators) -----------------
 *
 * pt_alloc_activations / pt_alloc_grads / pt_alloc_backward_buf allocate the
 * reference's host arrays (pitorch/train/pt_train.c:23-50, 334-425). Such a
 * struct is bound to a device trainer the first time a training call pairs
 * it with weights `w`: one trainer per llama2.c image that `w` points into
 * (pt_load_weights on a caller-owned blob), created on first use, which
 * uploads the image then. Its activations, gradients and backward buffers
 * live on the device; the host arrays carry what the reference's callers
 * read or hand between pipeline stages (pt_dist_pipeline.c:134,
 * dev/host/test_stage_train.c):
 *   - a staged forward call takes residuals[l_start] ([T, dim], l * T * dim)
 *     from the host and leaves residuals[l_end] there (the embedding leaves
 *     residuals[0], the head takes residuals[L]);
 *   - a staged backward call takes b->d_res ([T, dim]) from the host and
 *     leaves its result there (the head only leaves it, the embedding only
 *     takes it);
 *   - after a backward sequence (pt_backward, pt_backward_embed) the
 *     gradients are in g->_mem, after pt_backward_layers_range those of its
 *     layers;
 *   - an SGD call writes the tensors it updated back into the caller's image,
 *     so `w` reads the new weights as in the reference.
 * Between calls the device copy of the image is authoritative: a caller that
 * edits the image itself after binding must not expect the trainer to see it.
 */

#define PT_MAX_BINDS 64
#define PT_MAX_OWNED 256

typedef struct {
    const char *image;        /* byte 0 of the caller's llama2.c image */
    struct pt_device *dev;    /* device copy + trainer */
    pt_config_t cfg;
    int shared;
    int max_T;
    pt_grads_t *g;            /* the gradients bound here (one per trainer) */
} train_bind_t;

static train_bind_t g_binds[PT_MAX_BINDS];

static struct {
    const void *s;            /* a pt_activations_t / pt_grads_t / pt_backward_buf_t */
    int bind;                 /* index into g_binds, -1 until bound */
    int T;                    /* allocated T (activations, backward buffers) */
    int zero_pending;         /* grads: zeroed before being bound */
} g_owned[PT_MAX_OWNED];

static int owned_find(const void *s) {
    for (int i = 0; i < PT_MAX_OWNED; i++)
        if (g_owned[i].s == s) return i;
    return -1;
}

static void owned_add(const void *s, int T) {
    int i = owned_find(s);
    if (i < 0)
        for (i = 0; i < PT_MAX_OWNED && g_owned[i].s; i++) {}
    if (i >= PT_MAX_OWNED) pt_fatal("too many live training structs (max %d)", PT_MAX_OWNED);
    g_owned[i].s = s;
    g_owned[i].bind = -1;
    g_owned[i].T = T;
    g_owned[i].zero_pending = 0;
}

/* Forget a freed struct; the last struct of a binding releases its device
 * copy and trainer. */
static void owned_remove(const void *s) {
    int i = owned_find(s);
    if (i < 0) return;
    const int bi = g_owned[i].bind;
    memset(&g_owned[i], 0, sizeof(g_owned[i]));
    if (bi < 0) return;
    for (int k = 0; k < PT_MAX_OWNED; k++)
        if (g_owned[k].s && g_owned[k].bind == bi) return;
    train_bind_t *b = &g_binds[bi];
    if (b->dev) {
        if (b->dev->trainer) ptc_trainer_destroy(b->dev->trainer);
        b->dev->trainer = NULL;
        pt_device_close(b->dev);
    }
    memset(b, 0, sizeof(*b));
}

/* The trainer of the image `w` points into (created on first use). */
static int bind_of_weights(const pt_config_t *cfg, const pt_weights_t *w, int max_T) {
    if (!w || !w->token_embedding) pt_fatal("training call without the model's weights");
    const char *image = (const char *)w->token_embedding - 28;   /* llama2.c header: 7 ints */
    for (int i = 0; i < PT_MAX_BINDS; i++)
        if (g_binds[i].dev && g_binds[i].image == image) return i;
    for (int i = 0; i < PT_MAX_BINDS; i++) {
        if (g_binds[i].dev) continue;
        train_bind_t *b = &g_binds[i];
        b->image = image;
        b->cfg = *cfg;
        b->shared = ((const int *)image)[5] > 0;
        b->max_T = max_T;
        b->dev = pt_device_open(image, pt_file_size(image), 28, cfg, w, 1, 1, pt_pick_device(-1), 0, max_T);
        b->dev->trainer = ptc_trainer_create(b->dev->ctx, &b->dev->cfg, &b->dev->dw, max_T, 1, 1);
        ptc_trainer_zero_grads(b->dev->trainer);
        return i;
    }
    pt_fatal("too many training images (max %d)", PT_MAX_BINDS);
    return -1;
}

static void attach(int oi, int bi) {
    if (g_owned[oi].bind == bi) return;
    if (g_owned[oi].bind >= 0) pt_fatal("a training struct is already bound to another model image");
    g_owned[oi].bind = bi;
}

static void attach_grads(pt_grads_t *g, int bi) {
    int oi = owned_find(g);
    if (oi < 0) pt_fatal("pt_grads_t %p was not allocated by pt_alloc_grads", (void *)g);
    if (g_owned[oi].bind == bi) return;
    if (g_binds[bi].g && g_binds[bi].g != g) pt_fatal("a second pt_grads_t for the same model image");
    attach(oi, bi);
    g_binds[bi].g = g;
    if (g_owned[oi].zero_pending) ptc_trainer_zero_grads(g_binds[bi].dev->trainer);
    g_owned[oi].zero_pending = 0;
}

/* The binding of an owned struct, binding it through `w` if it has none. */
static int bind_struct(const void *s, const char *what, const pt_config_t *cfg, const pt_weights_t *w) {
    int oi = owned_find(s);
    if (oi < 0) pt_fatal("%s %p was not allocated by pt_alloc_* nor is a context member", what, s);
    if (g_owned[oi].bind >= 0) return g_owned[oi].bind;
    if (!w) pt_fatal("%s used before any call that names its weights", what);
    int bi = bind_of_weights(cfg, w, g_owned[oi].T);
    attach(oi, bi);
    return bi;
}

static ptc_trainer *bind_trainer(int bi) { return g_binds[bi].dev->trainer; }
static ptc_ctx *bind_ctx(int bi) { return g_binds[bi].dev->ctx; }

static void check_T(int bi, int T) {
    if (T < 1 || T > g_binds[bi].max_T)
        pt_fatal("training T=%d outside [1, %d] (the T the structs were allocated for)", T, g_binds[bi].max_T);
}

static void put_rows(int bi, float *dev, const float *host, int T) {
    ptc_h2d(bind_ctx(bi), dev, host, (size_t)T * g_binds[bi].cfg.dim * 4);
}
static void get_rows(int bi, float *host, const float *dev, int T) {
    ptc_d2h(bind_ctx(bi), host, dev, (size_t)T * g_binds[bi].cfg.dim * 4);
}

/* Copy device tensors [off, off + n) floats of the image back to the host. */
static void pull_image(int bi, const float *host_tensor, size_t n_floats) {
    struct pt_device *d = g_binds[bi].dev;
    if (!host_tensor || !n_floats) return;
    ptc_d2h(d->ctx, (void *)host_tensor, pt_dev_ptr(d, host_tensor), n_floats * 4);
}

/* After SGD on layers [l0, l1) and/or the head: the updated tensors back
 * into the caller's image. */
static void pull_weights(int bi, const pt_weights_t *w, int l0, int l1, int head) {
    const pt_config_t *c = &g_binds[bi].cfg;
    size_t D = c->dim, H = c->hidden_dim;
    size_t K = (size_t)c->n_kv_heads * (c->dim / c->n_heads);
    size_t n = (size_t)(l1 - l0);
    if (n > 0) {
        pull_image(bi, w->rms_att_weight + l0 * D, n * D);
        pull_image(bi, w->wq + l0 * D * D, n * D * D);
        pull_image(bi, w->wk + l0 * K * D, n * K * D);
        pull_image(bi, w->wv + l0 * K * D, n * K * D);
        pull_image(bi, w->wo + l0 * D * D, n * D * D);
        pull_image(bi, w->rms_ffn_weight + l0 * D, n * D);
        pull_image(bi, w->w1 + l0 * H * D, n * H * D);
        pull_image(bi, w->w2 + l0 * D * H, n * D * H);
        pull_image(bi, w->w3 + l0 * H * D, n * H * D);
    }
    if (head) {
        pull_image(bi, w->token_embedding, (size_t)c->vocab_size * D);
        pull_image(bi, w->rms_final_weight, D);
        if (!g_binds[bi].shared) pull_image(bi, w->wcls, (size_t)c->vocab_size * D);
    }
}

/* Gradients of layers [l0, l1) (and of the embedding/head when `rest`) into
 * g->_mem, which has the device buffer's layout. */
static void pull_grads(int bi, int l0, int l1, int rest) {
    pt_grads_t *g = g_binds[bi].g;
    if (!g || !g->_mem) return;
    ptc_trainer *t = bind_trainer(bi);
    ptc_trainer_sync(t);
    const float *dg = ptc_trainer_grads(t);
    if (rest) {
        ptc_d2h(bind_ctx(bi), g->_mem, dg, (size_t)g->_n_params * 4);
        return;
    }
    const pt_config_t *c = &g_binds[bi].cfg;
    size_t D = c->dim, H = c->hidden_dim;
    size_t K = (size_t)c->n_kv_heads * (c->dim / c->n_heads);
    size_t n = (size_t)(l1 - l0);
    float *const parts[9] = {g->rms_att_weight, g->wq, g->wk, g->wv, g->wo, g->rms_ffn_weight, g->w1, g->w2, g->w3};
    const size_t per[9] = {D, D * D, K * D, K * D, D * D, D, H * D, D * H, H * D};
    for (int k = 0; k < 9; k++) {
        float *h = parts[k] + l0 * per[k];
        ptc_d2h(bind_ctx(bi), h, dg + (h - g->_mem), n * per[k] * 4);
    }
}

void pt_alloc_activations(pt_activations_t *a, const pt_config_t *cfg, int T) {
    size_t D = cfg->dim, H = cfg->hidden_dim, L = cfg->n_layers, nh = cfg->n_heads, V = cfg->vocab_size;
    size_t K = (size_t)cfg->n_kv_heads * (cfg->dim / cfg->n_heads), t = (size_t)T;
    memset(a, 0, sizeof(*a));
    a->T = T;
    a->residuals = (float *)calloc((L + 1) * t * D, 4);
    a->residuals_att = (float *)calloc(L * t * D, 4);
    a->xb_att = (float *)calloc(L * t * D, 4);
    a->q = (float *)calloc(L * t * D, 4);
    a->k = (float *)calloc(L * t * K, 4);
    a->v = (float *)calloc(L * t * K, 4);
    a->att = (float *)calloc(L * nh * t * t, 4);
    a->att_out = (float *)calloc(L * t * D, 4);
    a->xb_ffn = (float *)calloc(L * t * D, 4);
    a->hb = (float *)calloc(L * t * H, 4);
    a->hb2 = (float *)calloc(L * t * H, 4);
    a->x_final = (float *)calloc(t * D, 4);
    a->logits = (float *)calloc(t * V, 4);
    a->scratch = (float *)calloc(H > D ? H : D, 4);
    owned_add(a, T);
}

void pt_free_activations(pt_activations_t *a) {
    owned_remove(a);
    free(a->residuals); free(a->residuals_att); free(a->xb_att); free(a->q); free(a->k); free(a->v);
    free(a->att); free(a->att_out); free(a->xb_ffn); free(a->hb); free(a->hb2); free(a->x_final);
    free(a->logits); free(a->scratch);
    memset(a, 0, sizeof(*a));
}

/* Gradient layout of pt_train.c:334-371 (tied classifier: wcls aliases the
 * embedding gradient), the layout of the device trainer's buffer. */
void pt_alloc_grads(pt_grads_t *g, const pt_config_t *cfg, int shared_weights) {
    size_t D = cfg->dim, H = cfg->hidden_dim, L = cfg->n_layers, V = cfg->vocab_size;
    size_t K = (size_t)cfg->n_kv_heads * (cfg->dim / cfg->n_heads);
    size_t n = V * D + L * (2 * D + 2 * D * D + 2 * K * D + 3 * H * D) + D + (shared_weights ? 0 : V * D);
    memset(g, 0, sizeof(*g));
    g->_mem = (float *)calloc(n, 4);
    g->_n_params = (int)n;
    float *p = g->_mem;
    g->token_embedding = p; p += V * D;
    g->rms_att_weight = p; p += L * D;
    g->wq = p; p += L * D * D;
    g->wk = p; p += L * K * D;
    g->wv = p; p += L * K * D;
    g->wo = p; p += L * D * D;
    g->rms_ffn_weight = p; p += L * D;
    g->w1 = p; p += L * H * D;
    g->w2 = p; p += L * D * H;
    g->w3 = p; p += L * H * D;
    g->rms_final_weight = p; p += D;
    g->wcls = shared_weights ? g->token_embedding : p;
    owned_add(g, 0);
}

void pt_free_grads(pt_grads_t *g) {
    int oi = owned_find(g);
    if (oi >= 0 && g_owned[oi].bind >= 0 && g_binds[g_owned[oi].bind].g == g) g_binds[g_owned[oi].bind].g = NULL;
    owned_remove(g);
    free(g->_mem);
    memset(g, 0, sizeof(*g));
}

void pt_alloc_backward_buf(pt_backward_buf_t *b, const pt_config_t *cfg, int T) {
    size_t D = cfg->dim, H = cfg->hidden_dim, V = cfg->vocab_size, t = (size_t)T;
    size_t K = (size_t)cfg->n_kv_heads * (cfg->dim / cfg->n_heads);
    size_t wt = V * D > H * D ? V * D : H * D;
    memset(b, 0, sizeof(*b));
    b->d_res = (float *)calloc(t * D, 4);
    b->d_aout = (float *)calloc(t * D, 4);
    b->d_q = (float *)calloc(t * D, 4);
    b->d_k = (float *)calloc(t * K, 4);
    b->d_v = (float *)calloc(t * K, 4);
    b->d_logit = (float *)calloc(V, 4);
    b->d_xb = (float *)calloc(D, 4);
    b->d_qpre = (float *)calloc(D, 4);
    b->d_kpre = (float *)calloc(K, 4);
    b->d_hid = (float *)calloc(H, 4);
    b->d_hid2 = (float *)calloc(H, 4);
    b->sh = (float *)calloc(H, 4);
    b->d_att_s = (float *)calloc(t, 4);
    b->d_pre_sm = (float *)calloc(t, 4);
    b->w_transpose = (float *)calloc(wt, 4);
    b->d_temp = (float *)calloc(H > D ? H : D, 4);
    b->d_logit_all = (float *)calloc(t * V, 4);
    b->drt_wo_all = (float *)calloc(t * D, 4);
    b->d_qpre_all = (float *)calloc(t * D, 4);
    b->d_kpre_all = (float *)calloc(t * K, 4);
    b->sh_all = (float *)calloc(t * H, 4);
    b->d_hid_all = (float *)calloc(t * H, 4);
    b->d_hid2_all = (float *)calloc(t * H, 4);
    b->drt_ffn_all = (float *)calloc(t * D, 4);
    owned_add(b, T);
}

void pt_free_backward_buf(pt_backward_buf_t *b) {
    owned_remove(b);
    float *const bufs[] = {b->d_res, b->d_aout, b->d_q, b->d_k, b->d_v, b->d_logit, b->d_xb, b->d_qpre,
                           b->d_kpre, b->d_hid, b->d_hid2, b->sh, b->d_att_s, b->d_pre_sm, b->w_transpose,
                           b->d_temp, b->d_logit_all, b->drt_wo_all, b->d_qpre_all, b->d_kpre_all, b->sh_all,
                           b->d_hid_all, b->d_hid2_all, b->drt_ffn_all};
    for (size_t i = 0; i < sizeof(bufs) / sizeof(bufs[0]); i++) free(bufs[i]);
    memset(b, 0, sizeof(*b));
}

/* Context-member structs (pt_pi_init / pt_host_init with max_T > 0) run on
 * the context's trainer with no host hand-off; caller-owned ones as above. */
static pt_context_t *member_ctx(const void *member) {
    for (int i = 0; i < PT_MAX_TRAIN_CTX; i++) {
        pt_context_t *c = g_train_ctx[i];
        if (c && (member == (const void *)&c->acts || member == (const void *)&c->grads ||
                  member == (const void *)&c->bb || member == (const void *)&c->w))
            return c;
    }
    return NULL;
}

void pt_zero_grads(pt_grads_t *g) {
    pt_context_t *ctx = member_ctx(g);
    if (ctx) {
        ptc_trainer_zero_grads(trainer(ctx));
        if (g->_mem) memset(g->_mem, 0, (size_t)g->_n_params * 4);
        return;
    }
    int oi = owned_find(g);
    if (oi < 0) pt_fatal("pt_grads_t %p was not allocated by pt_alloc_grads nor is a context member", (void *)g);
    if (g_owned[oi].bind >= 0) ptc_trainer_zero_grads(bind_trainer(g_owned[oi].bind));
    else g_owned[oi].zero_pending = 1;
    if (g->_mem) memset(g->_mem, 0, (size_t)g->_n_params * 4);
}

/* ---- whole-model passes (pt_train.h:66-159) -------------------------------- */

float pt_forward_train(const pt_config_t *cfg, const pt_weights_t *w, pt_activations_t *a,
                       const int *tokens, int T, pt_matvec_fn matvec, pt_trace_t *trace) {
    (void)matvec;
    pt_context_t *ctx = member_ctx(a);
    ptc_trainer *t;
    int n_layers;
    if (ctx) {
        t = trainer(ctx);
        n_layers = ctx->cfg.n_layers;
    } else {
        int bi = bind_struct(a, "pt_activations_t", cfg, w);
        check_T(bi, T);
        t = bind_trainer(bi);
        n_layers = g_binds[bi].cfg.n_layers;
    }
    pt_trace_begin(trace, "forward", "fwd", -1);
    ptc_trainer_set_tokens(t, tokens, T);
    ptc_trainer_fwd_embed(t);
    ptc_trainer_fwd_layers(t, 0, n_layers);
    float loss = ptc_trainer_fwd_head(t);
    pt_trace_end(trace);
    a->T = T;
    return loss;
}

void pt_backward(const pt_config_t *cfg, const pt_weights_t *w, pt_grads_t *g, const pt_activations_t *a,
                 pt_backward_buf_t *b, const int *tokens, int T, pt_matvec_fn matvec, pt_trace_t *trace) {
    (void)matvec;
    pt_context_t *ctx = member_ctx(a);
    ptc_trainer *t;
    int n_layers, bi = -1;
    if (ctx) {
        t = trainer(ctx);
        n_layers = ctx->cfg.n_layers;
    } else {
        bi = bind_struct(a, "pt_activations_t", cfg, w);
        attach_grads(g, bi);
        int ob = owned_find(b);
        if (ob < 0) pt_fatal("pt_backward_buf_t %p was not allocated by pt_alloc_backward_buf", (void *)b);
        attach(ob, bi);
        t = bind_trainer(bi);
        n_layers = g_binds[bi].cfg.n_layers;
    }
    pt_trace_begin(trace, "backward", "bwd", -1);
    ptc_trainer_set_tokens(t, tokens, T);
    ptc_trainer_bwd_head(t);
    ptc_trainer_bwd_layers(t, 0, n_layers);
    ptc_trainer_bwd_embed(t);
    ptc_trainer_sync(t);
    if (bi >= 0) pull_grads(bi, 0, 0, 1);
    pt_trace_end(trace);
}

/* SGD through the gradients' binding (context member or caller-owned). */
static void sgd(pt_weights_t *w, const pt_grads_t *g, float lr, const pt_config_t *cfg, int l0, int l1, int head,
                const char *what) {
    pt_context_t *ctx = member_ctx(g);
    if (ctx) {
        ptc_trainer *t = trainer(ctx);
        if (head) ptc_trainer_sgd_head(t, lr);
        if (l1 > l0) ptc_trainer_sgd_layers(t, lr, l0, l1);
        ptc_trainer_sync(t);
        ptc_decoder_weights_updated(ctx->dev->dec);
        return;
    }
    int bi = bind_struct(g, what, cfg, w);
    if (l0 < 0 || l1 > g_binds[bi].cfg.n_layers || l0 > l1)
        pt_fatal("%s: layer range [%d, %d) outside [0, %d)", what, l0, l1, g_binds[bi].cfg.n_layers);
    ptc_trainer *t = bind_trainer(bi);
    if (head) ptc_trainer_sgd_head(t, lr);
    if (l1 > l0) ptc_trainer_sgd_layers(t, lr, l0, l1);
    ptc_trainer_sync(t);
    ptc_decoder_weights_updated(g_binds[bi].dev->dec);
    pull_weights(bi, w, l0, l1, head);
}

void pt_sgd_update(pt_weights_t *w, const pt_grads_t *g, float lr, const pt_config_t *cfg) {
    pt_context_t *ctx = member_ctx(g);
    sgd(w, g, lr, cfg, 0, ctx ? ctx->cfg.n_layers : cfg->n_layers, 1, "pt_grads_t");
}

void pt_sgd_update_layers(pt_weights_t *w, const pt_grads_t *g, float lr, const pt_config_t *cfg,
                          int l_start, int l_end) {
    sgd(w, g, lr, cfg, l_start, l_end, 0, "pt_grads_t");
}

void pt_sgd_update_head(pt_weights_t *w, const pt_grads_t *g, float lr, const pt_config_t *cfg) {
    sgd(w, g, lr, cfg, 0, 0, 1, "pt_grads_t");
}

/* ---- staged passes for pipeline parallelism (pt_train.h:174-224) ---------- */

void pt_forward_train_embed(const pt_weights_t *w, pt_activations_t *a, const int *tokens, int T, int dim) {
    (void)dim;
    pt_context_t *ctx = member_ctx(a);
    if (ctx) {
        ptc_trainer *t = trainer(ctx);
        ptc_trainer_set_tokens(t, tokens, T);
        ptc_trainer_fwd_embed(t);
        ptc_trainer_sync(t);
        a->T = T;
        return;
    }
    int oi = owned_find(a);
    if (oi < 0) pt_fatal("pt_activations_t %p was not allocated by pt_alloc_activations", (void *)a);
    pt_config_t c;
    const char *image = (const char *)w->token_embedding - 28;
    pt_load_config(&c, image);
    int bi = bind_struct(a, "pt_activations_t", &c, w);
    check_T(bi, T);
    ptc_trainer *t = bind_trainer(bi);
    ptc_trainer_set_tokens(t, tokens, T);
    ptc_trainer_fwd_embed(t);
    ptc_trainer_sync(t);
    get_rows(bi, a->residuals, ptc_trainer_residual(t, 0), T);
    a->T = T;
}

void pt_forward_train_layers_range(const pt_config_t *cfg, const pt_weights_t *w, pt_activations_t *a, int T,
                                   int l_start, int l_end, pt_matvec_fn matvec, pt_trace_t *trace) {
    (void)matvec; (void)trace;
    pt_context_t *ctx = member_ctx(a);
    if (ctx) {
        ptc_trainer *t = trainer(ctx);
        if (T != a->T) pt_fatal("pt_forward_train_layers_range: T=%d but activations hold T=%d", T, a->T);
        ptc_trainer_fwd_layers(t, l_start, l_end);
        ptc_trainer_sync(t);
        return;
    }
    int bi = bind_struct(a, "pt_activations_t", cfg, w);
    check_T(bi, T);
    if (l_start < 0 || l_end > g_binds[bi].cfg.n_layers || l_start > l_end)
        pt_fatal("layer range [%d, %d) outside [0, %d)", l_start, l_end, g_binds[bi].cfg.n_layers);
    ptc_trainer *t = bind_trainer(bi);
    /* the layer range's input may have been written by the caller (the hand-off) */
    ptc_trainer_set_T(t, T);
    put_rows(bi, ptc_trainer_residual(t, l_start), a->residuals + (size_t)l_start * T * g_binds[bi].cfg.dim, T);
    ptc_trainer_fwd_layers(t, l_start, l_end);
    ptc_trainer_sync(t);
    get_rows(bi, a->residuals + (size_t)l_end * T * g_binds[bi].cfg.dim, ptc_trainer_residual(t, l_end), T);
    a->T = T;
}

float pt_forward_train_head(const pt_config_t *cfg, const pt_weights_t *w, pt_activations_t *a,
                            const int *tokens, int T, pt_matvec_fn matvec, pt_trace_t *trace) {
    (void)matvec; (void)trace;
    pt_context_t *ctx = member_ctx(a);
    if (ctx) {
        ptc_trainer *t = trainer(ctx);
        ptc_trainer_set_tokens(t, tokens, T);
        a->T = T;
        return ptc_trainer_fwd_head(t);
    }
    int bi = bind_struct(a, "pt_activations_t", cfg, w);
    check_T(bi, T);
    ptc_trainer *t = bind_trainer(bi);
    const int L = g_binds[bi].cfg.n_layers;
    ptc_trainer_set_tokens(t, tokens, T);
    put_rows(bi, ptc_trainer_residual(t, L), a->residuals + (size_t)L * T * g_binds[bi].cfg.dim, T);
    a->T = T;
    return ptc_trainer_fwd_head(t);
}

void pt_backward_head(const pt_config_t *cfg, const pt_weights_t *w, pt_grads_t *g, const pt_activations_t *a,
                      pt_backward_buf_t *b, const int *tokens, int T, pt_matvec_fn matvec, pt_trace_t *trace) {
    (void)matvec; (void)trace;
    pt_context_t *ctx = member_ctx(a);
    if (ctx) {
        ptc_trainer *t = trainer(ctx);
        ptc_trainer_set_tokens(t, tokens, T);
        ptc_trainer_bwd_head(t);
        ptc_trainer_sync(t);
        return;
    }
    int bi = bind_struct(a, "pt_activations_t", cfg, w);
    check_T(bi, T);
    attach_grads(g, bi);
    int ob = owned_find(b);
    if (ob < 0) pt_fatal("pt_backward_buf_t %p was not allocated by pt_alloc_backward_buf", (void *)b);
    attach(ob, bi);
    ptc_trainer *t = bind_trainer(bi);
    ptc_trainer_set_tokens(t, tokens, T);
    ptc_trainer_bwd_head(t);
    ptc_trainer_sync(t);
    get_rows(bi, b->d_res, ptc_trainer_dres(t), T);
}

void pt_backward_layers_range(const pt_config_t *cfg, const pt_weights_t *w, pt_grads_t *g,
                              const pt_activations_t *a, pt_backward_buf_t *b, int T, int l_start, int l_end,
                              pt_matvec_fn matvec, pt_trace_t *trace) {
    (void)matvec; (void)trace;
    pt_context_t *ctx = member_ctx(a);
    if (ctx) {
        ptc_trainer_bwd_layers(trainer(ctx), l_start, l_end);
        ptc_trainer_sync(trainer(ctx));
        return;
    }
    int bi = bind_struct(a, "pt_activations_t", cfg, w);
    check_T(bi, T);
    if (l_start < 0 || l_end > g_binds[bi].cfg.n_layers || l_start > l_end)
        pt_fatal("layer range [%d, %d) outside [0, %d)", l_start, l_end, g_binds[bi].cfg.n_layers);
    attach_grads(g, bi);
    int ob = owned_find(b);
    if (ob < 0) pt_fatal("pt_backward_buf_t %p was not allocated by pt_alloc_backward_buf", (void *)b);
    attach(ob, bi);
    ptc_trainer *t = bind_trainer(bi);
    ptc_trainer_set_T(t, T);
    put_rows(bi, ptc_trainer_dres(t), b->d_res, T);
    ptc_trainer_bwd_layers(t, l_start, l_end);
    ptc_trainer_sync(t);
    get_rows(bi, b->d_res, ptc_trainer_dres(t), T);
    pull_grads(bi, l_start, l_end, 0);
}

void pt_backward_embed(pt_grads_t *g, const pt_backward_buf_t *b, const int *tokens, int T, int dim) {
    (void)dim;
    pt_context_t *ctx = member_ctx(g);
    if (ctx) {
        ptc_trainer *t = trainer(ctx);
        ptc_trainer_set_tokens(t, tokens, T);
        ptc_trainer_bwd_embed(t);
        ptc_trainer_sync(t);
        return;
    }
    int bi = bind_struct(g, "pt_grads_t", NULL, NULL);
    check_T(bi, T);
    int ob = owned_find(b);
    if (ob < 0) pt_fatal("pt_backward_buf_t %p was not allocated by pt_alloc_backward_buf", (void *)b);
    attach(ob, bi);
    ptc_trainer *t = bind_trainer(bi);
    ptc_trainer_set_tokens(t, tokens, T);
    put_rows(bi, ptc_trainer_dres(t), b->d_res, T);
    ptc_trainer_bwd_embed(t);
    ptc_trainer_sync(t);
    pull_grads(bi, 0, 0, 1);
}
