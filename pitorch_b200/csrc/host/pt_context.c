/*
 * pt_context.c -- the pitorch context API (pitorch/pt.c) on a B200.
 *
 * pt_pi_init / pt_host_init upload the caller's .bin image once into the
 * context's device arena (pitorch/pt.c:38-114 placed state after the weights
 * in Pi RAM; here all state lives in the device arena) and create a decoder
 * whose step is a captured CUDA graph. The low-level staged functions of
 * llama2.h run the same kernels eagerly on the state's device twin.
 */
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "pt_device.h"

void pt_fatal(const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    fprintf(stderr, "pitorch_b200: fatal: ");
    vfprintf(stderr, fmt, ap);
    fprintf(stderr, "\n");
    va_end(ap);
    abort();
}

int pt_pick_device(int requested) {
    int n = ptc_device_count();
    if (n <= 0) pt_fatal("no CUDA device visible; pitorch_b200 has no CPU path");
    if (requested >= 0 && requested < n) return requested;
    const char *e = getenv("PT_DEVICE");
    if (e) {
        int d = atoi(e);
        if (d >= 0 && d < n) return d;
    }
    return 0;
}

const float *pt_dev_ptr(const struct pt_device *d, const float *host) {
    if (!host) return NULL;
    const char *h = (const char *)host;
    if (h < d->host_image || h >= d->host_image + d->image_bytes)
        pt_fatal("weight pointer %p is outside the uploaded image", (const void *)host);
    return (const float *)(d->dev_image + (h - d->host_image));
}

struct pt_device *pt_device_open(const void *image, size_t image_bytes, size_t header_bytes,
                                 const pt_config_t *local_cfg, const pt_weights_t *host_w,
                                 int has_embed, int has_head, int device, size_t arena_bytes,
                                 int max_T) {
    (void)max_T;
    struct pt_device *d = (struct pt_device *)calloc(1, sizeof(*d));
    size_t hd = (size_t)local_cfg->dim / local_cfg->n_heads;
    size_t kv = 2ull * local_cfg->n_layers * local_cfg->seq_len * local_cfg->n_kv_heads * hd * 4;
    size_t need = image_bytes + kv + (8ull << 20) + (size_t)local_cfg->vocab_size * 8;
    if (arena_bytes < need) arena_bytes = need;
    d->ctx = ptc_create(device, arena_bytes);
    d->owns_ctx = 1;
    d->host_image = (const char *)image;
    d->image_bytes = image_bytes;
    d->dev_image = (char *)ptc_upload_image(d->ctx, image, image_bytes, header_bytes);
    memcpy(&d->cfg, local_cfg, sizeof(ptc_config));
    d->dw.token_embedding = pt_dev_ptr(d, host_w->token_embedding);
    d->dw.rms_att_weight = pt_dev_ptr(d, host_w->rms_att_weight);
    d->dw.wq = pt_dev_ptr(d, host_w->wq);
    d->dw.wk = pt_dev_ptr(d, host_w->wk);
    d->dw.wv = pt_dev_ptr(d, host_w->wv);
    d->dw.wo = pt_dev_ptr(d, host_w->wo);
    d->dw.rms_ffn_weight = pt_dev_ptr(d, host_w->rms_ffn_weight);
    d->dw.w1 = pt_dev_ptr(d, host_w->w1);
    d->dw.w2 = pt_dev_ptr(d, host_w->w2);
    d->dw.w3 = pt_dev_ptr(d, host_w->w3);
    d->dw.rms_final_weight = pt_dev_ptr(d, host_w->rms_final_weight);
    d->dw.wcls = pt_dev_ptr(d, host_w->wcls);
    d->has_embed = has_embed;
    d->has_head = has_head;
    d->dec = ptc_decoder_create(d->ctx, &d->cfg, &d->dw, has_embed, has_head);
    return d;
}

void pt_device_close(struct pt_device *d) {
    if (!d) return;
    ptc_decoder_destroy(d->dec);
    if (d->owns_ctx) ptc_destroy(d->ctx);
    free(d);
}

/* ---- state registry: which device state backs a host pt_state_t ----------- */

#define PT_MAX_STATES 64
static struct {
    pt_state_t *s;
    struct pt_device *dev;
    int owned;          /* device created lazily for a pt_alloc_state state */
} g_states[PT_MAX_STATES];

static void bind_state(pt_state_t *s, struct pt_device *dev, int owned) {
    for (int i = 0; i < PT_MAX_STATES; i++)
        if (g_states[i].s == s || !g_states[i].s) {
            g_states[i].s = s;
            g_states[i].dev = dev;
            g_states[i].owned = owned;
            return;
        }
    pt_fatal("too many live decode states (max %d)", PT_MAX_STATES);
}

static int find_state(const pt_state_t *s) {
    for (int i = 0; i < PT_MAX_STATES; i++)
        if (g_states[i].s == s) return i;
    return -1;
}

static void unbind_state(const pt_state_t *s) {
    int i = find_state(s);
    if (i < 0) return;
    if (g_states[i].owned && g_states[i].dev) pt_device_close(g_states[i].dev);
    g_states[i].s = NULL;
    g_states[i].dev = NULL;
    g_states[i].owned = 0;
}

static void alloc_host_state(pt_state_t *s, const pt_config_t *cfg) {
    size_t hd = (size_t)cfg->dim / cfg->n_heads;
    size_t kvd = (size_t)cfg->n_kv_heads * hd;
    s->x = (float *)calloc(cfg->dim, 4);
    s->xb = (float *)calloc(cfg->dim, 4);
    s->xb2 = (float *)calloc(cfg->dim, 4);
    s->q = (float *)calloc(cfg->dim, 4);
    s->k = (float *)calloc(kvd, 4);
    s->v = (float *)calloc(kvd, 4);
    s->hb = (float *)calloc(cfg->hidden_dim, 4);
    s->hb2 = (float *)calloc(cfg->hidden_dim, 4);
    s->att = (float *)calloc((size_t)cfg->n_heads * cfg->seq_len, 4);
    s->logits = (float *)calloc(cfg->vocab_size, 4);
    size_t kv = (size_t)cfg->n_layers * cfg->seq_len * kvd;
    s->key_cache = (float *)calloc(kv ? kv : 1, 4);
    s->value_cache = (float *)calloc(kv ? kv : 1, 4);
}

static void free_host_state(pt_state_t *s) {
    free(s->x); free(s->xb); free(s->xb2); free(s->q); free(s->k); free(s->v);
    free(s->hb); free(s->hb2); free(s->att); free(s->logits);
    free(s->key_cache); free(s->value_cache);
    memset(s, 0, sizeof(*s));
}

/* llama2.h:59-63 */
void pt_alloc_state(pt_state_t *s, const pt_config_t *cfg) {
    alloc_host_state(s, cfg);
    bind_state(s, NULL, 1);
}

void pt_free_state(pt_state_t *s) {
    unbind_state(s);
    free_host_state(s);
}

/* The device twin of a host state; created on first use for states from
 * pt_alloc_state, from the image that `w` points into. */
struct pt_device *pt_state_device(const pt_config_t *cfg, const pt_weights_t *w, pt_state_t *s) {
    int i = find_state(s);
    if (i < 0) pt_fatal("pt_state_t %p was not created by pt_alloc_state / pt_*_init", (void *)s);
    if (g_states[i].dev) return g_states[i].dev;
    /* w->token_embedding is the first tensor of a full .bin (header 28 bytes) */
    const char *base = (const char *)w->token_embedding - 28;
    size_t bytes = pt_file_size(base);
    g_states[i].dev = pt_device_open(base, bytes, 28, cfg, w, 1, 1, pt_pick_device(-1), 0, 0);
    return g_states[i].dev;
}

/* ---- context init / free ---------------------------------------------------- */

static void init_common(pt_context_t *ctx, int max_T) {
    ctx->matvec = pt_matvec_gpu;
    ctx->max_T = max_T;
    ctx->sync_logits = 1;
    alloc_host_state(&ctx->state, &ctx->cfg);
    bind_state(&ctx->state, ctx->dev, 0);
}

void pt_train_init(pt_context_t *ctx, int max_T);   /* pt_train_api.c */
void pt_train_free(pt_context_t *ctx);

void pt_pi_init(pt_context_t *ctx, void *weight_data, int num_qpus, int max_T, unsigned arena_bytes) {
    memset(ctx, 0, sizeof(*ctx));
    int dim0 = *(const int *)weight_data;
    if (dim0 <= 0 || dim0 > 65536) pt_fatal("no weights at %p (dim=%d)", weight_data, dim0);
    pt_load_config(&ctx->cfg, weight_data);
    ctx->shared_weights = ((const int *)weight_data)[5] > 0;
    pt_load_weights(&ctx->w, &ctx->cfg, weight_data);
    int dev = pt_pick_device(num_qpus);
    ctx->num_qpus = dev;
    ctx->dev = pt_device_open(weight_data, pt_file_size(weight_data), 28, &ctx->cfg, &ctx->w, 1, 1,
                              dev, arena_bytes, max_T);
    init_common(ctx, max_T);
    if (max_T > 0) pt_train_init(ctx, max_T);
}

void pt_host_init(pt_context_t *ctx, void *weight_data, int max_T) {
    pt_pi_init(ctx, weight_data, -1, max_T, 0);
}

void pt_pi_init_shard(pt_context_t *ctx, pt_shard_info_t *shard_out, void *shard_data, int num_qpus,
                      int max_T, unsigned arena_bytes) {
    memset(ctx, 0, sizeof(*ctx));
    memset(shard_out, 0, sizeof(*shard_out));
    int dim0 = *(const int *)shard_data;
    if (dim0 <= 0 || dim0 > 65536) pt_fatal("no shard at %p (dim=%d)", shard_data, dim0);
    pt_config_t global_cfg;
    pt_load_shard_header(&global_cfg, shard_out, shard_data);
    ctx->shared_weights = ((const int *)shard_data)[5] > 0;
    pt_load_shard_weights(&ctx->w, &global_cfg, shard_out, shard_data);
    ctx->cfg = global_cfg;
    ctx->cfg.n_layers = shard_out->n_local;   /* pt.c:151-152 */
    int dev = pt_pick_device(num_qpus);
    ctx->num_qpus = dev;
    ctx->dev = pt_device_open(shard_data, pt_shard_file_size(shard_data), 56, &ctx->cfg, &ctx->w,
                              shard_out->has_embed, shard_out->has_head, dev, arena_bytes, max_T);
    ctx->dev->is_shard = 1;
    ctx->dev->shard = *shard_out;
    init_common(ctx, max_T);
    if (max_T > 0) pt_train_init(ctx, max_T);
}

void pt_free(pt_context_t *ctx) {
    if (ctx->max_T > 0) pt_train_free(ctx);
    unbind_state(&ctx->state);
    free_host_state(&ctx->state);
    if (ctx->dev) pt_device_close(ctx->dev);
    ctx->dev = NULL;
    if (ctx->trace) {
        free(ctx->trace);
        ctx->trace = NULL;
    }
}

struct ptc_ctx *pt_ptc_ctx(pt_context_t *ctx) { return ctx->dev ? ctx->dev->ctx : NULL; }
struct ptc_decoder *pt_ptc_decoder(pt_context_t *ctx) { return ctx->dev ? ctx->dev->dec : NULL; }
struct ptc_trainer *pt_ptc_trainer(pt_context_t *ctx) { return ctx->dev ? ctx->dev->trainer : NULL; }

/* ---- decode ------------------------------------------------------------------ */

/* pt.c:267-271 */
int pt_forward_step(pt_context_t *ctx, int token) {
    struct pt_device *d = ctx->dev;
    if (!d) pt_fatal("pt_forward_step on an uninitialised context");
    if (!d->has_embed || !d->has_head)
        pt_fatal("pt_forward_step needs embedding and head; use pt_dist_forward_step on shards");
    pt_trace_begin(ctx->trace, "forward_step", "fwd", -1);
    int next = ptc_decoder_step(d->dec, token, ctx->pos, ctx->sync_logits ? ctx->state.logits : NULL);
    pt_trace_end(ctx->trace);
    ctx->pos++;
    return next;
}

/* pt.c:273-280. The cache that decodes read is the device one; the host
 * key_cache/value_cache buffers are never written by this library (they stay
 * as calloc left them), so clearing them -- 75 MB and ~10 ms for stories110M
 * -- is skipped. */
void pt_reset_kv(pt_context_t *ctx) {
    if (ctx->dev) ptc_decoder_reset(ctx->dev->dec);
    ctx->pos = 0;
}

void pt_generate_greedy(pt_context_t *ctx, const int *prompt, int n_prompt, int n_pos, int *out_tokens) {
    struct pt_device *d = ctx->dev;
    if (!d || !d->has_embed || !d->has_head) pt_fatal("pt_generate_greedy needs a full-model context");
    ptc_decoder_generate(d->dec, prompt, n_prompt, n_pos, out_tokens);
    ctx->pos = n_pos;
}

/* pt.c:282-305 */
void pt_print_config(const pt_context_t *ctx) {
    const pt_config_t *c = &ctx->cfg;
    printf("pitorch (%dd %dL %dKv) | B200 cuda:%d\n", c->dim, c->n_layers, c->vocab_size / 1000,
           ctx->num_qpus);
    printf("  dim=%d hidden=%d L=%d H=%d kv=%d V=%d seq=%d\n", c->dim, c->hidden_dim, c->n_layers,
           c->n_heads, c->n_kv_heads, c->vocab_size, c->seq_len);
    if (ctx->max_T > 0) printf("  training: max_T=%d\n", ctx->max_T);
}

/* pt.c:310-322 */
void *pt_read_file(const char *path, long *out_size) {
    FILE *f = fopen(path, "rb");
    if (!f) { perror(path); exit(1); }
    fseek(f, 0, SEEK_END);
    long sz = ftell(f);
    fseek(f, 0, SEEK_SET);
    void *buf = malloc(sz);
    if (fread(buf, 1, sz, f) != (size_t)sz) { perror(path); exit(1); }
    fclose(f);
    if (out_size) *out_size = sz;
    return buf;
}

/* pt.c:326-340 */
void pt_enable_trace(pt_context_t *ctx, pt_trace_t *preallocated) {
    ctx->trace = preallocated ? preallocated : (pt_trace_t *)malloc(sizeof(pt_trace_t));
    if (ctx->trace) pt_trace_init(ctx->trace);
}

void pt_disable_trace(pt_context_t *ctx) {
    if (ctx->trace) ctx->trace->enabled = 0;
}

void pt_matvec_gpu(const float *W, const float *x, float *y, int out_dim, int in_dim) {
    ptc_matvec_host(W, x, y, out_dim, in_dim);
}

/* ---- low-level staged forward (llama2.h) on a state's device twin ----------- */

void pt_forward(const pt_config_t *cfg, const pt_weights_t *w, pt_state_t *s, int token, int pos,
                pt_matvec_fn matvec) {
    (void)matvec;
    struct pt_device *d = pt_state_device(cfg, w, s);
    if (!d->has_embed || !d->has_head) pt_fatal("pt_forward needs a full model; use the staged calls");
    (void)ptc_decoder_step(d->dec, token, pos, s->logits);
    ptc_decoder_get_xnorm(d->dec, s->x);
}

/* llama2.c:220-222 -- a row copy out of the caller's (host) embedding table. */
void pt_forward_embed(const pt_weights_t *w, float *x, int dim, int token) {
    memcpy(x, w->token_embedding + (size_t)token * dim, (size_t)dim * 4);
}

void pt_forward_layers_range(const pt_config_t *cfg, const pt_weights_t *w, pt_state_t *s, int pos,
                             int l_start, int l_end, pt_matvec_fn matvec) {
    (void)matvec;
    struct pt_device *d = pt_state_device(cfg, w, s);
    ptc_decoder_set_x(d->dec, s->x);
    ptc_decoder_enqueue_layers(d->dec, pos, l_start, l_end);
    ptc_decoder_get_x(d->dec, s->x);
}

void pt_forward_head(const pt_config_t *cfg, const pt_weights_t *w, pt_state_t *s, pt_matvec_fn matvec) {
    (void)matvec;
    struct pt_device *d = pt_state_device(cfg, w, s);
    if (!d->has_head) pt_fatal("pt_forward_head on a state without the classifier");
    ptc_decoder_set_x(d->dec, s->x);
    ptc_decoder_enqueue_head(d->dec);
    (void)ptc_decoder_fetch_next(d->dec, s->logits);
    ptc_decoder_get_xnorm(d->dec, s->x);
}
