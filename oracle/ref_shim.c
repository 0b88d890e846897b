/*
 * ref_shim.c -- TEST INFRASTRUCTURE ONLY.
 *
 * Compiled together with the reference's own, unmodified host C sources
 * (pitorch/pt.c host branch, model/, ops/core/, train/, profiler/trace.c,
 * text/pt_text.c) into oracle/_ref/libptref.so by oracle/Makefile. It only
 * adds ctypes-friendly entry points around the reference's public API; all
 * arithmetic is the reference's.
 */
#include <stdlib.h>
#include <string.h>

#include "pt.h"
#include "pt_ops.h"

typedef struct {
    pt_context_t ctx;
    void *blob;
} ref_handle;

/* pt_host_init on a private copy of the .bin blob (pt.c:232-248). */
void *ref_open(const void *blob, long bytes, int max_T) {
    ref_handle *h = (ref_handle *)calloc(1, sizeof(ref_handle));
    h->blob = malloc((size_t)bytes);
    memcpy(h->blob, blob, (size_t)bytes);
    pt_host_init(&h->ctx, h->blob, max_T);
    return h;
}

void ref_close(void *p) {
    ref_handle *h = (ref_handle *)p;
    if (!h) return;
    pt_free(&h->ctx);
    free(h->blob);
    free(h);
}

void ref_reset_kv(void *p) { pt_reset_kv(&((ref_handle *)p)->ctx); }

/* pt_forward_step (pt.c:267-271). */
int ref_forward_step(void *p, int token) {
    return pt_forward_step(&((ref_handle *)p)->ctx, token);
}

const float *ref_logits(void *p) { return ((ref_handle *)p)->ctx.state.logits; }

/* pt_train_step (pt.c:339-364). */
float ref_train_step(void *p, const int *tokens, int T, float lr) {
    return pt_train_step(&((ref_handle *)p)->ctx, tokens, T, lr);
}

const void *ref_blob(void *p) { return ((ref_handle *)p)->blob; }

const float *ref_grads(void *p, long *n) {
    ref_handle *h = (ref_handle *)p;
    if (n) *n = h->ctx.grads._n_params;
    return h->ctx.grads._mem;
}

/* Prefill + greedy loop as the reference's host harnesses drive it
 * (dev/host/test_generate_host.c:60-72), without the BOS/EOS stop. */
void ref_decode_greedy(void *p, const int *prompt, int n_prompt, int n_pos,
                       int *tokens_out, float *logits_out) {
    ref_handle *h = (ref_handle *)p;
    pt_reset_kv(&h->ctx);
    int V = h->ctx.cfg.vocab_size;
    int tok = prompt[0];
    for (int pos = 0; pos < n_pos; pos++) {
        int greedy = pt_forward_step(&h->ctx, tok);
        if (logits_out) memcpy(logits_out + (size_t)pos * V, h->ctx.state.logits, V * sizeof(float));
        int next = (pos + 1 < n_prompt) ? prompt[pos + 1] : greedy;
        tokens_out[pos] = next;
        tok = next;
    }
}

/* Staged forward on the context's own state (llama2.c:220-295), for the
 * pipeline (layer-range) parity fixtures. */
void ref_forward_embed(void *p, int token) {
    ref_handle *h = (ref_handle *)p;
    pt_forward_embed(&h->ctx.w, h->ctx.state.x, h->ctx.cfg.dim, token);
}
void ref_forward_layers_range(void *p, int pos, int l0, int l1) {
    ref_handle *h = (ref_handle *)p;
    pt_forward_layers_range(&h->ctx.cfg, &h->ctx.w, &h->ctx.state, pos, l0, l1, h->ctx.matvec);
}
void ref_forward_head(void *p) {
    ref_handle *h = (ref_handle *)p;
    pt_forward_head(&h->ctx.cfg, &h->ctx.w, &h->ctx.state, h->ctx.matvec);
}
float *ref_x(void *p) { return ((ref_handle *)p)->ctx.state.x; }

/* smatvec_cpu (pt_ops.c:72-80). */
void ref_matvec(const float *W, const float *x, float *y, int out_dim, int in_dim) {
    smatvec_cpu(W, x, y, out_dim, in_dim);
}
