#ifndef PITORCH_LLAMA2_H
#define PITORCH_LLAMA2_H

/*
 * Llama-2 model types and the decode forward pass -- drop-in for
 * pitorch/model/llama2.h. Same structs, field names and call signatures;
 * the arithmetic runs on the GPU (libpitorch_b200).
 *
 * Weight format: karpathy/llama2.c .bin (28-byte header, then tensors in the
 * order of pt_weights_t, freq_cis skipped; a negative vocab_size means an
 * untied classifier follows), as in pitorch/model/llama2.c:9-70.
 */

/* pitorch/model/llama2.h:10-18 */
typedef struct {
    int dim;
    int hidden_dim;
    int n_layers;
    int n_heads;
    int n_kv_heads;
    int vocab_size;
    int seq_len;
} pt_config_t;

/* pitorch/model/llama2.h:20-33 (HOST pointers into the caller's .bin blob) */
typedef struct {
    float *token_embedding;   /* [vocab_size, dim] */
    float *rms_att_weight;    /* [n_layers, dim] */
    float *wq;                /* [n_layers, dim, dim] */
    float *wk;                /* [n_layers, kv_dim, dim] */
    float *wv;                /* [n_layers, kv_dim, dim] */
    float *wo;                /* [n_layers, dim, dim] */
    float *rms_ffn_weight;    /* [n_layers, dim] */
    float *w1;                /* [n_layers, hidden_dim, dim] */
    float *w2;                /* [n_layers, dim, hidden_dim] */
    float *w3;                /* [n_layers, hidden_dim, dim] */
    float *rms_final_weight;  /* [dim] */
    float *wcls;              /* [vocab_size, dim] (may alias token_embedding) */
} pt_weights_t;

/* pitorch/model/llama2.h:35-48. In this build the live decode state
 * (including the KV cache) is on the GPU; after each forward call `x` and
 * `logits` hold host copies of the device values (logits only when the
 * owning context has sync_logits set). key_cache/value_cache are host
 * buffers of the reference's size kept for API compatibility (zero, never
 * written by the library); pt_reset_kv resets the device cache. */
typedef struct {
    float *x;
    float *xb;
    float *xb2;
    float *q;
    float *k;
    float *v;
    float *hb;
    float *hb2;
    float *att;
    float *logits;
    float *key_cache;
    float *value_cache;
} pt_state_t;

/* pitorch/model/llama2.h:50-54 */
void pt_load_config(pt_config_t *cfg, const void *data);
void pt_load_weights(pt_weights_t *w, const pt_config_t *cfg, void *data);

typedef void *(*pt_bump_alloc_fn)(unsigned bytes);

/* pitorch/model/llama2.h:59-63. Allocates the host-side state and binds it
 * to a device decode state on first use by pt_forward*. */
void pt_alloc_state(pt_state_t *s, const pt_config_t *cfg);
void pt_free_state(pt_state_t *s);

/* pitorch/model/llama2.h:70-71 */
unsigned pt_file_size(const void *data);

/* pitorch/model/llama2.h:73-75: y = W @ x, W is [out_dim, in_dim] row-major. */
typedef void (*pt_matvec_fn)(const float *W, const float *x, float *y,
                             int out_dim, int in_dim);

/* The GPU matvec with the pt_matvec_fn contract (host pointers, sync);
 * this build's ctx.matvec. Replaces the Pi's matvec_gpu (pitorch/pt.c:21-25). */
void pt_matvec_gpu(const float *W, const float *x, float *y, int out_dim, int in_dim);

/* pitorch/model/llama2.h:79-95. `matvec` is accepted for signature
 * compatibility; the GPU decode kernels are always used. */
void pt_forward(const pt_config_t *cfg, const pt_weights_t *w,
                pt_state_t *s, int token, int pos, pt_matvec_fn matvec);
void pt_forward_embed(const pt_weights_t *w, float *x, int dim, int token);
void pt_forward_layers_range(const pt_config_t *cfg, const pt_weights_t *w,
                             pt_state_t *s, int pos, int l_start, int l_end,
                             pt_matvec_fn matvec);
void pt_forward_head(const pt_config_t *cfg, const pt_weights_t *w,
                     pt_state_t *s, pt_matvec_fn matvec);

/* argmax with the reference's tie rule (first maximum, pitorch/ops/core/pt_ops.c:65-70). */
int pt_argmax(const float *x, int n);

#endif
