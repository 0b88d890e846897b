#ifndef PITORCH_TRAIN_H
#define PITORCH_TRAIN_H

/*
 * Training types and passes -- drop-in for pitorch/train/pt_train.h.
 * Same structs and signatures. In this build the activations, gradients and
 * backward buffers live on the GPU (allocated by pt_pi_init / pt_host_init
 * with max_T > 0); the host structs carry the sizes, and grads._mem is a
 * host mirror filled by pt_sync_grads() (pt.h). The staged functions run on
 * the GPU buffers of the context that owns the passed structs.
 */

#include "llama2.h"
#include "trace.h"

/* pitorch/train/pt_train.h:34-50 */
typedef struct {
    float *residuals;
    float *residuals_att;
    float *xb_att;
    float *q;
    float *k;
    float *v;
    float *att;
    float *att_out;
    float *xb_ffn;
    float *hb;
    float *hb2;
    float *x_final;
    float *logits;
    float *scratch;
    int T;
} pt_activations_t;

void pt_alloc_activations(pt_activations_t *a, const pt_config_t *cfg, int T);
void pt_free_activations(pt_activations_t *a);

/* pitorch/train/pt_train.h:66-68 */
float pt_forward_train(const pt_config_t *cfg, const pt_weights_t *w,
                       pt_activations_t *a, const int *tokens, int T,
                       pt_matvec_fn matvec, pt_trace_t *trace);

/* pitorch/train/pt_train.h:76-86 */
typedef struct {
    float *token_embedding;
    float *rms_att_weight;
    float *wq, *wk, *wv, *wo;
    float *rms_ffn_weight;
    float *w1, *w2, *w3;
    float *rms_final_weight;
    float *wcls;
    float *_mem;
    int _n_params;
} pt_grads_t;

void pt_alloc_grads(pt_grads_t *g, const pt_config_t *cfg, int shared_weights);
void pt_free_grads(pt_grads_t *g);
void pt_zero_grads(pt_grads_t *g);

/* pitorch/train/pt_train.h:103-129 */
typedef struct {
    float *d_res;
    float *d_aout;
    float *d_q;
    float *d_k;
    float *d_v;
    float *d_logit;
    float *d_xb;
    float *d_qpre;
    float *d_kpre;
    float *d_hid;
    float *d_hid2;
    float *sh;
    float *d_att_s;
    float *d_pre_sm;
    float *w_transpose;
    float *d_temp;
    float *d_logit_all;
    float *drt_wo_all;
    float *d_qpre_all;
    float *d_kpre_all;
    float *sh_all;
    float *d_hid_all;
    float *d_hid2_all;
    float *drt_ffn_all;
} pt_backward_buf_t;

void pt_alloc_backward_buf(pt_backward_buf_t *b, const pt_config_t *cfg, int T);
void pt_free_backward_buf(pt_backward_buf_t *b);

/* pitorch/train/pt_train.h:151-166 */
void pt_backward(const pt_config_t *cfg, const pt_weights_t *w,
                 pt_grads_t *g, const pt_activations_t *a,
                 pt_backward_buf_t *b, const int *tokens, int T,
                 pt_matvec_fn matvec, pt_trace_t *trace);
void pt_sgd_update(pt_weights_t *w, const pt_grads_t *g, float lr, const pt_config_t *cfg);
void pt_sgd_update_layers(pt_weights_t *w, const pt_grads_t *g, float lr,
                          const pt_config_t *cfg, int l_start, int l_end);
void pt_sgd_update_head(pt_weights_t *w, const pt_grads_t *g, float lr, const pt_config_t *cfg);

/* pitorch/train/pt_train.h:174-224 (staged, for pipeline parallelism) */
void pt_forward_train_embed(const pt_weights_t *w, pt_activations_t *a,
                            const int *tokens, int T, int dim);
void pt_forward_train_layers_range(const pt_config_t *cfg, const pt_weights_t *w,
                                   pt_activations_t *a, int T, int l_start, int l_end,
                                   pt_matvec_fn matvec, pt_trace_t *trace);
float pt_forward_train_head(const pt_config_t *cfg, const pt_weights_t *w,
                            pt_activations_t *a, const int *tokens, int T,
                            pt_matvec_fn matvec, pt_trace_t *trace);
void pt_backward_head(const pt_config_t *cfg, const pt_weights_t *w,
                      pt_grads_t *g, const pt_activations_t *a,
                      pt_backward_buf_t *b, const int *tokens, int T,
                      pt_matvec_fn matvec, pt_trace_t *trace);
void pt_backward_layers_range(const pt_config_t *cfg, const pt_weights_t *w,
                              pt_grads_t *g, const pt_activations_t *a,
                              pt_backward_buf_t *b, int T, int l_start, int l_end,
                              pt_matvec_fn matvec, pt_trace_t *trace);
void pt_backward_embed(pt_grads_t *g, const pt_backward_buf_t *b,
                       const int *tokens, int T, int dim);

#endif
