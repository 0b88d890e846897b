/*
 * pt_oracle.h -- TEST INFRASTRUCTURE ONLY.
 *
 * CPU restatement of pitorch's host algorithm for the decode/train hot path,
 * used by tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg as
 * the parity checker. Nothing in the product library links or calls this.
 *
 * Parity is pinned: tests/test_oracle_pins.py checks this restatement
 * bit-for-bit against the reference's own host C (compiled into
 * oracle/_ref/libptref.so by oracle/Makefile) and against the golden
 * vectors of the reference's op tests (tests/golden/).
 *
 * Every function cites the reference file:line whose arithmetic it restates,
 * in the same operation order, so that gcc -O2 -ffp-contract=off gives the
 * same float results as the reference built the same way.
 */
#ifndef PT_ORACLE_H
#define PT_ORACLE_H

#ifdef __cplusplus
extern "C" {
#endif

/* libm-free math (pitorch/ops/core/pt_math.c) */
float or_expf(float x);
float or_logf(float x);
float or_sinf(float x);
float or_cosf(float x);
float or_sqrtf(float x);

/* elementwise ops (pitorch/ops/core/pt_ops.c) */
void or_rmsnorm(float *o, const float *x, const float *w, int dim);
void or_softmax(float *x, int n);
void or_silu(float *x, int n);
void or_rope(float *q, float *k, int dim, int head_dim, int pos);
int  or_argmax(const float *x, int n);
void or_matvec(const float *W, const float *x, float *y, int rows, int cols);

/* backward primitives (pitorch/train/pt_backward_ops.c) */
void or_rmsnorm_backward(float *dx, float *dw, const float *dout,
                         const float *x, const float *w, int dim);
void or_rope_backward(float *dq, float *dk, const float *dq_out,
                      const float *dk_out, int dim, int head_dim, int pos);
void or_softmax_backward(float *dx, const float *dy, const float *y, int n);

/* ---- whole-model oracle ------------------------------------------------ */

typedef struct or_model or_model;

/* blob: llama2.c .bin contents (28-byte header + tensors). The oracle keeps
 * its own copy, so training never mutates the caller's buffer.
 * max_T > 0 allocates training buffers for sequences up to max_T. */
or_model *or_open(const void *blob, long blob_bytes, int max_T);
void      or_close(or_model *m);
void      or_config(const or_model *m, int out[7]);   /* dim,hidden,L,H,KV,V,seq */
void      or_reset_kv(or_model *m);

/* One decode position over all layers (pitorch/model/llama2.c:298-303).
 * Leaves logits inside the model; or_logits() returns them. */
void         or_forward(or_model *m, int token, int pos);
const float *or_logits(const or_model *m);
const float *or_x(const or_model *m);

/* Staged decode (pitorch/model/llama2.c:220-295) for pipeline parity. */
void or_forward_embed(or_model *m, int token);
void or_forward_layers_range(or_model *m, int pos, int l0, int l1);
void or_forward_head(or_model *m);
void or_set_x(or_model *m, const float *x);

/* Teacher-forced prompt then greedy argmax for n_pos positions, as
 * pt_forward_step is driven by the reference's decode loops
 * (pitorch/pt.c:267-271, pitorch/text/pt_text.c:338-361 without the
 * BOS/EOS stop). tokens_out[p] = token emitted at position p.
 * logits_out (nullable) receives n_pos * vocab floats. */
void or_decode_greedy(or_model *m, const int *prompt, int n_prompt, int n_pos,
                      int *tokens_out, float *logits_out);

/* zero_grads -> forward_train -> backward -> sgd (pitorch/pt.c:339-364). */
float or_train_step(or_model *m, const int *tokens, int T, float lr);

/* Forward-only training loss over T tokens (pitorch/train/pt_train.c:171-329). */
float or_forward_train(or_model *m, const int *tokens, int T);

/* Read back current (possibly trained) weights in .bin layout. */
const void *or_blob(const or_model *m);
long        or_blob_bytes(const or_model *m);
/* Gradient buffer after the last or_train_step (pt_grads_t._mem layout). */
const float *or_grads(const or_model *m, long *n_out);

#ifdef __cplusplus
}
#endif
#endif
