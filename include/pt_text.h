#ifndef PITORCH_TEXT_H
#define PITORCH_TEXT_H

/*
 * Text layer -- drop-in for pitorch/text/pt_text.h: tokenizer.bin parsing,
 * BPE encode / piece decode, the xorshift sampler (greedy, temperature,
 * top-p) and the pt_generate loop. Host string work; each position's
 * forward pass runs on the GPU, and with temperature 0 the argmax is taken
 * on the GPU without copying the logits back.
 *
 * tokenizer.bin: [u32 max_token_length] then per token
 * [f32 score][u32 len][len bytes] (dev/host/export_tokenizer.py:1-10).
 */

#include <stdint.h>

#include "llama2.h"

typedef struct {
    char *str;
    int id;
} pt_token_index_t;

/* pitorch/text/pt_text.h:19-27 */
typedef struct {
    char **vocab;
    float *vocab_scores;
    int vocab_size;
    int max_token_length;
    int sorted_ready;
    pt_token_index_t *sorted_vocab;
} pt_tokenizer_t;

/* pitorch/text/pt_text.h:30-44 */
void pt_tokenizer_init(pt_tokenizer_t *t, const void *data, int vocab_size);
void pt_load_tokenizer(pt_tokenizer_t *t, const void *combined_file, int vocab_size);
const char *pt_decode(pt_tokenizer_t *t, int prev_token, int token);
void pt_encode(pt_tokenizer_t *t, const char *text, int bos, int eos, int *tokens, int *n_tokens);
/* Release the tokenizer's tables (this build allocates them per tokenizer). */
void pt_tokenizer_free(pt_tokenizer_t *t);

/* pitorch/text/pt_text.h:48-58 */
typedef struct {
    int vocab_size;
    float temperature;
    float topp;
    uint64_t rng_state;
} pt_sampler_t;

void pt_sampler_init(pt_sampler_t *s, int vocab_size, float temp, float topp, uint64_t seed);
int pt_sample(pt_sampler_t *s, float *logits);

/* pitorch/text/pt_text.h:62-64. `s` must be a state created by
 * pt_alloc_state or the state of a context (its device twin runs the
 * forward passes); `matvec` is accepted for signature compatibility. */
void pt_generate(const pt_config_t *cfg, const pt_weights_t *w, pt_state_t *s,
                 pt_tokenizer_t *tok, pt_sampler_t *sampler,
                 const char *prompt, int max_tokens, pt_matvec_fn matvec);

#endif
