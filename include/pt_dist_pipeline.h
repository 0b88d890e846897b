#ifndef PT_DIST_PIPELINE_H
#define PT_DIST_PIPELINE_H

/*
 * Layer-pipeline API -- drop-in for pitorch/dist/pt_dist_pipeline.h.
 * All ranks call the same function; the implementation dispatches on
 * dist->has_embed / dist->has_head. Every call is synchronous on return.
 * Waits are bounded by dist->timeout_ms: a rank whose peer never answers
 * prints a "FAIL:" line (pt_dist_pipeline.c:87-90, 160-163) and the call
 * returns -1 (forward) or a result with total_ms == 0 (training) instead of
 * rebooting the board.
 */

#include "pt.h"
#include "pt_dist.h"

/* pitorch/dist/pt_dist_pipeline.h:71-72. Also joins the ring: rank 0
 * creates the NCCL unique id and hands it to the others over TCP at
 * $MASTER_ADDR:$PT_DIST_PORT (default $MASTER_PORT + 17, else 29517), then
 * every rank initialises its communicator on the context's device.
 * `ctx` is needed for the device; pass the context initialised from this
 * rank's shard. Returns 0, or -1 when the rendezvous times out. */
int pt_dist_setup_ctx(pt_dist_t *dist, pt_context_t *ctx, const pt_shard_info_t *shard,
                      int rank, int world_size);
/* Reference signature: configures the fields only; the communicator is
 * created on the first pipeline call (with the device of that call's ctx). */
void pt_dist_setup(pt_dist_t *dist, const pt_shard_info_t *shard, int rank, int world_size);

/* pitorch/dist/pt_dist_pipeline.h:81: a ring barrier (every rank returns
 * once all ranks joined). Returns 0 or -1 on timeout. */
int pt_dist_ring_sync(pt_dist_t *dist);

/* Decode hop transport in use once joined (no reference counterpart):
 * 1 = stores into the successor's memory over NVLink (ptc_hop_*),
 * 0 = NCCL send/recv, -1 = not joined. */
int pt_dist_transport(const pt_dist_t *dist);

/* pitorch/dist/pt_dist_pipeline.h:88 -- nothing to reset on NVLink; kept. */
void pt_dist_reset_links(pt_dist_t *dist);

/* pitorch/dist/pt_dist_pipeline.h:102 */
void pt_dist_set_verbose(pt_dist_t *dist, int verbose);

/* pitorch/dist/pt_dist_pipeline.h:107-110 */
typedef struct {
    float    loss;
    unsigned total_ms;
} pt_dist_result_t;

/* pitorch/dist/pt_dist_pipeline.h:120-121 (pt_dist_pipeline.c:128-278). */
pt_dist_result_t pt_dist_train_step(pt_context_t *ctx, pt_dist_t *dist,
                                    const int *tokens, int T, float lr);

/* pitorch/dist/pt_dist_pipeline.h:133 (pt_dist_pipeline.c:284-372).
 * Embed+head rank: returns the greedy next token; layer ranks return 0;
 * -1 on a communication timeout. */
int pt_dist_forward_step(pt_context_t *ctx, pt_dist_t *dist, int token);


/* ---- pitorch_b200 additions ---- */

/* Device-resident pipelined greedy decode of n_pos positions on every rank
 * (no host round trip per token): the head rank teacher-forces the prompt
 * and feeds each argmax back into its embedding on the GPU. Every rank must
 * call it with the same n_pos; only the head rank reads prompt and writes
 * out_tokens. Resets the KV caches first. Returns 0 or -1 on timeout. */
int pt_dist_generate_greedy(pt_context_t *ctx, pt_dist_t *dist, const int *prompt,
                            int n_prompt, int n_pos, int *out_tokens);

/* GPipe microbatched pipeline training step: the schedule the reference
 * runs by hand in dev/tests/dist/train_pp/test_train_pp_mb_rank{0,1}.c
 * (it has no library call for it). n_mb microbatches of T tokens each
 * (tokens holds n_mb * T ids, microbatch m at tokens + m * T) go forward
 * through the ring one after another, so neighbouring ranks work on
 * different microbatches at once; then backward in reverse order with the
 * gradients accumulated; then ONE SGD update with lr (the reference's test
 * passes lr / n_mb for the effective step of one microbatch). Every rank
 * calls it with the same T and n_mb (1 <= n_mb <= 16); only the head rank
 * reads tokens. The head rank returns the mean loss over the microbatches;
 * total_ms = 0 on a communication failure. */
pt_dist_result_t pt_dist_train_step_mb(pt_context_t *ctx, pt_dist_t *dist, const int *tokens, int T, int n_mb,
                                       float lr);

/* Data-parallel gradient averaging: after it, every rank holds the mean of
 * all ranks' gradients (pitorch/dist/collective/pt_allreduce.c:50-165, a
 * 2-rank GPIO protocol; here ncclAllReduce with ncclAvg on the device
 * gradients of ctx). Returns 0 or -1 on timeout. */
int pt_dist_allreduce_grads_avg(pt_context_t *ctx, pt_dist_t *dist);

/* Ranks in the NCCL communicator of a joined ring (ncclCommCount), or -1. */
int pt_dist_comm_size(const pt_dist_t *dist);

/* Vocab-parallel classifier (no reference counterpart: the reference's head
 * rank computes every vocab row, pitorch/model/llama2.c:194-198). After it,
 * every rank computes the logits of its 1/world share of the classifier rows
 * on the final residual, and the argmax is combined across ranks on the GPU
 * (ptc_decoder_set_vocab_parallel); token streams are unchanged. Collective:
 * every rank calls it once, after pt_dist_setup_ctx (or with a pt_dist_setup
 * ring, which it joins). Needs the NVLink hop transport and the reference's
 * shard layout (layers on ranks 0..world-2, embedding + classifier on the
 * last). Returns 0, or -1 with nothing changed when that does not hold or a
 * transfer timed out. Afterwards, in host-driven steps (pt_dist_forward_step)
 * every rank must set ctx->sync_logits alike: with it set, the head gathers
 * the other ranks' logits. */
int pt_dist_vocab_parallel(pt_context_t *ctx, pt_dist_t *dist);
/* 1 once pt_dist_vocab_parallel succeeded on this ring, else 0. */
int pt_dist_is_vocab_parallel(const pt_dist_t *dist);

/* Largest value of `v` over all ranks (for max-over-ranks timing). */
float pt_dist_max_float(pt_context_t *ctx, pt_dist_t *dist, float v);

/* Leave the ring (destroys the communicator). */
void pt_dist_free(pt_dist_t *dist);

/* The TCP rendezvous used by pt_dist_setup, exposed for tests: rank 0
 * sends `blob` (128 bytes) to ranks 1..world-1, which receive it. Returns 0
 * or -1 when a peer does not connect/answer within timeout_ms. */
int pt_dist_rendezvous(int rank, int world_size, const char *addr, int port, int timeout_ms,
                       unsigned char blob[128]);

#endif
