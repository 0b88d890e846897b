/*
 * ptc.h -- the thin C ABI between pitorch_b200's C host layer and its
 * sm_100a CUDA kernels. Plain pointers, ints and sizes only; no CUDA or
 * C++ types cross it (streams are passed as void *).
 *
 * The pitorch-compatible API (pt.h, llama2.h, pt_train.h, pt_shard.h,
 * pt_text.h, pt_dist_pipeline.h) is implemented in C on top of these calls.
 * Each entry point names the reference interface it replaces.
 *
 * Error convention: CUDA failures print the call site and abort(), the host
 * analogue of the reference's panic() (pitorch/runtime/gpu.c:107-108). Only
 * the communication waits return an error code (-1), as the reference's
 * recv_raw does on timeout (pitorch/dist/transport/pt_link_gpio.c:134-136).
 */
#ifndef PTC_H
#define PTC_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- runtime: replaces pitorch/runtime/{gpu.c,arena.c} ------------------ */

typedef struct ptc_ctx ptc_ctx;

/* Number of CUDA devices visible to this process. */
int ptc_device_count(void);

/* Open a context on `device`: its own stream and ONE device arena of
 * `arena_bytes` (bump-allocated, 256-byte aligned), replacing
 * qpu_enable + gpu_arena_init (pitorch/runtime/gpu.c:75-103, arena.c:10-16).
 * arena_bytes == 0 picks a size large enough for the caller's later
 * requests (the arena then grows in chunks instead). */
ptc_ctx *ptc_create(int device, size_t arena_bytes);
void ptc_destroy(ptc_ctx *c);

/* Bump allocation from the arena (gpu_arena_alloc, arena.c:18-26). */
void *ptc_alloc(ptc_ctx *c, size_t bytes);
/* Arena high-water mark and reset to a mark (gpu_arena_reset, arena.c:28-31). */
size_t ptc_arena_used(const ptc_ctx *c);
void ptc_arena_reset(ptc_ctx *c, size_t mark);

void *ptc_stream(ptc_ctx *c);
int ptc_device(const ptc_ctx *c);
int ptc_sm_count(const ptc_ctx *c);
void ptc_sync(ptc_ctx *c);
void ptc_h2d(ptc_ctx *c, void *dst, const void *src, size_t bytes);
void ptc_d2h(ptc_ctx *c, void *dst, const void *src, size_t bytes);
void ptc_d2d(ptc_ctx *c, void *dst, const void *src, size_t bytes);
void ptc_memset(ptc_ctx *c, void *dst, int value, size_t bytes);

/* Page-locked host buffers for the staged copies of the drop-in paths. */
void *ptc_host_alloc(size_t bytes);
void ptc_host_free(void *p);

/* Upload a llama2.c .bin image (or a SHRD shard) into the arena so that the
 * first tensor (at byte offset `header_bytes`) starts 256-byte aligned.
 * Returns the device address of byte 0 of the image. The host keeps the
 * mapping host_base -> device_base (pitorch/pt.c:56-58 points pt_weights_t
 * into the caller's blob; the device copy keeps the same offsets). */
void *ptc_upload_image(ptc_ctx *c, const void *image, size_t bytes, size_t header_bytes);

/* ---- matvec: replaces smatvec_tmu (pitorch/ops/matvec/matvec.c:13-86) ---- */

/* y = W . x, W row-major [rows, cols], all DEVICE pointers, on `stream`
 * (NULL = legacy default stream). Any shape; 128-bit path when cols % 4 == 0
 * and W/x are 16-byte aligned. Asynchronous. */
void ptc_matvec(const float *W, const float *x, float *y, int rows, int cols, void *stream);

/* Measurement hook (no reference counterpart): stream `bytes` (a multiple
 * of 16, 16-byte aligned) of DEVICE memory through L2-only loads with
 * 4 CTAs per SM, on `stream`. Timed over a buffer that fits in L2 and was
 * just read, it gives the L2 read bandwidth the matvec sweep's hot shapes
 * are compared with; over a buffer larger than L2, the HBM read bandwidth.
 * `sink` is a device float the kernel may write. */
void ptc_read_probe(const void *buf, size_t bytes, float *sink, void *stream);

/* Same contract as pitorch's pt_matvec_fn callback (llama2.h:74-75) and the
 * Pi's matvec_gpu wrapper (pt.c:21-25): HOST pointers, synchronous. W is
 * looked up among images uploaded with ptc_upload_image (and the registered
 * transposed-weight scratch); an unknown W is staged to the device first.
 * x is staged in, y copied back. */
void ptc_matvec_host(const float *W, const float *x, float *y, int rows, int cols);

/* Register / unregister a host range whose device copy ptc_matvec_host may
 * use instead of staging (the host-base -> device-base map). */
void ptc_register_range(const void *host, const void *dev, size_t bytes, ptc_ctx *owner);
void ptc_unregister_ctx(ptc_ctx *owner);

/* ---- decode: replaces pt_forward / pt_forward_layers_range /
 *      pt_forward_head + argmax (pitorch/model/llama2.c:220-303,
 *      pitorch/pt.c:267-271) ---------------------------------------------- */

typedef struct ptc_decoder ptc_decoder;

/* Model shape, same field order as pt_config_t (llama2.h:10-18). */
typedef struct {
    int dim, hidden_dim, n_layers, n_heads, n_kv_heads, vocab_size, seq_len;
} ptc_config;

/* DEVICE weight pointers, same field order as pt_weights_t (llama2.h:20-33).
 * Per-layer tensors hold `n_layers` (local) layers; absent parts are NULL. */
typedef struct {
    const float *token_embedding, *rms_att_weight, *wq, *wk, *wv, *wo,
        *rms_ffn_weight, *w1, *w2, *w3, *rms_final_weight, *wcls;
} ptc_weights;

/* A decoder owns the decode state (residual x, q, attention output, FFN
 * hidden, logits, KV cache [L][n_kv][seq][hd]) and two captured CUDA graphs
 * of one position: layers [0, n_layers) of `w`, preceded by the embedding
 * lookup when has_embed and followed by the head (final rmsnorm, classifier,
 * argmax) when has_head. */
ptc_decoder *ptc_decoder_create(ptc_ctx *c, const ptc_config *cfg, const ptc_weights *w,
                                int has_embed, int has_head);
void ptc_decoder_destroy(ptc_decoder *d);

/* Zero the KV cache and the device position (pt_reset_kv,
 * pitorch/pt.c:273-280). */
void ptc_decoder_reset(ptc_decoder *d);

/* One position. Input: `token` when has_embed, else the residual stream
 * previously set with ptc_decoder_set_x. Returns the argmax token when
 * has_head (else -1). If logits_host is non-NULL the vocab logits are
 * copied there. Synchronous. */
int ptc_decoder_step(ptc_decoder *d, int token, int pos, float *logits_host);

/* Residual stream access (the [pos | x] hand-off of the pipeline,
 * pitorch/dist/pt_dist_pipeline.c:296-357). */
void ptc_decoder_set_x(ptc_decoder *d, const float *x_host);
void ptc_decoder_get_x(ptc_decoder *d, float *x_host);
/* Final-normalised x left by the head (pt_forward_head normalises s->x in
 * place, llama2.c:293). */
void ptc_decoder_get_xnorm(ptc_decoder *d, float *x_host);
float *ptc_decoder_x_dev(ptc_decoder *d);
float *ptc_decoder_logits_dev(ptc_decoder *d);

/* Staged pieces, enqueued on the context stream without synchronising
 * (pt_forward_embed / pt_forward_layers_range / pt_forward_head,
 * llama2.c:220-295). Layer indices are local to the decoder's weights.
 * ptc_decoder_fetch_next synchronises and returns the last head's argmax. */
void ptc_decoder_enqueue_embed(ptc_decoder *d, int token);
void ptc_decoder_enqueue_layers(ptc_decoder *d, int pos, int l_start, int l_end);
void ptc_decoder_enqueue_head(ptc_decoder *d);
int ptc_decoder_fetch_next(ptc_decoder *d, float *logits_host);

/* Device-resident greedy decode of positions [0, n_pos): prompt tokens are
 * teacher-forced, then argmax feeds back on the device (no host round
 * trip per token). out_tokens[p] = token emitted at position p (host). */
void ptc_decoder_generate(ptc_decoder *d, const int *prompt, int n_prompt, int n_pos,
                          int *out_tokens);

/* Benchmark hooks: enqueue the device-loop step graph n times without
 * synchronising (inputs already resident), and time it with CUDA events on
 * the decoder's stream. ptc_decoder_generate_begin loads the prompt and
 * resets position 0. */
void ptc_decoder_generate_begin(ptc_decoder *d, const int *prompt, int n_prompt);
void ptc_decoder_enqueue_steps(ptc_decoder *d, int n);
void ptc_decoder_read_tokens(ptc_decoder *d, int *out_tokens, int n);

/* Pipeline hand-off: device addresses of the step's position / input token,
 * and layer / embedding launches that take them from the device (set by a
 * received message or by the previous head) instead of from the host. */
int *ptc_decoder_pos_dev(ptc_decoder *d);
/* Host steps of a pipeline's embedding rank with one wait per step: the
 * position and token through the decoder's pinned block (the decoder's
 * previous host-step work must have completed) and the embedding lookup
 * enqueued; then the copies of the argmax, the decode kernels' error word
 * and (logits != 0) the logits into pinned memory enqueued; and, once the
 * caller has waited for the stream, the argmax taken (an error word aborts,
 * as in ptc_decoder_fetch_next). */
void ptc_decoder_enqueue_embed_at(ptc_decoder *d, int token, int pos);
void ptc_decoder_enqueue_fetch(ptc_decoder *d, int logits);
int ptc_decoder_take_next(ptc_decoder *d, float *logits_host);
int *ptc_decoder_tok_dev(ptc_decoder *d);
void ptc_decoder_enqueue_layers_devpos(ptc_decoder *d, int l_start, int l_end);
void ptc_decoder_enqueue_embed_dev(ptc_decoder *d);
/* Timing hook (no reference counterpart): enqueue ONE kernel of the decode
 * step at position pos -- kind 0: layer l's attention block, 1: layer l's
 * FFN block, 2: the classifier head -- on the residual buffers of a full
 * decode. The decode state it leaves is not meaningful: call
 * ptc_decoder_reset before decoding again. */
void ptc_decoder_enqueue_kernel(ptc_decoder *d, int kind, int l, int pos);
/* Kernels one decode position launches (2 per layer + head when the layer
 * blocks are fused, 5 per layer + head otherwise). */
int ptc_decoder_launches_per_step(ptc_decoder *d);
/* Stream helpers for the pipeline's bounded waits: 0 = all queued work on
 * the context stream finished, 1 = still running after timeout_ms. */
int ptc_wait_deadline(ptc_ctx *c, int timeout_ms);

/* Pipeline links of a layer-range decoder (no reference counterpart: the
 * reference passes [pos | x] between boards over GPIO, pt_dist_pipeline.c:
 * 287-357). in_box is this rank's mailbox (ptc_mailbox_alloc; the previous
 * stage writes it), out_box the next stage's mailbox mapped from its owner
 * (ptc_mailbox_open), sent a device counter of the messages this rank has
 * sent on its link (shared with ptc_hop_send), err a device error word
 * (1: a wait ran out after timeout_ns on the GPU, 2: a message for another
 * position) and timeout_ns the bound of each wait. With links set, the
 * decoder captures stage graphs in which a layer rank's first attention
 * block and the embedding+head rank's classifier take x from in_box
 * themselves (no receive kernel), and in device-loop mode the classifier's
 * last CTA sends the next token's embedding row to out_box (no embedding or
 * send kernel). in_box NULL removes the links. Synchronises the decoder's
 * stream and re-captures its graphs. */
void ptc_decoder_set_links(ptc_decoder *d, const void *in_box, void *out_box, unsigned *sent, int *err,
                           long long timeout_ns);
/* Enqueue n positions of this rank's pipeline stage in link form (graphs of
 * 8 positions, then single ones). The positions start at the device
 * position (ptc_decoder_reset: 0); the embedding+head rank must also have
 * begun a device-loop decode (ptc_decoder_generate_begin) and sent the first
 * position's embedding row (ptc_hop_send); every rank enqueues the same n. */
void ptc_decoder_enqueue_stage(ptc_decoder *d, int n);
/* The number of positions of the device-loop decode just begun (default:
 * seq_len): an embedding+head stage's classifier sends no input past it. */
void ptc_decoder_set_stop(ptc_decoder *d, int n_pos);

/* Vocab-parallel classifier (no reference counterpart: the reference's head
 * rank computes all vocab rows, pitorch/model/llama2.c:194-198, inside its
 * ring, pitorch/dist/pt_dist_pipeline.c:290-333). Every rank of a pipeline
 * computes the logits of its own rows of the classifier on the final
 * residual and sends its argmax key to the combining ranks -- rank 0, which
 * then reads the next token's embedding row itself, and the head rank, which
 * keeps the token stream -- and these take the max over all ranks' keys.
 * Needs pipeline links (ptc_decoder_set_links). `box` is this rank's
 * classifier mailbox, ptc_mailbox_alloc(c, dim + 4 * ranks): the final
 * residual x[dim], then one 16-byte key slot per rank. NULL turns the split
 * off. Synchronises the decoder's stream and re-captures its graphs. */
#define PTC_VP_MAX_RANKS 8
typedef struct {
    int row0, rows;          /* this rank's classifier rows [row0, row0 + rows) */
    int ranks, rank;         /* ranks sharing the classifier; this rank's key slot */
    int combine;             /* 1: collect every rank's key and select the token */
    int x_local;             /* 1: this rank ran the last layer (its rows read its own residual) */
    int embed_local;         /* 1: layer 0 reads the token's embedding row (no input message) */
    const float *cls_rows;   /* device rows [row0, row0 + rows), dim floats each */
    const float *rms_final;  /* device final rmsnorm gain [dim] */
    const float *embedding;  /* device [vocab][dim] token embedding (embed_local), else NULL */
    const void *box;         /* this rank's classifier mailbox */
    void *x_out[PTC_VP_MAX_RANKS];  /* x_local: the other ranks' classifier mailboxes (mapped) */
    int n_x_out;
    void *key_out[2];        /* the combining ranks' classifier mailboxes other than this rank's */
    int n_key_out;
    unsigned *sent;          /* device counters: [0] residuals sent, [1] keys sent; zero at the start */
} ptc_vocab_split;
void ptc_decoder_set_vocab_parallel(ptc_decoder *d, const ptc_vocab_split *vp);
/* Host-driven step input of a pipeline rank: mode 0, position pos (through
 * the decoder's pinned block: its previous host-step work must have
 * completed), and the input token copied from device memory (tok_dev; NULL
 * keeps the token). */
void ptc_decoder_set_input(ptc_decoder *d, int pos, const int *tok_dev);

/* Weights were updated in place (training): refresh derived device copies. */
void ptc_decoder_weights_updated(ptc_decoder *d);
/* Phase timeline of the decode kernels (profiling; no reference
 * counterpart -- the reference's trace.c records host spans only). on != 0
 * clears the record and makes the attention block, the FFN block and the
 * classifier stamp %globaltimer (ns) at fixed points of their work; 0 stops
 * it. For position p (recorded modulo 16), kernel k (2l: attention block of
 * layer l, 2l+1: FFN block of layer l, 2L: classifier) and event e < 12,
 * entries 2i and 2i+1 with i = ((p % 16) * (2L + 1) + k) * 12 + e hold the
 * earliest and the latest stamp over the kernel's CTAs (an event a kernel
 * does not have keeps ~0 / 0). Tracing is a parameter of the kernels, so
 * turning it on or off synchronises the decoder's stream and re-captures
 * its graphs (call it between decodes). Returns the number of entries;
 * ptc_decoder_read_trace copies up to n of them and returns how many. */
size_t ptc_decoder_trace(ptc_decoder *d, int on);
size_t ptc_decoder_read_trace(ptc_decoder *d, unsigned long long *out, size_t n);

/* ---- GEMM: replaces sgemm_rect_tmu (pitorch/ops/gemm/gemm_rect.h:13-27,
 *      gemm_rect.c:28-104), C[M][N] (+)= A[M][K] * B[K][N] -------------------- */

/* fp32 GEMM on DEVICE pointers, asynchronous on `stream` (NULL = legacy
 * default stream). Operand layouts cover the three products of a linear
 * layer's training step:
 *   a_kcontig != 0: A(m,k) = A[m*lda + k]   else A(m,k) = A[k*lda + m]
 *   b_kcontig != 0: B(k,n) = B[n*ldb + k]   else B(k,n) = B[k*ldb + n]
 * accumulate != 0 adds into C (the reference's accumulate=1), else C is
 * overwritten. `workspace` (may be NULL) of workspace_floats floats lets
 * long-K products split K across CTAs into partial sums reduced in a fixed
 * order; with NULL the product runs unsplit. */
void ptc_sgemm(int M, int N, int K, const float *A, int lda, int a_kcontig,
               const float *B, int ldb, int b_kcontig, float *C, int ldc, int accumulate,
               float *workspace, size_t workspace_floats, void *stream);

/* Launch counters of the GEMM paths since the library was loaded (no
 * reference counterpart; the Pi build has one QPU path). out[0] tensor-core
 * (tcgen05) kernels, out[1] SIMT tile kernels, out[2] split-K reduction
 * kernels, out[3] SIMT launches whose K-splits were summed inside a
 * thread-block cluster. Counts are per process and cover every device. */
void ptc_gemm_counters(long long out[4]);

/* ptc_sgemm for callers that cannot allocate device memory -- no
 * counterpart in the reference. Code that runs while a stream is being
 * captured into a CUDA graph, inside an allocator callback, or under a host
 * framework that owns all device allocations cannot call cudaMalloc and may
 * have no workspace to pass. This variant takes only the caller's inputs and
 * output; its split-K partial sums live in one static device array of
 * PTC_SGEMM_NOALLOC_MAX_MN floats (4 MiB) that every GPU loading the library
 * keeps until exit. Same product and layouts as ptc_sgemm.
 *  - Returns 0 on success, -1 (with a message on stderr) when M*N exceeds
 *    PTC_SGEMM_NOALLOC_MAX_MN or the device set-up fails. A kernel launch
 *    that the CUDA runtime rejects (an invalid launch, or one made inside a
 *    capture that does not allow it) aborts the process, as every CUDA
 *    failure of this library does; it does not return -1.
 *  - The first call on a device looks up the array's device address
 *    (cudaGetSymbolAddress) for that device; make that first call before
 *    any stream capture.
 *  - Calls never allocate (no cudaMalloc/cudaFree), but they all share the
 *    one array: calls that overlap on the GPU (different streams, or other
 *    threads) race on it and must be serialised by the caller.
 *  - The array keeps the last call's partials; each call overwrites every
 *    partial it reads, so nothing needs clearing between calls. */
#define PTC_SGEMM_NOALLOC_MAX_MN (1u << 20)
int ptc_sgemm_noalloc(int M, int N, int K, const float *A, int lda, int a_kcontig,
                      const float *B, int ldb, int b_kcontig, float *C, int ldc, int accumulate,
                      void *stream);

/* ---- training: replaces pt_forward_train / pt_backward / pt_sgd_update
 *      and their staged variants (pitorch/train/pt_train.c:171-1383) -------- */

typedef struct ptc_trainer ptc_trainer;

/* Device activations, backward buffers and gradients for sequences of up to
 * max_T tokens over the `cfg.n_layers` (local) layers of `w`; the embedding
 * and/or head parts exist when has_embed / has_head. The weights in `w` are
 * updated in place by the SGD calls. Gradients use the reference layout
 * (pitorch/train/pt_train.c:334-371) for the owned parts. */
ptc_trainer *ptc_trainer_create(ptc_ctx *c, const ptc_config *cfg, const ptc_weights *w,
                                int max_T, int has_embed, int has_head);
void ptc_trainer_destroy(ptc_trainer *t);

/* zero_grads -> forward -> backward -> SGD; returns the loss (pt.c:339-364). */
float ptc_trainer_step(ptc_trainer *t, const int *tokens, int T, float lr);

/* Staged pieces (enqueue only, except fwd_head which returns the loss). */
void ptc_trainer_set_tokens(ptc_trainer *t, const int *tokens, int T);
/* The sequence length of the next staged calls without new tokens (a layer
 * range that receives its input rows from another stage). */
void ptc_trainer_set_T(ptc_trainer *t, int T);
void ptc_trainer_zero_grads(ptc_trainer *t);
void ptc_trainer_fwd_embed(ptc_trainer *t);
void ptc_trainer_fwd_layers(ptc_trainer *t, int l_start, int l_end);
float ptc_trainer_fwd_head(ptc_trainer *t);
void ptc_trainer_bwd_head(ptc_trainer *t);
void ptc_trainer_bwd_layers(ptc_trainer *t, int l_start, int l_end);
void ptc_trainer_bwd_embed(ptc_trainer *t);
void ptc_trainer_sgd_layers(ptc_trainer *t, float lr, int l_start, int l_end);
void ptc_trainer_sgd_head(ptc_trainer *t, float lr);
void ptc_trainer_sync(ptc_trainer *t);

/* Device buffers: gradients (n_params floats), residual stream entering
 * layer l ([T, dim]), and the residual gradient d_res ([T, dim]). */
size_t ptc_trainer_n_params(ptc_trainer *t);
float *ptc_trainer_grads(ptc_trainer *t);
float *ptc_trainer_residual(ptc_trainer *t, int l);
float *ptc_trainer_dres(ptc_trainer *t);

/* Microbatch activation sets for pipeline schedules (GPipe): n sets in all,
 * each a full forward state for max_T tokens; ptc_trainer_select makes the
 * forward/backward calls use set m (gradients and weights are shared, so
 * backward calls accumulate). ptc_trainer_dres_save is the selected set's
 * [T, dim] buffer for keeping its residual gradient across a schedule. */
void ptc_trainer_set_microbatches(ptc_trainer *t, int n);
void ptc_trainer_select(ptc_trainer *t, int m);
float *ptc_trainer_dres_save(ptc_trainer *t);

/* ---- CUDA event timing on a context's stream ----------------------------- */
typedef struct ptc_timer ptc_timer;
ptc_timer *ptc_timer_create(ptc_ctx *c);
void ptc_timer_start(ptc_timer *t);
void ptc_timer_stop(ptc_timer *t);
float ptc_timer_ms(ptc_timer *t);     /* synchronises on the stop event */
void ptc_timer_destroy(ptc_timer *t);

/* ---- Pipeline hop over NVLink peer memory ----------------------------------
 * The decode hop of pitorch/dist/pt_dist_pipeline.c:287-333 ([pos | x] from
 * one stage to the next, there over GPIO). Each rank allocates a mailbox in
 * its own memory and exports it (CUDA IPC handle of
 * PTC_MAILBOX_HANDLE_BYTES) to the rank that sends to it. ptc_hop_send
 * writes pos and x into the successor's mailbox with peer stores and then
 * publishes ++*sent; ptc_hop_recv waits (at most timeout_ns on the GPU; on
 * expiry *err = 1 and nothing is copied) until its mailbox holds message
 * ++*recvd, then copies x (and pos, when pos is not NULL) out. The counters
 * are device ints of the caller, zero at the start. */
#define PTC_MAILBOX_HANDLE_BYTES 64
void *ptc_mailbox_alloc(ptc_ctx *c, int dim);
void ptc_mailbox_free(void *box);
int ptc_mailbox_handle(void *box, void *handle_out);
void *ptc_mailbox_open(ptc_ctx *c, const void *handle);  /* NULL when the peer cannot be mapped */
void ptc_mailbox_close(void *peer);
void ptc_hop_send(ptc_ctx *c, const float *x, const int *pos, void *peer_box, unsigned *sent, int dim);
/* The kernel after a ptc_hop_recv may start while the receive still waits
 * (it streams its weights meanwhile and reads x only after the receive
 * completed). */
void ptc_hop_recv(ptc_ctx *c, const void *box, float *x, int *pos, unsigned *recvd, int dim, int *err,
                  long long timeout_ns);

/* ---- CUDA graphs of work enqueued on a context's stream ------------------
 * No reference counterpart (the Pi runtime has no command graphs). Between
 * ptc_capture_begin and ptc_capture_end, calls that enqueue on the context's
 * stream (ptc_matvec with ptc_stream(c), the decoder's enqueue calls) are
 * recorded instead of run; ptc_graph_launch replays them with one launch. */
typedef struct ptc_graph ptc_graph;
void ptc_capture_begin(ptc_ctx *c);
ptc_graph *ptc_capture_end(ptc_ctx *c);
void ptc_graph_launch(ptc_graph *g);
void ptc_graph_destroy(ptc_graph *g);

#ifdef __cplusplus
}
#endif
#endif
