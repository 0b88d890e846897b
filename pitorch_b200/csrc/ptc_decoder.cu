// ptc_decoder.cu -- decode state and the captured CUDA graphs of one
// position (host side of the decode kernels).
//
// Graphs captured per decoder, all built from the same PDL-chained kernels
// (ptc_decode_kernels.cu):
//   host graph:     [copy {pos, token} from pinned memory] -> kernels; the
//                   classifier's last CTA stores the argmax into pinned
//                   memory itself (pt_forward_step path)
//   device graphs:  kernels only, for one position and for DEV_TOKENS
//                   positions; position and token advance on the device, so
//                   a whole greedy decode is a chain of graph launches.
#include <stddef.h>
#include <stdio.h>
#include <string.h>
#include <time.h>

#include "../../include/ptc.h"
#include "ptc_common.cuh"
#include "ptc_decode.cuh"
#include "ptc_internal.h"

using ptc::DecodeModel;
using ptc::StepState;

struct HostIO {
    int pos;
    int tok;
    int next;
    int err;   // the decode kernels' error word, fetched with next
};

struct ptc_decoder {
    ptc_ctx *ctx;
    cudaStream_t stream;
    DecodeModel m;
    int has_embed, has_head, n_sm;
    HostIO *io;            // pinned
    float *stage;          // pinned staging for logits / x
    int *d_tokens;         // [seq + 1]
    int mode;              // current StepState.mode on the device
    cudaGraphExec_t g_host, g_dev;
    cudaGraphExec_t g_devk;  // DEV_TOKENS device-loop tokens per launch (null: not used)
    int fetch_logits;      // ptc_decoder_enqueue_fetch copied the logits into stage
    int w2t_stale;         // the weights changed since w2t was derived (re-derived before the next decode)
    unsigned long long *trace_buf;  // phase timeline record (m.trace while tracing)
    size_t trace_n;        // its entries
    // pipeline stage graphs (ptc_decoder_set_links): STAGE_POS positions and one
    cudaGraphExec_t g_stage, g_stage1;
};

// Positions per captured pipeline stage graph.
constexpr int STAGE_POS = 8;

// The kernels of `n` positions of this rank's pipeline stage, in link form:
// a layer rank's layers (the first attention block waits for its mailbox)
// and the send of its output; the embedding+head rank's classifier (waits for
// its mailbox, sends the next embedding row). The k-th position decodes
// step->pos + k and expects message step->recvd + k + 1; only the last one
// moves both on. With the vocab-parallel classifier every rank also runs its
// classifier rows after its layers (rank 0's first layer reads the token's
// embedding row instead of a message, the last layer rank sends its output
// to every rank's classifier mailbox), and the classifiers move the
// positions and counts on.
static void enqueue_stage_kernels(ptc_decoder *d, int n, cudaStream_t s) {
    for (int k = 0; k < n; k++) {
        DecodeModel mk = d->m;
        mk.link_mode = 1;
        mk.tok_off = k;
        mk.adv = k == n - 1;
        if (mk.L > 0) {
            ptc::launch_layers(mk, 0, mk.L, mk.vp_rows > 0 && !mk.link_recv, d->n_sm, s);
            ptc::launch_stage_send(mk, s);
            if (mk.vp_rows > 0) ptc::launch_head(mk, d->n_sm, s);
        } else {
            ptc::launch_head(mk, d->n_sm, s);
        }
    }
}

static cudaGraphExec_t capture_stage(ptc_decoder *d, int n) {
    cudaGraph_t g;
    PTC_CHECK(cudaStreamBeginCapture(d->stream, cudaStreamCaptureModeThreadLocal));
    enqueue_stage_kernels(d, n, d->stream);
    PTC_CHECK(cudaStreamEndCapture(d->stream, &g));
    cudaGraphExec_t ge;
    PTC_CHECK(cudaGraphInstantiate(&ge, g, 0));
    PTC_CHECK(cudaGraphDestroy(g));
    return ge;
}

static void enqueue_kernels(ptc_decoder *d, const DecodeModel &m, cudaStream_t s, int *host_next) {
    if (d->has_embed && m.L == 0) ptc::launch_embed(m, s);
    ptc::launch_layers(m, 0, m.L, d->has_embed != 0, d->n_sm, s);
    if (d->has_head) ptc::launch_head(m, d->n_sm, s, host_next);
}

// Device-loop tokens per graph launch. Inside one graph the programmatic
// launch chain runs on from one token's classifier into the next token's
// first layer, whose weight copies then overlap the classifier instead of
// starting after a graph boundary.
constexpr int DEV_TOKENS = 8;

static cudaGraphExec_t capture(ptc_decoder *d, bool host_io) {
    cudaStream_t s = d->stream;
    cudaGraph_t g;
    PTC_CHECK(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
    if (host_io)
        PTC_CHECK(cudaMemcpyAsync(d->m.step, d->io, 2 * sizeof(int), cudaMemcpyHostToDevice, s));
    // host steps: the classifier's last CTA stores the token into the pinned
    // io->next itself (4 bytes over PCIe), so the graph ends with the kernel
    enqueue_kernels(d, d->m, s, host_io ? &d->io->next : nullptr);
    PTC_CHECK(cudaStreamEndCapture(s, &g));
    cudaGraphExec_t ge;
    PTC_CHECK(cudaGraphInstantiate(&ge, g, 0));
    PTC_CHECK(cudaGraphDestroy(g));
    return ge;
}

// (Re)capture the host-step graph, the one-position device-loop graph and the
// DEV_TOKENS-position one from the current d->m.
static void capture_graphs(ptc_decoder *d) {
    if (d->g_host) PTC_CHECK(cudaGraphExecDestroy(d->g_host));
    if (d->g_dev) PTC_CHECK(cudaGraphExecDestroy(d->g_dev));
    if (d->g_devk) PTC_CHECK(cudaGraphExecDestroy(d->g_devk));
    if (d->g_stage) PTC_CHECK(cudaGraphExecDestroy(d->g_stage));
    if (d->g_stage1) PTC_CHECK(cudaGraphExecDestroy(d->g_stage1));
    d->g_stage = d->g_stage1 = nullptr;
    if (d->m.in_box) {   // a pipeline stage: its link-form graphs
        d->g_stage = capture_stage(d, STAGE_POS);
        d->g_stage1 = capture_stage(d, 1);
    }
    d->g_host = capture(d, true);
    d->g_dev = capture(d, false);
    d->g_devk = nullptr;
    const DecodeModel &m = d->m;
    if (d->has_embed && d->has_head && m.L > 0) {
        cudaStream_t s = d->stream;
        cudaGraph_t g;
        PTC_CHECK(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
        for (int k = 0; k < DEV_TOKENS; k++) {
            DecodeModel mk = m;
            mk.tok_off = k;
            mk.adv = k == DEV_TOKENS - 1;
            enqueue_kernels(d, mk, s, nullptr);
        }
        PTC_CHECK(cudaStreamEndCapture(s, &g));
        PTC_CHECK(cudaGraphInstantiate(&d->g_devk, g, 0));
        PTC_CHECK(cudaGraphDestroy(g));
    }
}

// A decode kernel whose bounded wait expired left a code in m.err; report it
// at the next synchronisation point (the reference's panic analogue).
static void report_err(const ptc_decoder *d, int e) {
    if (e == ptc::ERR_POS_RANGE)
        PTC_FATAL("decode kernel reported error %d: a position at or past seq_len %d was decoded", e, d->m.seq);
    if (e) PTC_FATAL("decode kernel reported error %d (bounded wait on a weight stage expired)", e);
}

static void check_err(ptc_decoder *d) {
    int e = 0;
    PTC_CHECK(cudaMemcpy(&e, d->m.err, sizeof(int), cudaMemcpyDeviceToHost));
    report_err(d, e);
}

static void set_mode(ptc_decoder *d, int mode) {
    if (d->mode == mode) return;
    PTC_CHECK(cudaMemcpyAsync(&d->m.step->mode, &mode, sizeof(int), cudaMemcpyHostToDevice, d->stream));
    PTC_CHECK(cudaStreamSynchronize(d->stream));
    d->mode = mode;
}

extern "C" ptc_decoder *ptc_decoder_create(ptc_ctx *c, const ptc_config *cfg, const ptc_weights *w,
                                           int has_embed, int has_head) {
    PTC_CHECK(cudaSetDevice(ptc_device(c)));
    ptc_decoder *d = new ptc_decoder();
    memset(&d->m, 0, sizeof(d->m));
    d->m.adv = 1;   // every single-token launch advances the device position
    d->m.link_recv = 1;   // a linked layer rank takes its input from its mailbox
    d->ctx = c;
    d->stream = ptc_ctx_stream(c);
    d->has_embed = has_embed;
    d->has_head = has_head;
    d->n_sm = ptc_sm_count(c);
    DecodeModel &m = d->m;
    m.dim = cfg->dim;
    m.hidden = cfg->hidden_dim;
    m.L = cfg->n_layers;
    m.nh = cfg->n_heads;
    m.nkv = cfg->n_kv_heads;
    m.V = cfg->vocab_size;
    m.seq = cfg->seq_len;
    m.hd = m.dim / m.nh;
    m.kvd = m.nkv * m.hd;
    if (m.dim % 4 || m.hidden % 4 || m.hd % 2)
        PTC_FATAL("decode needs dim, hidden_dim multiples of 4 and an even head_dim (got %d, %d, %d)",
                  m.dim, m.hidden, m.hd);
    if (m.dim > 2048 || m.hidden > 2048) PTC_FATAL("decode supports dim, hidden_dim <= 2048");
    if (m.nh % m.nkv) PTC_FATAL("n_heads must be a multiple of n_kv_heads");
    m.emb = w->token_embedding;
    m.rms_att = w->rms_att_weight;
    m.wq = w->wq;
    m.wk = w->wk;
    m.wv = w->wv;
    m.wo = w->wo;
    m.rms_ffn = w->rms_ffn_weight;
    m.w1 = w->w1;
    m.w2 = w->w2;
    m.w3 = w->w3;
    m.rms_final = w->rms_final_weight;
    m.wcls = w->wcls;
    if (has_embed && !m.emb) PTC_FATAL("decoder with embedding but no token_embedding");
    if (has_head && (!m.wcls || !m.rms_final)) PTC_FATAL("decoder with head but no classifier");

    m.x = (float *)ptc_alloc(c, m.dim * 4);
    m.xn = (float *)ptc_alloc(c, m.dim * 4);
    m.q = (float *)ptc_alloc(c, m.dim * 4);
    m.att = (float *)ptc_alloc(c, m.dim * 4);
    m.hb = (float *)ptc_alloc(c, (size_t)m.hidden * 4);
    m.logits = (float *)ptc_alloc(c, (size_t)m.V * 4);
    size_t kv = (size_t)m.L * m.seq * m.kvd * 4;
    m.kc = (float *)ptc_alloc(c, kv ? kv : 4);
    m.vc = (float *)ptc_alloc(c, kv ? kv : 4);
    m.att_chunk = 64;
    m.n_chunks = (m.seq + m.att_chunk - 1) / m.att_chunk;
    if (!ptc::decode_attn_limits_ok(m.hd, m.att_chunk, m.n_chunks))
        PTC_FATAL("attention limits: head_dim %d (multiple of 4, <= 64), seq_len %d (<= 64 chunks of 64)", m.hd, m.seq);
    m.att_part = (float *)ptc_alloc(c, (size_t)m.nh * m.n_chunks * (m.hd + 2) * 4);
    m.att_ticket = (unsigned *)ptc_alloc(c, (size_t)m.nh * 4);
    m.step = (StepState *)ptc_alloc(c, sizeof(StepState));
    m.err = (int *)ptc_alloc(c, sizeof(int));
    d->d_tokens = (int *)ptc_alloc(c, (size_t)(m.seq + 1) * 4);

    cudaStream_t s = d->stream;
    // Fused FFN (default where it fits; PTC_DECODE_FUSED=0 selects the
    // five-kernel layer): needs the transposed w2 and the hand-over buffers.
    // PTC_DECODE_FUSED=0: five kernels per layer; =ffn: fused FFN only;
    // default: fused attention block + fused FFN (two kernels per layer).
    const char *want_fused = getenv("PTC_DECODE_FUSED");
    const bool no_fuse = want_fused && want_fused[0] == '0';
    const bool ffn_only = want_fused && strcmp(want_fused, "ffn") == 0;
    m.ffn_rows = ptc::decode_ffn_rows(m.dim, m.hidden, d->n_sm);
    m.fused_ffn = m.L > 0 && m.ffn_rows > 0 && !no_fuse;
    m.attn_stage = ptc::decode_attn_stage(m.dim, m.nh, m.nkv, m.seq);
    m.fused_attn = m.fused_ffn && m.attn_stage > 0 && !ffn_only;
    m.tickets = (unsigned *)ptc_alloc(c, 64);
    PTC_CHECK(cudaMemsetAsync(m.tickets, 0, 64, s));
    if (m.fused_attn) {
        float2 *rope = (float2 *)ptc_alloc(c, (size_t)m.seq * (m.hd / 2) * sizeof(float2));
        ptc::build_rope_table(rope, m.seq, m.hd, s);
        m.rope = rope;
    }
    if (m.fused_ffn) {
        float *w2t = (float *)ptc_alloc(c, (size_t)m.L * m.hidden * m.dim * 4);
        ptc::transpose_w2(m, w2t, s);
        m.w2t = w2t;
    }
    d->trace_n = (size_t)2 * ptc::TRACE_POS * (2 * m.L + 1) * ptc::TRACE_EV;
    d->trace_buf = (unsigned long long *)ptc_alloc(c, d->trace_n * sizeof(unsigned long long));
    m.trace = nullptr;
    if (m.fused_ffn) {
        m.xm = (float *)ptc_alloc(c, (size_t)m.dim * 4);
        m.xo = (float *)ptc_alloc(c, (size_t)m.L * m.dim * 4);
        PTC_CHECK(cudaMemsetAsync(m.xm, 0, (size_t)m.dim * 4, s));
        PTC_CHECK(cudaMemsetAsync(m.xo, 0, (size_t)m.L * m.dim * 4, s));
    }
    PTC_CHECK(cudaMemsetAsync(m.x, 0, m.dim * 4, s));
    PTC_CHECK(cudaMemsetAsync(m.kc, 0, kv ? kv : 4, s));
    PTC_CHECK(cudaMemsetAsync(m.vc, 0, kv ? kv : 4, s));
    PTC_CHECK(cudaMemsetAsync(m.att_ticket, 0, (size_t)m.nh * 4, s));
    PTC_CHECK(cudaMemsetAsync(m.err, 0, sizeof(int), s));
    StepState st;
    memset(&st, 0, sizeof(st));
    st.tokens = d->d_tokens;
    PTC_CHECK(cudaMemcpyAsync(m.step, &st, sizeof(st), cudaMemcpyHostToDevice, s));
    PTC_CHECK(cudaStreamSynchronize(s));
    d->mode = 0;

    d->io = (HostIO *)ptc_host_alloc(sizeof(HostIO));
    memset(d->io, 0, sizeof(HostIO));
    size_t stage = (size_t)(m.V > m.dim ? m.V : m.dim) * 4;
    d->stage = (float *)ptc_host_alloc(stage);

    d->g_host = d->g_dev = d->g_devk = nullptr;
    d->g_stage = d->g_stage1 = nullptr;
    capture_graphs(d);

    return d;
}

// Re-derive device-side copies that depend on the weights (the transposed
// w2 of the fused FFN) after an in-place update.
// Training steps mark the transposed w2 stale; the decode entry points below
// re-derive it (on the decoder's stream, after the update) before they
// enqueue layer kernels, so a run of training steps pays for it once.
extern "C" void ptc_decoder_weights_updated(ptc_decoder *d) {
    if (d->m.w2t) d->w2t_stale = 1;
}

static void refresh_derived(ptc_decoder *d) {
    if (!d->w2t_stale) return;
    ptc::transpose_w2(d->m, (float *)d->m.w2t, d->stream);
    d->w2t_stale = 0;
}

// Tracing is a kernel parameter (m.trace non-null), so the untraced kernels
// pay nothing for it: turning it on or off re-captures the graphs.
extern "C" size_t ptc_decoder_trace(ptc_decoder *d, int on) {
    PTC_CHECK(cudaStreamSynchronize(d->stream));
    if (on) {   // earliest stamps start high, latest stamps low
        unsigned long long *h = (unsigned long long *)malloc(d->trace_n * sizeof(unsigned long long));
        for (size_t i = 0; i < d->trace_n; i++) h[i] = (i & 1) ? 0ull : ~0ull;
        PTC_CHECK(cudaMemcpy(d->trace_buf, h, d->trace_n * sizeof(unsigned long long), cudaMemcpyHostToDevice));
        free(h);
    }
    unsigned long long *want = on ? d->trace_buf : nullptr;
    if (d->m.trace != want) {
        d->m.trace = want;
        capture_graphs(d);
    }
    return d->trace_n;
}

extern "C" size_t ptc_decoder_read_trace(ptc_decoder *d, unsigned long long *out, size_t n) {
    if (n > d->trace_n) n = d->trace_n;
    PTC_CHECK(cudaMemcpyAsync(out, d->trace_buf, n * sizeof(unsigned long long), cudaMemcpyDeviceToHost, d->stream));
    PTC_CHECK(cudaStreamSynchronize(d->stream));
    return n;
}

extern "C" void ptc_decoder_destroy(ptc_decoder *d) {
    if (!d) return;
    cudaStreamSynchronize(d->stream);
    cudaGraphExecDestroy(d->g_host);
    cudaGraphExecDestroy(d->g_dev);
    if (d->g_devk) cudaGraphExecDestroy(d->g_devk);
    if (d->g_stage) cudaGraphExecDestroy(d->g_stage);
    if (d->g_stage1) cudaGraphExecDestroy(d->g_stage1);
    ptc_host_free(d->io);
    ptc_host_free(d->stage);
    delete d;  // device buffers belong to the context arena
}

extern "C" void ptc_decoder_reset(ptc_decoder *d) {
    // position 0 (a pipeline layer rank keeps its position on the device)
    PTC_CHECK(cudaMemsetAsync(&d->m.step->pos, 0, sizeof(int), d->stream));
    size_t kv = (size_t)d->m.L * d->m.seq * d->m.kvd * 4;
    if (kv) {
        PTC_CHECK(cudaMemsetAsync(d->m.kc, 0, kv, d->stream));
        PTC_CHECK(cudaMemsetAsync(d->m.vc, 0, kv, d->stream));
    }
    // the fused layers' accumulation buffers start from zero (a completed
    // step leaves them so; a timing hook may not)
    if (d->m.fused_ffn) {
        PTC_CHECK(cudaMemsetAsync(d->m.xm, 0, (size_t)d->m.dim * 4, d->stream));
        PTC_CHECK(cudaMemsetAsync(d->m.xo, 0, (size_t)d->m.L * d->m.dim * 4, d->stream));
        PTC_CHECK(cudaMemsetAsync(d->m.tickets, 0, 64, d->stream));
    }
    PTC_CHECK(cudaStreamSynchronize(d->stream));
}

// io->next before the classifier of a host step has stored its token
constexpr int NEXT_PENDING = -2;

// Wait for the classifier's store into the pinned io->next (it fences after
// the store): the token is back before the graph's completion would reach
// the host through the stream. Bounded: after 2 s of spinning the stream is
// synchronised instead, which reports a failed launch. Work later enqueued
// on the stream stays ordered after the still-finishing graph.
static void wait_next(ptc_decoder *d) {
    volatile int *w = &d->io->next;
    struct timespec t0, t;
    clock_gettime(CLOCK_MONOTONIC, &t0);
    for (unsigned it = 1;; it++) {
        if (*w != NEXT_PENDING) return;
        if ((it & 1023) == 0) {
            clock_gettime(CLOCK_MONOTONIC, &t);
            if ((t.tv_sec - t0.tv_sec) * 1000000000L + (t.tv_nsec - t0.tv_nsec) > 2000000000L) break;
        }
    }
    PTC_CHECK(cudaStreamSynchronize(d->stream));
}

extern "C" int ptc_decoder_step(ptc_decoder *d, int token, int pos, float *logits_host) {
    if (pos < 0 || pos >= d->m.seq) PTC_FATAL("decode position %d outside [0, %d)", pos, d->m.seq);
    refresh_derived(d);
    if (d->has_embed && (token < 0 || token >= d->m.V))
        PTC_FATAL("token %d outside [0, %d)", token, d->m.V);
    set_mode(d, 0);
    d->io->pos = pos;
    d->io->tok = token;
    d->io->next = d->has_head ? NEXT_PENDING : -1;   // overwritten by the classifier
    PTC_CHECK(cudaGraphLaunch(d->g_host, d->stream));
    if (logits_host && d->has_head) {
        PTC_CHECK(cudaMemcpyAsync(d->stage, d->m.logits, (size_t)d->m.V * 4, cudaMemcpyDeviceToHost,
                                  d->stream));
        PTC_CHECK(cudaStreamSynchronize(d->stream));
        memcpy(logits_host, d->stage, (size_t)d->m.V * 4);
    } else if (d->has_head) {
        wait_next(d);
    } else {
        PTC_CHECK(cudaStreamSynchronize(d->stream));
    }
    const int next = d->io->next;
    if (next < 0 || next >= d->m.V) {
        PTC_CHECK(cudaStreamSynchronize(d->stream));
        check_err(d);
    }
    return d->has_head ? next : -1;
}

extern "C" void ptc_decoder_set_x(ptc_decoder *d, const float *x_host) {
    set_mode(d, 0);
    memcpy(d->stage, x_host, (size_t)d->m.dim * 4);
    PTC_CHECK(cudaMemcpyAsync(d->m.x, d->stage, (size_t)d->m.dim * 4, cudaMemcpyHostToDevice, d->stream));
    PTC_CHECK(cudaStreamSynchronize(d->stream));
}

static void get_vec(ptc_decoder *d, const float *src, float *x_host) {
    PTC_CHECK(cudaMemcpyAsync(d->stage, src, (size_t)d->m.dim * 4, cudaMemcpyDeviceToHost, d->stream));
    PTC_CHECK(cudaStreamSynchronize(d->stream));
    memcpy(x_host, d->stage, (size_t)d->m.dim * 4);
}

extern "C" void ptc_decoder_get_x(ptc_decoder *d, float *x_host) { get_vec(d, d->m.x, x_host); }
extern "C" void ptc_decoder_get_xnorm(ptc_decoder *d, float *x_host) { get_vec(d, d->m.xn, x_host); }
extern "C" float *ptc_decoder_x_dev(ptc_decoder *d) { return d->m.x; }
extern "C" float *ptc_decoder_logits_dev(ptc_decoder *d) { return d->m.logits; }

extern "C" void ptc_decoder_generate_begin(ptc_decoder *d, const int *prompt, int n_prompt) {
    // (a combining rank of a vocab-parallel classifier selects tokens too)
    if ((!d->has_embed || !d->has_head) && !(d->m.vp_rows > 0 && d->m.vp_combine))
        PTC_FATAL("device-loop decode needs embedding and head");
    if (n_prompt < 1 || n_prompt > d->m.seq) PTC_FATAL("prompt length %d outside [1, %d]", n_prompt, d->m.seq);
    for (int i = 0; i < n_prompt; i++)
        if (prompt[i] < 0 || prompt[i] >= d->m.V) PTC_FATAL("prompt token %d outside [0, %d)", prompt[i], d->m.V);
    PTC_CHECK(cudaMemcpyAsync(d->d_tokens, prompt, (size_t)n_prompt * 4, cudaMemcpyHostToDevice, d->stream));
    StepState st;
    memset(&st, 0, sizeof(st));
    st.pos = 0;
    st.tok = prompt[0];
    st.n_prompt = n_prompt;
    st.mode = 1;
    st.tokens = d->d_tokens;
    st.stop = d->m.seq;
    // everything before the link's message count, which outlives decodes
    PTC_CHECK(cudaMemcpyAsync(d->m.step, &st, offsetof(StepState, recvd), cudaMemcpyHostToDevice, d->stream));
    PTC_CHECK(cudaStreamSynchronize(d->stream));
    d->mode = 1;
}

extern "C" void ptc_decoder_enqueue_steps(ptc_decoder *d, int n) {
    refresh_derived(d);
    int i = 0;
    if (d->g_devk)
        for (; i + DEV_TOKENS <= n; i += DEV_TOKENS) PTC_CHECK(cudaGraphLaunch(d->g_devk, d->stream));
    for (; i < n; i++) PTC_CHECK(cudaGraphLaunch(d->g_dev, d->stream));
}

extern "C" void ptc_decoder_read_tokens(ptc_decoder *d, int *out_tokens, int n) {
    // tokens[p + 1] is the token emitted at position p.
    PTC_CHECK(cudaMemcpyAsync(out_tokens, d->d_tokens + 1, (size_t)n * 4, cudaMemcpyDeviceToHost, d->stream));
    PTC_CHECK(cudaStreamSynchronize(d->stream));
    check_err(d);
}

extern "C" void ptc_decoder_generate(ptc_decoder *d, const int *prompt, int n_prompt, int n_pos,
                                     int *out_tokens) {
    if (n_pos > d->m.seq) PTC_FATAL("n_pos %d exceeds seq_len %d", n_pos, d->m.seq);
    ptc_decoder_reset(d);
    ptc_decoder_generate_begin(d, prompt, n_prompt);
    ptc_decoder_enqueue_steps(d, n_pos);
    ptc_decoder_read_tokens(d, out_tokens, n_pos);
}

// ---- staged, eager launches --------------------------------------------------

static void put_step_int(ptc_decoder *d, int *field, int v) {
    // Pageable source: the runtime reads it before returning.
    PTC_CHECK(cudaMemcpyAsync(field, &v, sizeof(int), cudaMemcpyHostToDevice, d->stream));
}

extern "C" void ptc_decoder_enqueue_embed(ptc_decoder *d, int token) {
    if (!d->has_embed) PTC_FATAL("decoder has no embedding");
    if (token < 0 || token >= d->m.V) PTC_FATAL("token %d outside [0, %d)", token, d->m.V);
    set_mode(d, 0);
    put_step_int(d, &d->m.step->tok, token);
    ptc::launch_embed(d->m, d->stream);
}

extern "C" void ptc_decoder_enqueue_layers(ptc_decoder *d, int pos, int l_start, int l_end) {
    refresh_derived(d);
    if (pos < 0 || pos >= d->m.seq) PTC_FATAL("decode position %d outside [0, %d)", pos, d->m.seq);
    if (l_start < 0 || l_end > d->m.L || l_start > l_end)
        PTC_FATAL("layer range [%d, %d) outside [0, %d)", l_start, l_end, d->m.L);
    set_mode(d, 0);
    put_step_int(d, &d->m.step->pos, pos);
    ptc::launch_layers(d->m, l_start, l_end, false, d->n_sm, d->stream);
}

// Mode is the caller's: host-mode callers set it through the functions that
// take a host token/position; the pipeline's device loop keeps mode 1.
extern "C" void ptc_decoder_enqueue_head(ptc_decoder *d) {
    if (!d->has_head) PTC_FATAL("decoder has no head");
    ptc::launch_head(d->m, d->n_sm, d->stream);
}

extern "C" int ptc_decoder_fetch_next(ptc_decoder *d, float *logits_host) {
    PTC_CHECK(cudaMemcpyAsync(&d->io->next, &d->m.step->next, sizeof(int), cudaMemcpyDeviceToHost, d->stream));
    if (logits_host)
        PTC_CHECK(cudaMemcpyAsync(d->stage, d->m.logits, (size_t)d->m.V * 4, cudaMemcpyDeviceToHost, d->stream));
    PTC_CHECK(cudaStreamSynchronize(d->stream));
    if (logits_host) memcpy(logits_host, d->stage, (size_t)d->m.V * 4);
    check_err(d);
    return d->io->next;
}

// Host steps of the pipeline's embedding rank: position and token go through
// the pinned io block in one copy (the previous step's copies from it have
// completed: the pipeline step waits for its stream before returning), and
// the argmax, the error word and the logits come back with copies enqueued
// before the caller's single wait for the stream.
extern "C" void ptc_decoder_enqueue_embed_at(ptc_decoder *d, int token, int pos) {
    if (!d->has_embed) PTC_FATAL("decoder has no embedding");
    if (token < 0 || token >= d->m.V) PTC_FATAL("token %d outside [0, %d)", token, d->m.V);
    if (pos < 0 || pos >= d->m.seq) PTC_FATAL("decode position %d outside [0, %d)", pos, d->m.seq);
    set_mode(d, 0);
    d->io->pos = pos;
    d->io->tok = token;
    PTC_CHECK(cudaMemcpyAsync(d->m.step, d->io, 2 * sizeof(int), cudaMemcpyHostToDevice, d->stream));
    ptc::launch_embed(d->m, d->stream);
}

extern "C" void ptc_decoder_enqueue_fetch(ptc_decoder *d, int logits) {
    PTC_CHECK(cudaMemcpyAsync(&d->io->next, &d->m.step->next, sizeof(int), cudaMemcpyDeviceToHost, d->stream));
    PTC_CHECK(cudaMemcpyAsync(&d->io->err, d->m.err, sizeof(int), cudaMemcpyDeviceToHost, d->stream));
    d->fetch_logits = logits && d->has_head;
    if (d->fetch_logits)
        PTC_CHECK(cudaMemcpyAsync(d->stage, d->m.logits, (size_t)d->m.V * 4, cudaMemcpyDeviceToHost, d->stream));
}

extern "C" int ptc_decoder_take_next(ptc_decoder *d, float *logits_host) {
    report_err(d, d->io->err);
    if (logits_host && d->fetch_logits) memcpy(logits_host, d->stage, (size_t)d->m.V * 4);
    return d->io->next;
}

extern "C" int *ptc_decoder_pos_dev(ptc_decoder *d) { return &d->m.step->pos; }
extern "C" int *ptc_decoder_tok_dev(ptc_decoder *d) { return &d->m.step->tok; }

extern "C" void ptc_decoder_enqueue_layers_devpos(ptc_decoder *d, int l_start, int l_end) {
    refresh_derived(d);
    if (l_start < 0 || l_end > d->m.L || l_start > l_end)
        PTC_FATAL("layer range [%d, %d) outside [0, %d)", l_start, l_end, d->m.L);
    ptc::launch_layers(d->m, l_start, l_end, false, d->n_sm, d->stream);
}

extern "C" void ptc_decoder_enqueue_kernel(ptc_decoder *d, int kind, int l, int pos) {
    refresh_derived(d);
    if (pos < 0 || pos >= d->m.seq) PTC_FATAL("decode position %d outside [0, %d)", pos, d->m.seq);
    set_mode(d, 0);
    put_step_int(d, &d->m.step->pos, pos);
    if (kind == 2) {
        if (!d->has_head) PTC_FATAL("decoder has no head");
        ptc::launch_head(d->m, d->n_sm, d->stream);
        return;
    }
    if (l < 0 || l >= d->m.L) PTC_FATAL("layer %d outside [0, %d)", l, d->m.L);
    ptc::launch_block(d->m, kind, l, d->n_sm, d->stream);
}

extern "C" int ptc_decoder_launches_per_step(ptc_decoder *d) {
    const ptc::DecodeModel &m = d->m;
    const int per_layer = m.fused_attn ? 2 : m.fused_ffn ? 4 : 5;
    return per_layer * m.L + (d->has_head || m.vp_rows > 0 ? 1 : 0) + (d->has_embed && m.L == 0 ? 1 : 0);
}

extern "C" void ptc_decoder_enqueue_embed_dev(ptc_decoder *d) {
    if (!d->has_embed) PTC_FATAL("decoder has no embedding");
    ptc::launch_embed(d->m, d->stream);
}

extern "C" void ptc_decoder_set_links(ptc_decoder *d, const void *in_box, void *out_box, unsigned *sent, int *err,
                                      long long timeout_ns) {
    PTC_CHECK(cudaStreamSynchronize(d->stream));
    if (in_box && (!out_box || !sent || !err)) PTC_FATAL("pipeline links need out_box, sent and err");
    if (in_box && d->m.L > 0 && !d->m.fused_attn)
        PTC_FATAL("pipeline links need the fused attention block (two kernels per layer)");
    if (in_box && d->m.L == 0 && !(d->has_embed && d->has_head))
        PTC_FATAL("a pipeline stage without layers must hold the embedding and the classifier");
    d->m.in_box = (const unsigned char *)in_box;
    d->m.out_box = (unsigned char *)out_box;
    d->m.link_sent = sent;
    d->m.link_err = err;
    d->m.link_timeout_ns = (unsigned long long)(timeout_ns > 0 ? timeout_ns : 0);
    capture_graphs(d);
}

extern "C" void ptc_decoder_set_vocab_parallel(ptc_decoder *d, const ptc_vocab_split *vp) {
    PTC_CHECK(cudaStreamSynchronize(d->stream));
    DecodeModel &m = d->m;
    if (!vp) {
        m.vp_rows = 0;
        m.n_cls_out = m.n_key_out = 0;
        m.link_recv = 1;
        capture_graphs(d);
        return;
    }
    if (!m.in_box) PTC_FATAL("the vocab-parallel classifier needs pipeline links (ptc_decoder_set_links)");
    if (vp->ranks < 2 || vp->ranks > PTC_VP_MAX_RANKS || vp->rank < 0 || vp->rank >= vp->ranks)
        PTC_FATAL("vocab-parallel rank %d of %d (2 to %d ranks)", vp->rank, vp->ranks, PTC_VP_MAX_RANKS);
    if (vp->rows < 1 || vp->row0 < 0 || vp->row0 + vp->rows > m.V)
        PTC_FATAL("vocab-parallel rows [%d, %d) outside [0, %d)", vp->row0, vp->row0 + vp->rows, m.V);
    if (!vp->cls_rows || !vp->rms_final || !vp->box || !vp->sent) PTC_FATAL("vocab-parallel split without weights or mailbox");
    if (vp->embed_local && (!vp->embedding || m.L == 0))
        PTC_FATAL("a vocab-parallel rank that embeds needs the table and the first layers");
    if (vp->n_x_out < 0 || vp->n_x_out > PTC_VP_MAX_RANKS || vp->n_key_out < 0 || vp->n_key_out > 2)
        PTC_FATAL("vocab-parallel targets: %d residual, %d key", vp->n_x_out, vp->n_key_out);
    if (vp->x_local != (vp->n_x_out > 0)) PTC_FATAL("the last layer rank (x_local) sends the final residual");
    m.vp_row0 = vp->row0;
    m.vp_rows = vp->rows;
    m.vp_ranks = vp->ranks;
    m.vp_rank = vp->rank;
    m.vp_combine = vp->combine ? 1 : 0;
    m.vp_x_local = vp->x_local ? 1 : 0;
    m.vp_W = vp->cls_rows;
    m.rms_final = vp->rms_final;
    if (vp->embed_local) m.emb = vp->embedding;
    m.link_recv = vp->embed_local ? 0 : 1;
    m.cls_box = (const unsigned char *)vp->box;
    m.n_cls_out = vp->n_x_out;
    for (int j = 0; j < vp->n_x_out; j++) m.cls_out[j] = (unsigned char *)vp->x_out[j];
    m.n_key_out = vp->n_key_out;
    for (int j = 0; j < vp->n_key_out; j++)
        m.key_out[j] = reinterpret_cast<ptc::KeySlot *>((unsigned char *)vp->key_out[j] + sizeof(ptc::MailboxHeader) +
                                                        (size_t)m.dim * 4);
    m.cls_sent = vp->sent;
    m.key_sent = vp->sent + 1;
    capture_graphs(d);
}

extern "C" void ptc_decoder_set_input(ptc_decoder *d, int pos, const int *tok_dev) {
    if (pos < 0 || pos >= d->m.seq) PTC_FATAL("decode position %d outside [0, %d)", pos, d->m.seq);
    set_mode(d, 0);
    // through the pinned io block, like ptc_decoder_enqueue_embed_at
    d->io->pos = pos;
    PTC_CHECK(cudaMemcpyAsync(&d->m.step->pos, &d->io->pos, sizeof(int), cudaMemcpyHostToDevice, d->stream));
    if (tok_dev)
        PTC_CHECK(cudaMemcpyAsync(&d->m.step->tok, tok_dev, sizeof(int), cudaMemcpyDeviceToDevice, d->stream));
}

extern "C" void ptc_decoder_set_stop(ptc_decoder *d, int n_pos) {
    if (n_pos < 1 || n_pos > d->m.seq) PTC_FATAL("decode length %d outside [1, %d]", n_pos, d->m.seq);
    PTC_CHECK(cudaMemcpyAsync(&d->m.step->stop, &n_pos, sizeof(int), cudaMemcpyHostToDevice, d->stream));
    PTC_CHECK(cudaStreamSynchronize(d->stream));
}

extern "C" void ptc_decoder_enqueue_stage(ptc_decoder *d, int n) {
    refresh_derived(d);
    if (!d->m.in_box) PTC_FATAL("ptc_decoder_enqueue_stage without pipeline links");
    int i = 0;
    for (; i + STAGE_POS <= n; i += STAGE_POS) PTC_CHECK(cudaGraphLaunch(d->g_stage, d->stream));
    for (; i < n; i++) PTC_CHECK(cudaGraphLaunch(d->g_stage1, d->stream));
}
