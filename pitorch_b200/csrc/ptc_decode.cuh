// ptc_decode.cuh -- device-side data layout of one decode context.
#pragma once

#include <stdint.h>

#include "../../include/ptc.h"
#include "ptc_common.cuh"

namespace ptc {

// Per-step control block, resident in device memory. The decode kernels read
// the position and input token from here, and the classifier kernel's last
// CTA writes the argmax and (in device-loop mode) advances the position, so
// a whole greedy decode can run without host round trips.
struct StepState {
    int pos;                  // position being decoded
    int tok;                  // input token at pos
    int next;                 // argmax of this step's logits
    int n_prompt;             // device-loop mode: prompt length
    int mode;                 // 0: host drives pos/tok; 1: device loop
    int pad0;
    unsigned done;            // classifier CTAs finished (reset by the last)
    unsigned pad1;
    unsigned long long amax;  // packed (value, index) running argmax
    int *tokens;              // device-loop mode: token stream [seq]
    int stop;                 // device-loop mode: positions of this decode (the last is stop - 1)
    // Pipeline stage: messages taken from this rank's mailbox so far (the
    // sender's count of the same link). Kept across decodes: the fields
    // above it are rewritten when a decode begins, this one never.
    unsigned recvd;
    // Vocab-parallel classifier: final residuals taken from this rank's
    // classifier mailbox, and key rounds collected from the other ranks
    // (kept across decodes like recvd).
    unsigned cls_recvd;
    unsigned key_recvd;
    unsigned pad2;
};

// Everything the decode kernels need for one model replica.
struct DecodeModel {
    int dim, hidden, L, nh, nkv, V, seq, hd, kvd;
    // weights, device pointers into the uploaded .bin image
    const float *emb, *rms_att, *wq, *wk, *wv, *wo, *rms_ffn, *w1, *w2, *w3,
        *rms_final, *wcls;
    // activations
    float *x;        // [dim] residual stream
    float *xn;       // [dim] final-normalised x (pt_forward_head's in-place rmsnorm)
    float *q;        // [dim] post-RoPE query
    float *att;      // [dim] attention output (input of wo)
    float *hb;       // [hidden] silu(w1 x) * (w3 x)
    float *logits;   // [V]
    // Fused-FFN path: xm is the post-attention residual (FFN input), xo the
    // per-layer outputs [L][dim] that the next layer consumes, w2t the
    // transposed w2 [L][hidden][dim]. The FFN kernel accumulates into a
    // zeroed buffer; whoever reads a layer input last zeroes it again.
    float *xm, *xo;
    const float *w2t;
    int fused_ffn;   // 1: k_ffn replaces k_mv<FFN13> + k_mv<RESID>(w2)
    int ffn_rows;    // hidden units per k_ffn CTA (capacity of its shared memory)
    int fused_attn;  // 1: k_attn_fused replaces k_mv<QKV> + k_attn + k_mv<RESID>(wo)
    int attn_stage;  // floats of k_attn_fused's shared staging region
    unsigned *tickets;  // [0] k_attn_fused, [1] k_ffn: CTAs done reading their input
    const float2 *rope;  // [seq][hd/2] (cos, sin) of the RoPE angle (k_attn_fused)
    // KV cache, head-major: [L][nkv][seq][hd]
    float *kc, *vc;
    // attention split-K partials: [nh][n_chunks][hd + 2] and per-head tickets
    float *att_part;
    unsigned *att_ticket;
    int att_chunk;   // positions per attention CTA
    int n_chunks;    // ceil(seq / att_chunk)
    StepState *step;
    int *err;        // set (non-zero) by a kernel whose bounded wait expired
    // Several device-loop tokens captured in one graph: the kernels of the
    // graph's k-th token decode position step->pos + tok_off (step->pos is
    // advanced only by the classifier of the last token, adv = 1), and layer
    // 0 reads step->tok after its wait when tok_off > 0, since it may start
    // while the previous token's classifier still runs.
    int tok_off;
    int adv;
    // Phase timeline (ptc_decoder_trace), stamped only when non-null (the
    // decoder re-captures its graphs to turn it on or off):
    // for traced position p, kernel k of the position (2l: attention block of
    // layer l, 2l+1: its FFN block, 2L: the classifier) and event e, the
    // earliest and the latest %globaltimer over the kernel's CTAs at
    // trace[2 * (((p % TRACE_POS) * (2L + 1) + k) * TRACE_EV + e)] (+1).
    unsigned long long *trace;
    // Pipeline links (ptc_decoder_set_links; null on a single GPU). While
    // link_mode is set (the decoder's stage graphs), the first layer's
    // attention block -- or, on the embedding+head rank, the classifier --
    // takes x from in_box, waiting on the GPU for the message of its
    // position; in device-loop mode the classifier's last CTA sends the next
    // token's embedding row to out_box itself.
    const unsigned char *in_box;   // this rank's mailbox (MailboxHeader, then x)
    unsigned char *out_box;        // the next stage's mailbox (peer memory)
    unsigned *link_sent;           // messages this rank has sent on its out link
    int *link_err;                 // 1: a mailbox wait expired, 2: a message for another position
    unsigned long long link_timeout_ns;
    int link_mode;
    int link_recv;   // link form: the first layer takes x from in_box (else the token's embedding row)
    // Vocab-parallel classifier (ptc_decoder_set_vocab_parallel; vp_rows 0:
    // off). Every rank of the pipeline computes the logits of its rows
    // [vp_row0, vp_row0 + vp_rows) of the classifier on the final residual
    // and sends its argmax key to the combining ranks, which take the max
    // over all ranks' keys as the step's token.
    int vp_row0, vp_rows;
    int vp_ranks, vp_rank;
    int vp_combine;          // this rank collects the keys (rank 0 and the head rank)
    int vp_x_local;          // this rank ran the last layer: its slice reads m.x
    const float *vp_W;       // the classifier rows of this rank (row vp_row0 first)
    const unsigned char *cls_box;    // this rank's classifier mailbox: MailboxHeader, x[dim], KeySlot[vp_ranks]
    unsigned char *cls_out[PTC_VP_MAX_RANKS];  // the last layer rank: mailboxes the final x goes to
    int n_cls_out;
    KeySlot *key_out[2];     // the combining ranks' key slots (slot vp_rank is this rank's)
    int n_key_out;
    unsigned *cls_sent;      // final residuals this rank has sent
    unsigned *key_sent;      // keys this rank has sent (once per position, to every combining rank)
};

constexpr int TRACE_POS = 16;
constexpr int TRACE_EV = 12;

// Decode matvec staging: each CTA streams its contiguous block of weight rows
// through a ring of shared-memory stages filled by bulk (TMA) copies.
constexpr int MV_THREADS = 256;
constexpr int MV_STAGES = 4;
constexpr int MV_STAGE_BYTES = 24 * 1024;
constexpr int MV_BAR_BYTES = 128;   // mbarriers at the front, stages 128-byte aligned after

// Fused FFN (k_ffn): one CTA per SM, whole w1/w3/w2t row blocks resident.
constexpr int FF_THREADS = 256;
constexpr int FF_MAX_SMEM = 200 * 1024;

// Error codes written to DecodeModel::err.
constexpr int ERR_MBAR_TIMEOUT = 1;
constexpr int ERR_POS_RANGE = 2;   // a kernel was asked for a position outside [0, seq_len)

}  // namespace ptc
