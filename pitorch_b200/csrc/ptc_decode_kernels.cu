// ptc_decode_kernels.cu -- the batch-1 decode step as fused sm_100a kernels.
//
// One decode position of pitorch's pt_forward (pitorch/model/llama2.c:224-303)
// becomes, per layer,
//   k_qkv    rmsnorm + [wq;wk;wv] matvec + RoPE + KV-cache write
//   k_attn   causal attention over positions <= pos, split over position
//            chunks, merged by the last CTA of each head
//   k_resid  x += wo . att
//   k_ffn13  rmsnorm + w1/w3 matvecs + silu(w1 x) * (w3 x)
//   k_resid  x += w2 . hb
// and, once, k_cls: final rmsnorm + the vocab-row classifier + argmax.
//
// Every matvec is memory-bound fp32 (0.5 flop/byte): each warp owns whole
// rows, lanes read consecutive 16-byte chunks of a row (128-bit, coalesced,
// L1-bypassing), the input vector sits in registers, and a shuffle tree
// reduces each row. Kernels are launched with programmatic dependent launch:
// a kernel issues its weight loads -- which never depend on the previous
// kernel -- before griddepcontrol.wait, so weight streaming for kernel N+1
// overlaps the tail of kernel N.
#include "ptc_common.cuh"
#include "ptc_decode.cuh"
#include "ptc_internal.h"

#include <cooperative_groups.h>
#include <string.h>

#include <utility>

namespace cg = cooperative_groups;

namespace ptc {

// ---------------------------------------------------------------------------
// Row/vector helpers. A row of `cols` floats is c4 = cols/4 float4s; lane
// `lane` owns float4 indices lane, lane+32, ..., lane+32*(NV-1).
// ---------------------------------------------------------------------------

template <int NV>
__device__ __forceinline__ void load_row(float4 (&w)[NV], const float *row, int c4, int lane) {
    const float4 *r4 = reinterpret_cast<const float4 *>(row);
#pragma unroll
    for (int v = 0; v < NV; v++) {
        int c = lane + 32 * v;
        w[v] = (c < c4) ? ldg_stream(r4 + c) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
}

// Activations written by an earlier kernel: read through L2 only.
template <int NV>
__device__ __forceinline__ void load_act(float4 (&x)[NV], const float *src, int c4, int lane) {
    const float4 *s4 = reinterpret_cast<const float4 *>(src);
#pragma unroll
    for (int v = 0; v < NV; v++) {
        int c = lane + 32 * v;
        x[v] = (c < c4) ? __ldcg(s4 + c) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
}

template <int NV>
__device__ __forceinline__ float row_dot(const float4 (&w)[NV], const float4 (&x)[NV]) {
    float acc = 0.f;
#pragma unroll
    for (int v = 0; v < NV; v++) acc = dot4(w[v], x[v], acc);
    return warp_sum(acc);
}

// In-register rmsnorm (pitorch/ops/core/pt_ops.c:5-12): o = (x * s) * g with
// s = 1 / sqrt(mean(x^2) + 1e-5).
template <int NV>
__device__ __forceinline__ void rmsnorm_regs(float4 (&x)[NV], const float *gain, int dim, int lane) {
    float ss = 0.f;
#pragma unroll
    for (int v = 0; v < NV; v++)
        ss += x[v].x * x[v].x + x[v].y * x[v].y + x[v].z * x[v].z + x[v].w * x[v].w;
    ss = warp_sum(ss);
    float s = rms_scale(ss, dim);
    const float4 *g4 = reinterpret_cast<const float4 *>(gain);
    int c4 = dim >> 2;
#pragma unroll
    for (int v = 0; v < NV; v++) {
        int c = lane + 32 * v;
        if (c < c4) {
            float4 g = __ldg(g4 + c);
            x[v].x = __fmul_rn(__fmul_rn(x[v].x, s), g.x);
            x[v].y = __fmul_rn(__fmul_rn(x[v].y, s), g.y);
            x[v].z = __fmul_rn(__fmul_rn(x[v].z, s), g.z);
            x[v].w = __fmul_rn(__fmul_rn(x[v].w, s), g.w);
        }
    }
}

template <int NV>
__device__ __forceinline__ void load_gain(float4 (&g)[NV], const float *gain, int c4, int lane) {
    const float4 *g4 = reinterpret_cast<const float4 *>(gain);
#pragma unroll
    for (int v = 0; v < NV; v++) {
        const int c = lane + 32 * v;
        g[v] = (c < c4) ? __ldg(g4 + c) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
}

// rmsnorm with the gain already in registers (pitorch/ops/core/pt_ops.c:5-12).
template <int NV>
__device__ __forceinline__ void rmsnorm_pre(float4 (&x)[NV], const float4 (&g)[NV], int dim) {
    float ss = 0.f;
#pragma unroll
    for (int v = 0; v < NV; v++)
        ss += x[v].x * x[v].x + x[v].y * x[v].y + x[v].z * x[v].z + x[v].w * x[v].w;
    ss = warp_sum(ss);
    const float s = rms_scale(ss, dim);
#pragma unroll
    for (int v = 0; v < NV; v++) {
        x[v].x = __fmul_rn(__fmul_rn(x[v].x, s), g[v].x);
        x[v].y = __fmul_rn(__fmul_rn(x[v].y, s), g[v].y);
        x[v].z = __fmul_rn(__fmul_rn(x[v].z, s), g[v].z);
        x[v].w = __fmul_rn(__fmul_rn(x[v].w, s), g[v].w);
    }
}

template <int NV>
__device__ __forceinline__ void store_vec(float *dst, const float4 (&x)[NV], int c4, int lane) {
    float4 *d4 = reinterpret_cast<float4 *>(dst);
#pragma unroll
    for (int v = 0; v < NV; v++) {
        int c = lane + 32 * v;
        if (c < c4) d4[c] = x[v];
    }
}

// The input vector of a kernel, read ONCE per CTA: its threads load
// consecutive float4s into shared memory, and after a block barrier every
// warp takes its lanes' float4s from there. Reading it per warp made all
// warps of all CTAs fetch the same few L2 lines (about a thousand requests
// per line per kernel), which queued at the L2 slices holding them.
__device__ __forceinline__ void stage_vec(float4 *s_x4, const float *src, int c4) {
    const float4 *src4 = reinterpret_cast<const float4 *>(src);
    for (int i = threadIdx.x; i < c4; i += blockDim.x) s_x4[i] = __ldcg(src4 + i);
}

template <int NV>
__device__ __forceinline__ void vec_from_smem(float4 (&x)[NV], const float4 *s_x4, int c4, int lane) {
#pragma unroll
    for (int v = 0; v < NV; v++) {
        const int c = lane + 32 * v;
        x[v] = (c < c4) ? s_x4[c] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
}

// The same from a pipeline mailbox, written by another GPU: volatile loads.
__device__ __forceinline__ void stage_vec_cv(float4 *s_x4, const float *src, int c4) {
    const float4 *src4 = reinterpret_cast<const float4 *>(src);
    for (int i = threadIdx.x; i < c4; i += blockDim.x) s_x4[i] = __ldcv(src4 + i);
}

// Thread 0 of a CTA: wait for the message `want` (the link's message count)
// of position `pos` in this rank's mailbox, polling its sequence word with
// acquire semantics and giving up after m.link_timeout_ns of %globaltimer.
// After an expired wait, or a message for another position, the link error
// word is set (the host turns it into the reference's -1) and later waits on
// the broken link return at once; the kernel then computes on whatever the
// mailbox holds, and reaches all of its barriers.
__device__ __forceinline__ void box_poll(const DecodeModel &m, const unsigned char *box, unsigned want, int pos) {
    const MailboxHeader *h = reinterpret_cast<const MailboxHeader *>(box);
    if (*reinterpret_cast<volatile int *>(m.link_err)) return;
    const unsigned long long t0 = globaltimer_ns();
    while ((int)(ld_acquire_sys(&h->seq) - want) < 0) {
        if (globaltimer_ns() - t0 > m.link_timeout_ns) {
            atomicExch(m.link_err, 1);
            return;
        }
        __nanosleep(64);
    }
    if (__ldcv(&h->pos) != pos) atomicExch(m.link_err, 2);
}

__device__ __forceinline__ void link_poll(const DecodeModel &m, unsigned want, int pos) {
    box_poll(m, m.in_box, want, pos);
}

__device__ __forceinline__ const float *mailbox_x(const unsigned char *box) {
    return reinterpret_cast<const float *>(box + sizeof(MailboxHeader));
}

// Vocab-parallel classifier, thread 0 of the last CTA: send this rank's key
// for position p to the combining ranks (peer stores of the slot, then its
// sequence number with release semantics at system scope); a combining rank
// then waits for every other rank's key of p -- bounded like box_poll -- and
// returns the max over all ranks' keys, i.e. the argmax over the whole
// vocabulary with the single-GPU tie order (keys carry global row indices).
__device__ __forceinline__ unsigned long long vp_exchange(const DecodeModel &m, unsigned long long key, int p) {
    if (m.n_key_out) {
        const unsigned sq = *m.key_sent + 1;
        *m.key_sent = sq;
        for (int j = 0; j < m.n_key_out; j++) {
            KeySlot *ks = m.key_out[j] + m.vp_rank;
            ks->key = key;
            ks->pos = p;
        }
        __threadfence_system();
        for (int j = 0; j < m.n_key_out; j++) st_release_sys(&(m.key_out[j] + m.vp_rank)->seq, sq);
    }
    if (!m.vp_combine) return key;
    const KeySlot *slots = reinterpret_cast<const KeySlot *>(m.cls_box + sizeof(MailboxHeader) + (size_t)m.dim * 4);
    const unsigned want = m.step->key_recvd + m.tok_off + 1;
    if (*reinterpret_cast<volatile int *>(m.link_err)) return key;
    const unsigned long long t0 = globaltimer_ns();
    for (int q = 0; q < m.vp_ranks; q++) {
        if (q == m.vp_rank) continue;
        const KeySlot *ks = slots + q;
        while ((int)(ld_acquire_sys(&ks->seq) - want) < 0) {
            if (globaltimer_ns() - t0 > m.link_timeout_ns) {
                atomicExch(m.link_err, 1);
                return key;
            }
            __nanosleep(32);
        }
        if (__ldcv(&ks->pos) != p) atomicExch(m.link_err, 2);
        const unsigned long long kq = __ldcv(&ks->key);
        key = kq > key ? kq : key;
    }
    return key;
}

// Bytes of the shared-memory copy of an n-float vector (128-byte multiple).
__host__ __device__ constexpr int vec_smem_bytes(int n) { return (n * 4 + 127) / 128 * 128; }

// Phase timeline stamp by thread 0 of a CTA, only in the kernels' traced
// instantiation (template flag TR; the untraced ones carry no trace code):
// the slot of (position, kernel k, event e) keeps the earliest and the
// latest time.
__device__ __forceinline__ void trace_ev(const DecodeModel &m, bool on, int pos, int k, int e) {
    if (!on || threadIdx.x != 0) return;
    const unsigned long long t = globaltimer_ns();
    unsigned long long *slot = m.trace + 2 * (((size_t)(pos % TRACE_POS) * (2 * m.L + 1) + k) * TRACE_EV + e);
    atomicMin(slot, t);
    atomicMax(slot + 1, t);
}


// L2 eviction priority of the decode kernels' own loads: the layer weights
// and the KV rows are read once per token and marked evict_first, so that
// they do not push the small activation vectors and the next kernels' data
// out of L2 (measured 5052 -> 5139 tok/s at 110M against no hint; an
// evict_last mark on the classifier rows changed nothing).
constexpr int kPolWeights = POL_FIRST;
constexpr int kPolKV = POL_FIRST;

// A position outside the KV cache: the kernels compute nothing that could be
// mistaken for a result of it and record the error for the host.
__device__ __forceinline__ void flag_pos_range(const DecodeModel &m) {
    if (threadIdx.x == 0 && blockIdx.x == 0 && blockIdx.y == 0) atomicExch(m.err, ERR_POS_RANGE);
}

// ---------------------------------------------------------------------------
// k_attn: grid (n_heads, n_chunks), 256 threads. CTA (h, c) covers positions
// [c*CH, c*CH+CH) ∩ [0, pos] (CH = 64): scores q.k * 1/sqrt(hd), a
// chunk-local softmax numerator with pitorch's exp, and the weighted value
// sum. The last CTA of each head merges the chunks with the usual
// max-rescaling, which equals softmax-then-weight (llama2.c:250-274) up to
// float rounding. Every phase issues its loads independently (4 threads per
// position for the scores, (float4 column, position group) threads for the
// values and the merge), so a phase costs one memory round trip.
// ---------------------------------------------------------------------------
constexpr int ATT_THREADS = 256;
constexpr int ATT_MAX_CHUNKS = 64;
constexpr int ATT_MERGE_PER_THREAD = 4;   // chunks per merge thread: needs n_chunks <= 4 * groups

__global__ void __launch_bounds__(ATT_THREADS, 2) k_attn(DecodeModel m, int l) {
    pdl_trigger();
    __shared__ float s_p[ATT_MAX_CHUNKS];
    __shared__ float s_l[ATT_MAX_CHUNKS];
    __shared__ __align__(16) float s_o[ATT_THREADS * 4];
    __shared__ float s_stat[2];
    __shared__ int s_last;

    const int h = blockIdx.x, c = blockIdx.y;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int hd = m.hd, hd4 = hd >> 2, CH = m.att_chunk;
    const int kvh = h / (m.nh / m.nkv);
    const int ngrp = ATT_THREADS / hd4;      // position groups for the value pass
    const int d4 = tid % hd4, grp = tid / hd4;
    // The position and every K/V row before it were written by earlier
    // launches (earlier tokens, or this graph's first node), so they are
    // read before the wait; only q and the row of `pos` come from the
    // kernel this one depends on.
    const int pos_raw = __ldcg(&m.step->pos) + m.tok_off;
    if (pos_raw < 0 || pos_raw >= m.seq) {
        flag_pos_range(m);
        return;
    }
    const int pos = pos_raw;
    const int t0 = c * CH;
    const int nc = pos / CH + 1;   // chunks holding positions <= pos
    if (c >= nc) return;           // no positions here: not part of the merge
    const int n = min(CH, pos + 1 - t0);
    const int jcur = pos - t0;     // the current position's slot, if < n
    const size_t head_base = ((size_t)l * m.nkv + kvh) * m.seq;
    const float4 *kb = reinterpret_cast<const float4 *>(m.kc + (head_base + t0) * hd);
    const float4 *vb = reinterpret_cast<const float4 *>(m.vc + (head_base + t0) * hd);
    const int js = tid >> 2, sub = tid & 3;
    constexpr int QK = 4, VP = 4;
    float4 kv[QK], vpre[VP], qv[QK];
#pragma unroll
    for (int i = 0; i < QK; i++) {
        const int cc = sub + 4 * i;
        kv[i] = (cc < hd4 && js < n && js < jcur - 1) ? __ldcg(kb + (size_t)js * hd4 + cc)
                                                      : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int k = 0; k < VP; k++) {
        const int j = grp + ngrp * k;
        vpre[k] = (grp < ngrp && j < n && j < jcur - 1) ? __ldcg(vb + (size_t)j * hd4 + d4)
                                                        : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    pdl_wait();
    // the row of pos - 1 (written by the previous position's kernels, which
    // a short chain of programmatic launches may not have finished when this
    // kernel starts) is read after the wait, with the row of pos
#pragma unroll
    for (int i = 0; i < QK; i++) {
        const int cc = sub + 4 * i;
        if (cc < hd4 && js == jcur - 1 && js >= 0) kv[i] = __ldcg(kb + (size_t)js * hd4 + cc);
    }
#pragma unroll
    for (int k = 0; k < VP; k++)
        if (grp < ngrp && grp + ngrp * k == jcur - 1 && jcur >= 1) vpre[k] = __ldcg(vb + (size_t)(jcur - 1) * hd4 + d4);
    const float scale = __fdiv_rn(1.0f, pt_sqrtf((float)hd));
    float *part = m.att_part + ((size_t)h * m.n_chunks + c) * (hd + 2);
    const float4 *q4 = reinterpret_cast<const float4 *>(m.q + h * hd);
#pragma unroll
    for (int i = 0; i < QK; i++) {
        const int cc = sub + 4 * i;
        qv[i] = (cc < hd4) ? __ldcg(q4 + cc) : make_float4(0.f, 0.f, 0.f, 0.f);
        if (cc < hd4 && js == jcur) kv[i] = __ldcg(kb + (size_t)js * hd4 + cc);
    }
#pragma unroll
    for (int k = 0; k < VP; k++)
        if (grp < ngrp && grp + ngrp * k == jcur) vpre[k] = __ldcg(vb + (size_t)jcur * hd4 + d4);
    {
        float acc = 0.f;
#pragma unroll
        for (int i = 0; i < QK; i++) acc = dot4(kv[i], qv[i], acc);
        acc += __shfl_xor_sync(0xffffffffu, acc, 1);
        acc += __shfl_xor_sync(0xffffffffu, acc, 2);
        if (js < n && sub == 0) s_p[js] = __fmul_rn(acc, scale);
    }
    __syncthreads();
    if (warp == 0) {
        float mx = -3.4028235e+38f;
        for (int j = lane; j < n; j += 32) mx = fmaxf(mx, s_p[j]);
        mx = warp_max(mx);
        float sum = 0.f;
        for (int j = lane; j < n; j += 32) {
            const float e = pt_expf(__fsub_rn(s_p[j], mx));
            s_p[j] = e;
            sum += e;
        }
        sum = warp_sum(sum);
        if (lane == 0) { s_stat[0] = mx; s_stat[1] = sum; }
    }
    __syncthreads();
    if (grp < ngrp) {
        float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int k = 0; k < VP; k++) {
            const int j = grp + ngrp * k;
            if (j < n) {
                const float e = s_p[j];
                o.x = fmaf(e, vpre[k].x, o.x); o.y = fmaf(e, vpre[k].y, o.y);
                o.z = fmaf(e, vpre[k].z, o.z); o.w = fmaf(e, vpre[k].w, o.w);
            }
        }
        reinterpret_cast<float4 *>(s_o)[grp * hd4 + d4] = o;
    }
    __syncthreads();
    {
        if (nc == 1) {   // one chunk: normalise and finish here
            const float inv = __fdiv_rn(1.0f, s_stat[1]);
            for (int d = tid; d < hd; d += ATT_THREADS) {
                float o = 0.f;
                for (int g = 0; g < ngrp; g++) o += s_o[g * hd + d];
                m.att[h * hd + d] = o * inv;
            }
            return;
        }
        for (int d = tid; d < hd; d += ATT_THREADS) {
            float o = 0.f;
            for (int g = 0; g < ngrp; g++) o += s_o[g * hd + d];
            part[d] = o;
        }
        if (tid == 0) { part[hd] = s_stat[0]; part[hd + 1] = s_stat[1]; }
    }
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        const unsigned ticket = atomicAdd(&m.att_ticket[h], 1u);
        s_last = (ticket == (unsigned)nc - 1);
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    // Merge the nc chunk partials of this head: every load (chunk maxima,
    // sums and this thread's slice of the partial outputs) is issued in one
    // round, then the max-rescaling runs from shared memory and registers.
    const float *hp = m.att_part + (size_t)h * m.n_chunks * (hd + 2);
    constexpr int MK = ATT_MERGE_PER_THREAD;
    float4 po[MK];
#pragma unroll
    for (int q = 0; q < MK; q++) {
        const int k = grp + ngrp * q;
        const float *pk = hp + (size_t)k * (hd + 2) + 4 * d4;
        po[q] = (grp < ngrp && k < nc) ? make_float4(__ldcg(pk), __ldcg(pk + 1), __ldcg(pk + 2), __ldcg(pk + 3))
                                        : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    for (int k = tid; k < nc; k += ATT_THREADS) {
        s_p[k] = __ldcg(hp + (size_t)k * (hd + 2) + hd);
        s_l[k] = __ldcg(hp + (size_t)k * (hd + 2) + hd + 1);
    }
    __syncthreads();
    if (warp == 0) {
        float M = -3.4028235e+38f;
        for (int k = lane; k < nc; k += 32) M = fmaxf(M, s_p[k]);
        M = warp_max(M);
        if (lane == 0) s_stat[0] = M;
    }
    __syncthreads();
    const float M = s_stat[0];
    for (int k = tid; k < nc; k += ATT_THREADS) s_p[k] = pt_expf(__fsub_rn(s_p[k], M));
    __syncthreads();
    if (tid == 0) {
        float L = 0.f;
        for (int k = 0; k < nc; k++) L = fmaf(s_p[k], s_l[k], L);
        s_stat[1] = __fdiv_rn(1.0f, L);
    }
    if (grp < ngrp) {
        float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int q = 0; q < MK; q++) {
            const int k = grp + ngrp * q;
            if (k < nc) {
                const float w = s_p[k];
                o.x = fmaf(w, po[q].x, o.x); o.y = fmaf(w, po[q].y, o.y);
                o.z = fmaf(w, po[q].z, o.z); o.w = fmaf(w, po[q].w, o.w);
            }
        }
        reinterpret_cast<float4 *>(s_o)[grp * hd4 + d4] = o;
    }
    __syncthreads();
    const float invL = s_stat[1];
    for (int d = tid; d < hd; d += ATT_THREADS) {
        float o = 0.f;
        for (int g = 0; g < ngrp; g++) o += s_o[g * hd + d];
        m.att[h * hd + d] = o * invL;
    }
    if (tid == 0) m.att_ticket[h] = 0u;
}

// ---------------------------------------------------------------------------
// k_mv: the decode matvecs. Grid = one CTA per SM; CTA b owns a contiguous
// block of "items" (a row, or a row pair) and streams the item rows through
// MV_STAGES shared-memory stages with bulk (TMA) copies signalled on
// mbarriers. The first stages are issued BEFORE griddepcontrol.wait: weights
// never depend on the previous kernel, so under programmatic dependent
// launch this kernel's weight stream overlaps the tail of the previous one.
// After the wait the CTA loads the (small) input vector from L2 into
// registers, and each warp reduces its items from shared memory.
//
//   MV_QKV    item = row pair (2j, 2j+1) of [wq; wk; wv]; rmsnorm(x) in;
//             RoPE epilogue, k/v into the KV cache slot of pos
//             (llama2.c:238-248). Layer 0 reads the token's embedding row.
//   MV_FFN13  item = hidden unit i: rows w1[i], w3[i]; rmsnorm(x) in;
//             hb[i] = silu(h1) * h3 (llama2.c:280-285)
//   MV_RESID  item = row r of W (wo or w2); x[r] += W[r] . in (:276-277, :286-287)
//   MV_CLS    item = vocab row r; rmsnorm(x, rms_final) in; logits[r] and a
//             greedy argmax (llama2.c:293-294, pt.c:270)
// ---------------------------------------------------------------------------
enum MvMode { MV_QKV = 0, MV_FFN13 = 1, MV_RESID = 2, MV_CLS = 3 };

// Ring geometry of the classifier (the other modes use MV_STAGES stages of
// MV_STAGE_BYTES).
#ifndef PTC_CLS_STAGE_KB
#define PTC_CLS_STAGE_KB 24
#endif
#ifndef PTC_CLS_STAGES
#define PTC_CLS_STAGES 4
#endif
constexpr int CLS_STAGE_BYTES = PTC_CLS_STAGE_KB * 1024;
constexpr int CLS_STAGES = PTC_CLS_STAGES;
static_assert(CLS_STAGES * 8 <= MV_BAR_BYTES && MV_STAGES * 8 <= MV_BAR_BYTES, "mbarriers do not fit");

struct MvArgs {
    const float *W;    // MV_RESID: the matrix; MV_CLS: wcls
    const float *in;   // MV_RESID: input vector; MV_QKV: the layer input x
    float *res_in;        // MV_RESID: residual source, row r read once
    float *res_out;       // MV_RESID: receives res_in[r] + W[r] . in
    int zero_res_in;      // MV_RESID: clear res_in[r] after reading it
    int n_items;       // items over the whole grid
    int cols;          // row length in floats
    int slots;         // rows per item
    int per_stage;     // items per shared-memory stage
    int l;             // layer
    int from_embedding;
    int *host_next;    // MV_CLS: pinned host word that also receives the argmax (null: none)
    int recv;          // MV_CLS: x from this rank's mailbox (pipeline head rank)
    int send_next;     // MV_CLS, device loop: the next token's embedding row to the next stage
    int vp;            // MV_CLS: this rank's rows of a vocab-parallel classifier (link form)
    int row0;          // MV_CLS: global index of the first row (vocab-parallel slice)
    int vp_cls;        // MV_CLS: x from this rank's classifier mailbox (vocab-parallel)
    int adv_recvd;     // MV_CLS, last position of a graph: this stage's layers took one message per position
};

template <int MODE>
__device__ __forceinline__ void mv_issue(const DecodeModel &m, const MvArgs &a, float *stage, uint64_t *bar,
                                         int c0, int c1) {
    const size_t rb = (size_t)a.cols * 4;  // bytes per row
    const int n = c1 - c0;
    if (MODE == MV_QKV) {
        // virtual rows [2c0, 2c1) of [wq; wk; wv], split at the matrix edges
        const size_t D = m.dim, K = m.kvd;
        const float *base[3] = {m.wq + (size_t)a.l * D * D, m.wk + (size_t)a.l * K * D,
                                m.wv + (size_t)a.l * K * D};
        const int edge[4] = {0, m.dim, m.dim + m.kvd, m.dim + 2 * m.kvd};
        mbar_expect_tx(bar, (unsigned)(2 * n * rb));
        const int r0 = 2 * c0, r1 = 2 * c1;
        for (int s = 0; s < 3; s++) {
            const int lo = max(r0, edge[s]), hi = min(r1, edge[s + 1]);
            if (lo < hi)
                bulk_g2s(stage + (size_t)(lo - r0) * a.cols, base[s] + (size_t)(lo - edge[s]) * a.cols,
                         (unsigned)((hi - lo) * rb), bar);
        }
    } else if (MODE == MV_FFN13) {
        const size_t off = (size_t)a.l * m.hidden * m.dim + (size_t)c0 * m.dim;
        mbar_expect_tx(bar, (unsigned)(2 * n * rb));
        bulk_g2s(stage, m.w1 + off, (unsigned)(n * rb), bar);
        bulk_g2s(stage + (size_t)a.per_stage * a.cols, m.w3 + off, (unsigned)(n * rb), bar);
    } else {
        mbar_expect_tx(bar, (unsigned)(n * rb));
        bulk_g2s(stage, a.W + (size_t)c0 * a.cols, (unsigned)(n * rb), bar);
    }
}

template <int NV>
__device__ __forceinline__ float smem_row_dot(const float *row, const float4 (&x)[NV], int c4, int lane) {
    const float4 *r4 = reinterpret_cast<const float4 *>(row);
    float acc = 0.f;
#pragma unroll
    for (int v = 0; v < NV; v++) {
        const int c = lane + 32 * v;
        if (c < c4) acc = dot4(r4[c], x[v], acc);
    }
    return warp_sum(acc);
}

template <int NV, int MODE, bool TR>
__global__ void __launch_bounds__(MV_THREADS, 2) k_mv(DecodeModel m, MvArgs a) {
    pdl_trigger();
    extern __shared__ __align__(128) unsigned char smem_raw[];
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem_raw);
    // the input vector, staged once per CTA (not for the classifier: its x
    // read queues behind its own 98 MB stream either way, and the 3 KB would
    // keep it from sharing an SM with the last FFN block)
    float4 *s_x4 = reinterpret_cast<float4 *>(smem_raw + MV_BAR_BYTES);
    float *stages = reinterpret_cast<float *>(smem_raw + MV_BAR_BYTES + (MODE == MV_CLS ? 0 : vec_smem_bytes(a.cols)));
    __shared__ unsigned long long s_best[MV_THREADS / 32];
    __shared__ int s_last;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int NW = MV_THREADS / 32;
    const int it0 = (int)((long)a.n_items * blockIdx.x / gridDim.x);
    const int it1 = (int)((long)a.n_items * (blockIdx.x + 1) / gridDim.x);
    const int ps = a.per_stage;
    const int n_chunks = (it1 - it0 + ps - 1) / ps;
    constexpr int NST = MODE == MV_CLS ? CLS_STAGES : MV_STAGES;
    const int stage_floats = (MODE == MV_CLS ? CLS_STAGE_BYTES : MV_STAGE_BYTES) / 4;
    const int c4 = a.cols >> 2;

    if (tid == 0) {
        for (int s = 0; s < NST; s++) mbar_init(&bars[s], 1);
        mbar_init_fence();
    }
    __syncthreads();
    if (tid == 0)
        for (int k = 0; k < n_chunks && k < NST; k++)
            mv_issue<MODE>(m, a, stages + k * stage_floats, &bars[k], it0 + k * ps, min(it1, it0 + (k + 1) * ps));

    // Everything that does not come from the kernel this one depends on is
    // loaded before the wait: rmsnorm gains (weights), the position and --
    // for layer 0 -- the token's embedding row (set by an earlier launch).
    float4 xr[NV], gr[NV];
    int pos = 0;
    constexpr bool tr = MODE == MV_CLS && TR;
    const int tpos = (tr || (MODE == MV_CLS && (a.recv || a.vp_cls))) ? __ldcg(&m.step->pos) + m.tok_off : 0;
    // the link's message for this position (read before the wait: only the
    // last kernel of a graph moves the count on)
    const unsigned want = (MODE == MV_CLS && a.recv)     ? __ldcg(&m.step->recvd) + m.tok_off + 1
                          : (MODE == MV_CLS && a.vp_cls) ? __ldcg(&m.step->cls_recvd) + m.tok_off + 1
                                                         : 0u;
    trace_ev(m, tr, tpos, 2 * m.L, 0);
    const bool early = MODE == MV_QKV && a.from_embedding && m.tok_off == 0;
    if (MODE == MV_QKV) {
        pos = __ldcg(&m.step->pos) + m.tok_off;
        load_gain<NV>(gr, m.rms_att + (size_t)a.l * m.dim, c4, lane);
        if (early) stage_vec(s_x4, m.emb + (size_t)__ldcg(&m.step->tok) * m.dim, c4);
    } else if (MODE == MV_FFN13) {
        load_gain<NV>(gr, m.rms_ffn + (size_t)a.l * m.dim, c4, lane);
    } else if (MODE == MV_CLS) {
        load_gain<NV>(gr, m.rms_final, c4, lane);
    }
    pdl_wait();
    trace_ev(m, tr, tpos, 2 * m.L, 1);
    // residual rows this warp will update (RESID): issued with the input
    constexpr int XPRE = 4;
    float xres[XPRE];
    if (MODE == MV_RESID) {
#pragma unroll
        for (int q = 0; q < XPRE; q++) {
            const int i = it0 + warp + q * NW;   // this warp's q-th item (direct mode)
            xres[q] = (lane == 0 && n_chunks <= NST && i < it1) ? __ldcg(a.res_in + i) : 0.f;
        }
    }
    if (MODE == MV_CLS) {
        if (a.recv || a.vp_cls) {   // pipeline: x is the last layer rank's message
            const unsigned char *box = a.recv ? m.in_box : m.cls_box;
            if (tid == 0) box_poll(m, box, want, tpos);
            __syncthreads();
            const float4 *b4 = reinterpret_cast<const float4 *>(mailbox_x(box));
#pragma unroll
            for (int v = 0; v < NV; v++) {
                const int c = lane + 32 * v;
                xr[v] = (c < c4) ? __ldcv(b4 + c) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
        } else {
            load_act<NV>(xr, m.x, c4, lane);
        }
    } else {
        if (!early) {
            const float *src = a.in;
            if (MODE == MV_QKV && a.from_embedding) src = m.emb + (size_t)__ldcg(&m.step->tok) * m.dim;
            if (MODE == MV_FFN13) src = m.x;
            stage_vec(s_x4, src, c4);
        }
        __syncthreads();
        vec_from_smem<NV>(xr, s_x4, c4, lane);
    }
    if (MODE == MV_QKV) {
        if (a.from_embedding && blockIdx.x == 0 && warp == 0) store_vec<NV>(m.x, xr, c4, lane);
        rmsnorm_pre<NV>(xr, gr, m.dim);
    } else if (MODE == MV_FFN13) {
        rmsnorm_pre<NV>(xr, gr, m.dim);
    } else if (MODE == MV_CLS) {
        rmsnorm_pre<NV>(xr, gr, m.dim);
        if (blockIdx.x == 0 && warp == 0) store_vec<NV>(m.xn, xr, c4, lane);
        trace_ev(m, tr, tpos, 2 * m.L, 2);
    }
    const bool pos_ok = (MODE != MV_QKV) || (pos >= 0 && pos < m.seq);
    if (!pos_ok) flag_pos_range(m);

    unsigned long long best = 0ull;
    bool ok = true;
    // One item (row or row pair) from a filled stage: dot products + epilogue.
    auto do_item = [&](const float *stage, int li, int i, float xo) {
        if (MODE == MV_QKV) {
            const float a0 = smem_row_dot<NV>(stage + (size_t)(2 * li) * a.cols, xr, c4, lane);
            const float a1 = smem_row_dot<NV>(stage + (size_t)(2 * li + 1) * a.cols, xr, c4, lane);
            if (lane == 0 && pos_ok) {
                const int r0 = 2 * i, hd = m.hd;
                if (r0 < m.dim + m.kvd) {
                    const bool is_q = r0 < m.dim;
                    const int j = is_q ? r0 : r0 - m.dim;
                    const float th = rope_theta(j, hd, pos);
                    const float cs = pt_cosf(th), sn = pt_sinf(th);
                    const float o0 = __fsub_rn(__fmul_rn(a0, cs), __fmul_rn(a1, sn));
                    const float o1 = __fadd_rn(__fmul_rn(a0, sn), __fmul_rn(a1, cs));
                    if (is_q) {
                        m.q[j] = o0;
                        m.q[j + 1] = o1;
                    } else {
                        float *dst = m.kc + (((size_t)a.l * m.nkv + j / hd) * m.seq + pos) * hd + (j % hd);
                        dst[0] = o0;
                        dst[1] = o1;
                    }
                } else {
                    const int j = r0 - m.dim - m.kvd;
                    float *dst = m.vc + (((size_t)a.l * m.nkv + j / hd) * m.seq + pos) * hd + (j % hd);
                    dst[0] = a0;
                    dst[1] = a1;
                }
            }
        } else if (MODE == MV_FFN13) {
            const float h1 = smem_row_dot<NV>(stage + (size_t)li * a.cols, xr, c4, lane);
            const float h3 = smem_row_dot<NV>(stage + (size_t)(ps + li) * a.cols, xr, c4, lane);
            if (lane == 0) m.hb[i] = silu_mul(h1, h3);
        } else if (MODE == MV_RESID) {
            const float v = smem_row_dot<NV>(stage + (size_t)li * a.cols, xr, c4, lane);
            if (lane == 0) {
                a.res_out[i] = __fadd_rn(xo, v);
                if (a.zero_res_in) a.res_in[i] = 0.f;
            }
        } else {
            const float v = smem_row_dot<NV>(stage + (size_t)li * a.cols, xr, c4, lane);
            if (lane == 0) {
                m.logits[a.row0 + i] = v;
                const unsigned long long key = argmax_key(v, a.row0 + i);
                if (key > best) best = key;
            }
        }
    };
    if (n_chunks <= NST) {
        // The whole block is in flight at once: each warp takes its items
        // directly, waiting only for the stage that holds each one.
        int q = 0;
        for (int i = it0 + warp; i < it1; i += NW, q++) {
            const int k = (i - it0) / ps;
            if (!mbar_wait_bounded(&bars[k], 0u, m.err, ERR_MBAR_TIMEOUT)) {
                ok = false;
                break;
            }
            float xo = 0.f;
            if (MODE == MV_RESID && lane == 0) {
#pragma unroll
                for (int t = 0; t < XPRE; t++) if (t == q) xo = xres[t];
                if (q >= XPRE) xo = __ldcg(a.res_in + i);
            }
            do_item(stages + k * stage_floats, (i - it0) % ps, i, xo);
        }
        // a warp that gave up leaves copies in flight: let them land
        if (!ok && lane == 0)
            for (int k = 0; k < n_chunks; k++) mbar_wait_bounded(&bars[k], 0u, nullptr, 0);
    } else {
        for (int k = 0; k < n_chunks; k++) {
            const int s = k % NST;
            const float *stage = stages + s * stage_floats;
            const bool got = mbar_wait_bounded(&bars[s], (unsigned)((k / NST) & 1), m.err, ERR_MBAR_TIMEOUT);
            if (__syncthreads_or(!got)) {   // block-uniform give-up
                ok = false;
                if (tid == 0)   // let copies still in flight land before the CTA exits
                    for (int kk = k + 1; kk < n_chunks && kk < k + NST; kk++)
                        mbar_wait_bounded(&bars[kk % NST], (unsigned)((kk / NST) & 1), nullptr, 0);
                break;
            }
            const int c0 = it0 + k * ps, c1 = min(it1, c0 + ps);
            for (int i = c0 + warp; i < c1; i += NW)
                do_item(stage, i - c0, i, (MODE == MV_RESID && lane == 0) ? __ldcg(a.res_in + i) : 0.f);
            __syncthreads();
            if (tid == 0 && k + NST < n_chunks) {
                fence_proxy_async_smem();
                const int kk = k + NST;
                mv_issue<MODE>(m, a, stages + s * stage_floats, &bars[s], it0 + kk * ps, min(it1, it0 + (kk + 1) * ps));
            }
        }
    }
    (void)ok;
    if (MODE != MV_CLS) return;

    if (lane == 0) s_best[warp] = best;
    __syncthreads();
    trace_ev(m, tr, tpos, 2 * m.L, 6);
    StepState *st = m.step;
    int err_seen = 0;   // thread 0: an earlier kernel's expired wait (host steps)
    if (tid == 0) {
        if (a.host_next) err_seen = __ldcg(m.err);   // its latency overlaps the atomics below
        unsigned long long b = 0ull;
        for (int w = 0; w < NW; w++) b = s_best[w] > b ? s_best[w] : b;
        // the CTA's best key, then its ticket with release semantics (which
        // orders the max before it) and acquire semantics (so the last CTA
        // sees every other CTA's max): two global round trips in all
        if (b) red_max_u64(&st->amax, b);
        const unsigned ticket = atom_add_acq_rel(&st->done, 1u);
        s_last = (ticket == gridDim.x - 1);
    }
    __syncthreads();
    if (!s_last) return;
    __shared__ int s_send_tok, s_send_pos;
    if (tid == 0) {
        unsigned long long key = __ldcg(&st->amax);
        const int p = st->pos + m.tok_off;
        st->amax = 0ull;
        st->done = 0u;
        // vocab-parallel: this rank's key out, and on a combining rank the
        // max over every rank's key in
        if (a.vp) key = vp_exchange(m, key, p);
        int send_tok = -1;
        if (!a.vp || m.vp_combine) {
            const int next = argmax_key_index(key);
            st->next = next;
            if (a.host_next) {   // straight into the host's pinned word: no copy node after the kernel
                // -1 sends the host to the error word, so a token computed after an
                // expired wait is never returned as valid
                *reinterpret_cast<volatile int *>(a.host_next) = err_seen ? -1 : next;
                __threadfence_system();   // on its way to the host before the grid ends
            }
            if (st->mode == 1 && p < m.seq) {
                int t = next;
                if (p + 1 < st->n_prompt) t = st->tokens[p + 1];
                else st->tokens[p + 1] = next;
                st->tok = t;
                if (m.adv) st->pos = p + 1;
                if (a.send_next && p + 1 < st->stop) send_tok = t;
            }
        }
        if (m.adv) {
            // every rank of a vocab-parallel split keeps its own position; the
            // message counts move on by the positions of this graph
            if (a.vp) st->pos = p + 1;
            if (a.recv || a.adv_recvd) st->recvd = st->recvd + m.tok_off + 1;
            if (a.vp_cls) st->cls_recvd = st->cls_recvd + m.tok_off + 1;
            if (a.vp && m.vp_combine) st->key_recvd = st->key_recvd + m.tok_off + 1;
        }
        s_send_tok = send_tok;
        s_send_pos = p + 1;
    }
    __syncthreads();
    if (s_send_tok >= 0) {
        // Pipeline head rank: the next position's input -- the embedding row
        // of the token just chosen -- goes straight into the first layer
        // rank's mailbox (peer stores over NVLink), published after a
        // system-scope fence; no embedding or send kernel follows.
        MailboxHeader *oh = reinterpret_cast<MailboxHeader *>(m.out_box);
        float4 *ox = reinterpret_cast<float4 *>(m.out_box + sizeof(MailboxHeader));
        const float4 *er = reinterpret_cast<const float4 *>(m.emb + (size_t)s_send_tok * m.dim);
        for (int i = tid; i < c4; i += MV_THREADS) ox[i] = __ldg(er + i);
        if (tid == 0) oh->pos = s_send_pos;
        __threadfence_system();
        __syncthreads();
        if (tid == 0) {
            const unsigned sq = *m.link_sent + 1;
            *m.link_sent = sq;
            st_release_sys(&oh->seq, sq);
        }
    }
    // no fence for the step state: the next kernel reads it after
    // griddepcontrol.wait, and the host after the stream synchronises --
    // both see a completed grid's writes
    trace_ev(m, tr, tpos, 2 * m.L, 7);
}

// A pipeline layer rank's output: x (m.x, complete -- this kernel is
// launched without programmatic overlap, after the last layer's kernels)
// into the next stage's mailbox with peer stores, published after a
// system-scope fence. The last position of a stage graph (adv) then moves
// the rank's own position and message count on. With the vocab-parallel
// classifier the last layer rank sends its output to every other rank's
// classifier mailbox instead (the ranks' own classifiers then move the
// positions and counts on).
//
// It must stay a full boundary: the next position's first attention block
// reads the K/V rows of earlier positions before its griddepcontrol.wait,
// and on a rank with one or two layers the row of the position just decoded
// is written only a few kernels earlier. Launched programmatically (and
// releasing its dependent at once), that block could start while the row
// was still being written: on 8 GPUs (1-2 layers per rank) the token stream
// then diverged at position 51.
__global__ void k_stage_send(DecodeModel m) {
    const int pos = __ldcg(&m.step->pos) + m.tok_off;
    const bool bcast = m.vp_rows && m.n_cls_out;   // (stage graphs only: link form)
    const int n_out = bcast ? m.n_cls_out : 1;
    const float4 *x4 = reinterpret_cast<const float4 *>(m.x);
    for (int i = threadIdx.x; i < m.dim / 4; i += blockDim.x) {
        const float4 v = __ldcg(x4 + i);
        for (int j = 0; j < n_out; j++)
            reinterpret_cast<float4 *>((bcast ? m.cls_out[j] : m.out_box) + sizeof(MailboxHeader))[i] = v;
    }
    if (threadIdx.x < n_out)
        reinterpret_cast<MailboxHeader *>(bcast ? m.cls_out[threadIdx.x] : m.out_box)->pos = pos;
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned *ctr = bcast ? m.cls_sent : m.link_sent;
        const unsigned sq = *ctr + 1;
        *ctr = sq;
        for (int j = 0; j < n_out; j++)
            st_release_sys(&reinterpret_cast<MailboxHeader *>(bcast ? m.cls_out[j] : m.out_box)->seq, sq);
        if (m.adv && !m.vp_rows) {
            m.step->pos = pos + 1;
            m.step->recvd = m.step->recvd + m.tok_off + 1;
        }
    }
}

void launch_stage_send(const DecodeModel &m, cudaStream_t s) {
    k_stage_send<<<1, 256, 0, s>>>(m);
    PTC_CHECK(cudaGetLastError());
}

// ---------------------------------------------------------------------------
// k_ffn: the whole feed-forward block of one layer in one kernel
// (llama2.c:279-287): rmsnorm(x) -> h1 = w1 x, h3 = w3 x -> hb = silu(h1)*h3
// -> x_out = x + w2 hb. CTA b owns hidden units [j0, j1): it holds their
// w1 and w3 rows and the matching rows of the transposed w2 (w2t[j] = column
// j of w2) in shared memory, all fetched by bulk copies before
// griddepcontrol.wait. After the wait it normalises x, produces its hb
// values, and adds its partial w2 product -- a full dim-vector -- into the
// zeroed output with vector reductions at L2 (CTA 0 also adds the residual).
// The split over hidden units makes w2 a split-K product summed by L2
// atomics, so no other kernel has to wait for hb.
// ---------------------------------------------------------------------------
constexpr int FF_MAX_ROWS = 64;

struct FfnArgs {
    const float *xin;  // FFN input and residual (post-attention x)
    float *xout;       // zero on entry; receives x + w2 . hb
    float *xclear;     // cleared once every CTA has read the input (null: none)
    int l;
};

template <int NV, bool TR>
__global__ void __launch_bounds__(FF_THREADS, 1) k_ffn(DecodeModel m, FfnArgs a) {
    pdl_trigger();
    extern __shared__ __align__(128) unsigned char smem_raw[];
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem_raw);
    const int dim = m.dim, c4 = dim >> 2, R = m.ffn_rows;
    float4 *s_x4 = reinterpret_cast<float4 *>(smem_raw + MV_BAR_BYTES);                    // the FFN input
    float *w1s = reinterpret_cast<float *>(smem_raw + MV_BAR_BYTES + vec_smem_bytes(dim));   // [R][dim]
    float *w3s = w1s + (size_t)R * dim;                                 // [R][dim]
    float *w2s = w3s + (size_t)R * dim;                                 // [R][dim]
    __shared__ float s_hb[FF_MAX_ROWS];
    __shared__ int s_last;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int NW = FF_THREADS / 32;
    const int j0 = (int)((long)m.hidden * blockIdx.x / gridDim.x);
    const int j1 = (int)((long)m.hidden * (blockIdx.x + 1) / gridDim.x);
    const int nj = j1 - j0;
    const unsigned bytes = (unsigned)nj * (unsigned)dim * 4u;
    constexpr bool tr = TR;
    const int tpos = tr ? __ldcg(&m.step->pos) + m.tok_off : 0;
    trace_ev(m, tr, tpos, 2 * a.l + 1, 0);
    if (tid == 0) {
        mbar_init(&bars[0], 1);
        mbar_init(&bars[1], 1);
        mbar_init_fence();
    }
    __syncthreads();
    if (tid == 0) {
        // one bulk copy per row: the rows then stream in parallel (one copy
        // per matrix measured 3.6 us/token slower at 110M)
        const size_t off = ((size_t)a.l * m.hidden + j0) * dim;
        const unsigned rb = (unsigned)dim * 4u;
        constexpr int pk = kPolWeights;
        const uint64_t pol = make_l2_policy(pk);
        mbar_expect_tx(&bars[0], 2u * bytes);
        mbar_expect_tx(&bars[1], bytes);
        for (int j = 0; j < nj; j++) {
            bulk_g2s_pol(w1s + (size_t)j * dim, m.w1 + off + (size_t)j * dim, rb, &bars[0], pk, pol);
            bulk_g2s_pol(w3s + (size_t)j * dim, m.w3 + off + (size_t)j * dim, rb, &bars[0], pk, pol);
        }
        for (int j = 0; j < nj; j++)
            bulk_g2s_pol(w2s + (size_t)j * dim, m.w2t + off + (size_t)j * dim, rb, &bars[1], pk, pol);
    }
    float4 xr[NV], gr[NV];
    load_gain<NV>(gr, m.rms_ffn + (size_t)a.l * dim, c4, lane);
    pdl_wait();
    trace_ev(m, tr, tpos, 2 * a.l + 1, 1);
    stage_vec(s_x4, a.xin, c4);
    __syncthreads();
    // x is in shared memory: the CTA is done with a.xin and takes its ticket
    // now; the result is only looked at when the CTA ends
    unsigned ticket = 0u;
    if (a.xclear && tid == FF_THREADS - 1) ticket = atomicAdd(&m.tickets[1], 1u);
    vec_from_smem<NV>(xr, s_x4, c4, lane);
    // the residual this thread adds (CTA 0)
    constexpr int RV = 2;   // float4 columns per thread: dim <= 4 * RV * FF_THREADS
    float4 res[RV];
#pragma unroll
    for (int r = 0; r < RV; r++) {
        const int c = tid + r * FF_THREADS;
        res[r] = (blockIdx.x == 0 && c < c4) ? s_x4[c] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    rmsnorm_pre<NV>(xr, gr, dim);
    trace_ev(m, tr, tpos, 2 * a.l + 1, 2);

    // A failed wait is recorded in m.err; the CTA then skips its products
    // but still takes part in the ticket.
    bool ok = __syncthreads_and(mbar_wait_bounded(&bars[0], 0u, m.err, ERR_MBAR_TIMEOUT));
    trace_ev(m, tr, tpos, 2 * a.l + 1, 3);
    if (ok)
        for (int j = warp; j < nj; j += NW) {
            const float h1 = smem_row_dot<NV>(w1s + (size_t)j * dim, xr, c4, lane);
            const float h3 = smem_row_dot<NV>(w3s + (size_t)j * dim, xr, c4, lane);
            if (lane == 0) s_hb[j] = silu_mul(h1, h3);
        }
    trace_ev(m, tr, tpos, 2 * a.l + 1, 8);
    if (ok) ok = mbar_wait_bounded(&bars[1], 0u, m.err, ERR_MBAR_TIMEOUT);
    ok = __syncthreads_and(ok);   // also publishes s_hb
    trace_ev(m, tr, tpos, 2 * a.l + 1, 4);
    if (ok) {
        const float4 *w2s4 = reinterpret_cast<const float4 *>(w2s);
#pragma unroll
        for (int r = 0; r < RV; r++) {
            const int c = tid + r * FF_THREADS;
            if (c < c4) {
                float4 acc = res[r];
                for (int j = 0; j < nj; j++) {
                    const float h = s_hb[j];
                    const float4 w = w2s4[(size_t)j * c4 + c];
                    acc.x = fmaf(h, w.x, acc.x);
                    acc.y = fmaf(h, w.y, acc.y);
                    acc.z = fmaf(h, w.z, acc.z);
                    acc.w = fmaf(h, w.w, acc.w);
                }
                red_add_v4(a.xout + 4 * c, acc);
            }
        }
    } else if (tid == 0) {   // let the copies still in flight land before exiting
        mbar_wait_bounded(&bars[0], 0u, nullptr, 0);
        mbar_wait_bounded(&bars[1], 0u, nullptr, 0);
    }
    trace_ev(m, tr, tpos, 2 * a.l + 1, 7);
    if (a.xclear) {
        if (tid == FF_THREADS - 1) s_last = (ticket == gridDim.x - 1);
        __syncthreads();
        if (s_last) {
            for (int i = tid; i < c4; i += FF_THREADS)
                reinterpret_cast<float4 *>(a.xclear)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (tid == 0) m.tickets[1] = 0u;
        }
    }
}

// ---------------------------------------------------------------------------
// k_attn_fused: the attention half of one layer (llama2.c:229-277) as one
// kernel of n_heads clusters of AC CTAs. Cluster h does, for head h:
//   1. rmsnorm(x) and its share of the head's 3*hd q/k/v rows (held in shared
//      memory, bulk-copied before griddepcontrol.wait), computed as row
//      pairs so each warp applies RoPE to its q/k pairs; every CTA sends its
//      results to all CTAs of the cluster through distributed shared memory;
//      cluster barrier;
//   2. attention over its chunk of positions [0, pos] (K/V rows of earlier
//      positions were loaded into registers before the wait), kept as an
//      online-softmax partial (max, sum, unnormalised output); partials are
//      exchanged through distributed shared memory; cluster barrier;
//   3. every CTA merges the AC partials into the head's attention output and
//      multiplies it by its slice of wo (rows [o0, o1), columns of head h),
//      adding the result into the zeroed output with vector reductions; the
//      cluster of head 0 also adds the residual x; CTA 0 writes the new K/V
//      row of `pos` into the cache.
// The only grid-wide dependency is the output sum at L2, so the layer's
// attention costs one kernel boundary instead of three.
// ---------------------------------------------------------------------------
constexpr int AC = 8;                 // CTAs per head (cluster size, portable)
constexpr int AT_THREADS = 256;
constexpr int AT_MAX_HD = 64;
constexpr int AT_ROUND = 64;          // positions per attention round (4 threads each)
constexpr int AT_MAX_OUT = 256;       // wo rows per CTA (dim <= 2048)
constexpr int AT_PAIRS = 2;           // q/k/v row pairs per warp (3*hd/AC <= 32 rows per CTA)

struct AttnArgs {
    const float *xin;  // layer input; null: the embedding row of step->tok (layer 0)
    float *xout;       // zero on entry; receives x + wo . attention
    float *xclear;     // cleared once every CTA has read the input
    int l;
    int stage_floats;  // shared staging region (q/k/v rows, then wo slice + value sums)
    int recv;          // x from this rank's mailbox (a pipeline layer rank's first layer)
};

template <int NV, bool TR>
__global__ void __launch_bounds__(AT_THREADS, 2) k_attn_fused(DecodeModel m, AttnArgs a) {
    // The next kernel (k_ffn) may start at once: its 18.9 MB (110M) weight
    // stream must be resident by its wait. Releasing it later, after this
    // kernel's input read, measured slower (its stream then lands on this
    // kernel's cluster exchange instead).
    pdl_trigger();
    cg::cluster_group cluster = cg::this_cluster();
    extern __shared__ __align__(128) unsigned char smem_raw[];
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem_raw);   // [0] q/k/v rows
    float4 *s_x4 = reinterpret_cast<float4 *>(smem_raw + MV_BAR_BYTES);   // the layer input x
    float *stage = reinterpret_cast<float *>(smem_raw + MV_BAR_BYTES + vec_smem_bytes(m.dim));
    __shared__ __align__(16) float s_qkv[3 * AT_MAX_HD];        // this head's q, k, v (all CTAs' rows)
    __shared__ __align__(16) float s_part[AC][AT_MAX_HD + 4];   // per-CTA o[hd], max, sum
    __shared__ __align__(16) float s_att[AT_MAX_HD];
    __shared__ __align__(16) float s_res[AT_MAX_OUT];
    __shared__ float s_sc[AT_ROUND];
    __shared__ int s_last;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int NW = AT_THREADS / 32;
    const int r = (int)cluster.block_rank();
    const int h = blockIdx.x / AC;
    const int dim = m.dim, hd = m.hd, hd4 = hd >> 2, c4 = dim >> 2, l = a.l;
    const int q0 = 3 * hd * r / AC, q1 = 3 * hd * (r + 1) / AC;   // q/k/v rows of this CTA
    const int o0 = dim * r / AC, o1 = dim * (r + 1) / AC;         // wo rows of this CTA
    const int pos_raw = __ldcg(&m.step->pos) + m.tok_off;
    const bool pos_ok = pos_raw >= 0 && pos_raw < m.seq;
    // out of range: computed at position 0 so that every cluster barrier is
    // still reached, with no K/V write and the error recorded
    const int pos = pos_ok ? pos_raw : 0;
    if (!pos_ok) flag_pos_range(m);
    constexpr bool tr = TR;
    trace_ev(m, tr, pos, 2 * l, 0);
    // the link's message for this position (read before the wait: only the
    // last kernel of a graph moves the count on)
    const unsigned want = a.recv ? __ldcg(&m.step->recvd) + m.tok_off + 1 : 0u;
    // positions of this CTA: [t0, t1) of [0, pos]
    const int ppc = (pos + AC) / AC;
    const int t0 = min(r * ppc, pos + 1), t1 = min(t0 + ppc, pos + 1);
    const size_t head_base = ((size_t)l * m.nkv + h) * m.seq;

    if (tid == 0) {
        mbar_init(&bars[0], 1);
        mbar_init_fence();
    }
    __syncthreads();
    constexpr int pkw = kPolWeights, pkk = kPolKV;
    const uint64_t polw = make_l2_policy(pkw), polk = make_l2_policy(pkk);
    if (tid == 0) {
        const size_t D = dim, K = m.kvd;
        const float *mats[3] = {m.wq + (size_t)l * D * D, m.wk + (size_t)l * K * D, m.wv + (size_t)l * K * D};
        mbar_expect_tx(&bars[0], (unsigned)((q1 - q0) * dim * 4));
        // one bulk copy per row, as in k_ffn (0.9 us/token faster at 110M
        // than one copy per matrix segment)
        for (int sgm = 0; sgm < 3; sgm++) {
            const int lo = max(q0, sgm * hd), hi = min(q1, (sgm + 1) * hd);
            for (int r = lo; r < hi; r++)
                bulk_g2s_pol(stage + (size_t)(r - q0) * dim, mats[sgm] + (size_t)(h * hd + r - sgm * hd) * dim,
                             (unsigned)(dim * 4), &bars[0], pkw, polw);
        }
    }
    if (tid == 32 && t1 - t0 > AT_ROUND) {
        // positions past the first round are read after the wait: warm L2
        const int tp = t0 + AT_ROUND, te = min(t1, pos);
        if (te > tp) {
            prefetch_l2_pol(m.kc + (head_base + tp) * hd, (unsigned)((te - tp) * hd * 4), pkk, polk);
            prefetch_l2_pol(m.vc + (head_base + tp) * hd, (unsigned)((te - tp) * hd * 4), pkk, polk);
        }
    }
    // K/V rows of the first round's earlier positions up to pos - 2: written
    // by earlier tokens, so read before the wait (the row of pos comes from
    // step 2, the row of pos - 1 is read after the wait: a chain of
    // programmatic launches only a few kernels long -- a model or pipeline
    // stage of one or two layers -- can start this block before the previous
    // position's attention block has written it).
    const int js = tid >> 2, sub = tid & 3;
    const int ngrp = AT_THREADS / hd4, d4 = tid % hd4, grp = tid / hd4;
    constexpr int QK = 4, VP = 4;
    float4 kv[QK], vpre[VP];
    {
        const float4 *kb = reinterpret_cast<const float4 *>(m.kc + (head_base + t0) * hd);
        const float4 *vb = reinterpret_cast<const float4 *>(m.vc + (head_base + t0) * hd);
        const int n0 = min(AT_ROUND, t1 - t0);
#pragma unroll
        for (int i = 0; i < QK; i++) {
            const int cc = sub + 4 * i;
            kv[i] = (cc < hd4 && js < n0 && t0 + js < pos - 1) ? ldcg_pol(kb + (size_t)js * hd4 + cc, pkk, polk)
                                                               : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int k = 0; k < VP; k++) {
            const int j = grp + ngrp * k;
            vpre[k] = (grp < ngrp && j < n0 && t0 + j < pos - 1) ? ldcg_pol(vb + (size_t)j * hd4 + d4, pkk, polk)
                                                                 : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
    float4 xr[NV], gr[NV];
    load_gain<NV>(gr, m.rms_att + (size_t)l * dim, c4, lane);
    // RoPE factors of pos for the pair this thread rotates (tid < hd)
    // RoPE factors of pos for the q/k row pairs this warp computes (each warp
    // owns whole pairs, so it rotates them before the exchange)
    float2 rcs[AT_PAIRS];
#pragma unroll
    for (int k = 0; k < AT_PAIRS; k++) {
        const int pr = q0 + 2 * warp + 2 * NW * k;
        rcs[k] = (pr < q1 && pr < 2 * hd) ? __ldg(m.rope + (size_t)pos * (hd / 2) + (pr % hd) / 2)
                                          : make_float2(1.f, 0.f);
    }
    // layer 0 reads the token's embedding row: before the wait when this is
    // the graph's first token, after it otherwise
    const float *xsrc = a.xin ? a.xin : m.emb + (size_t)(m.tok_off == 0 ? __ldcg(&m.step->tok) : 0) * dim;
    if (!a.xin && m.tok_off == 0) stage_vec(s_x4, xsrc, c4);
    // every CTA of the cluster runs before any remote store (no memory
    // ordering needed here, so the relaxed form)
    asm volatile("barrier.cluster.arrive.relaxed.aligned;\n\tbarrier.cluster.wait.aligned;" ::: "memory");
    pdl_wait();
    {   // the row of pos - 1, if in this CTA's first round
        const int jr = pos - 1 - t0;
        if (jr >= 0 && jr < min(AT_ROUND, t1 - t0)) {
            const float4 *kb = reinterpret_cast<const float4 *>(m.kc + (head_base + pos - 1) * hd);
            const float4 *vb = reinterpret_cast<const float4 *>(m.vc + (head_base + pos - 1) * hd);
#pragma unroll
            for (int i = 0; i < QK; i++) {
                const int cc = sub + 4 * i;
                if (cc < hd4 && js == jr) kv[i] = ldcg_pol(kb + cc, pkk, polk);
            }
#pragma unroll
            for (int k = 0; k < VP; k++)
                if (grp < ngrp && grp + ngrp * k == jr) vpre[k] = ldcg_pol(vb + d4, pkk, polk);
        }
    }
    trace_ev(m, tr, pos, 2 * l, 1);
    if (a.recv) {   // pipeline layer rank: x is the previous stage's message
        if (tid == 0) link_poll(m, want, pos);
        __syncthreads();
        stage_vec_cv(s_x4, mailbox_x(m.in_box), c4);
    } else {
        if (!a.xin && m.tok_off != 0) xsrc = m.emb + (size_t)__ldcg(&m.step->tok) * dim;
        if (a.xin || m.tok_off != 0) stage_vec(s_x4, xsrc, c4);
    }
    __syncthreads();
    vec_from_smem<NV>(xr, s_x4, c4, lane);
    if (h == 0)
        for (int i = tid; i < (o1 - o0) / 4; i += AT_THREADS) reinterpret_cast<float4 *>(s_res)[i] = s_x4[o0 / 4 + i];
    rmsnorm_pre<NV>(xr, gr, dim);
    trace_ev(m, tr, pos, 2 * l, 2);

    // 1. q/k/v row pairs, RoPE on the q and k pairs (llama2.c:238-245), then
    //    to every CTA's s_qkv
    bool bad = !mbar_wait_bounded(&bars[0], 0u, m.err, ERR_MBAR_TIMEOUT);
    trace_ev(m, tr, pos, 2 * l, 3);
#pragma unroll
    for (int k = 0; k < AT_PAIRS; k++) {
        const int pr = q0 + 2 * warp + 2 * NW * k;
        if (pr < q1) {
            float v0 = smem_row_dot<NV>(stage + (size_t)(pr - q0) * dim, xr, c4, lane);
            float v1 = smem_row_dot<NV>(stage + (size_t)(pr + 1 - q0) * dim, xr, c4, lane);
            if (pr < 2 * hd) {
                const float cs = rcs[k].x, sn = rcs[k].y;
                const float a0 = v0, a1 = v1;
                v0 = __fsub_rn(__fmul_rn(a0, cs), __fmul_rn(a1, sn));
                v1 = __fadd_rn(__fmul_rn(a0, sn), __fmul_rn(a1, cs));
            }
            if (lane < AC) {
                float *dst = cluster.map_shared_rank(s_qkv, lane);
                dst[pr] = v0;
                dst[pr + 1] = v1;
            }
        }
    }
    trace_ev(m, tr, pos, 2 * l, 8);
    // This CTA's q/k/v values are in every CTA's s_qkv: arrive (release) on
    // the cluster barrier now and wait for it only before reading s_qkv, so
    // the copies below are issued while the barrier completes.
    asm volatile("barrier.cluster.arrive.aligned;" ::: "memory");
    __syncthreads();
    // Every thread of this CTA has consumed the layer input (rmsnorm, the
    // residual copy), so the CTA takes its ticket now; the result is only
    // looked at when the CTA ends, where the last one clears the buffer.
    unsigned ticket = 0u;
    if (tid == AT_THREADS - 1) ticket = atomicAdd(&m.tickets[0], 1u);
    // The staging rows are consumed by this CTA's warps: the wo slice (rows
    // [o0, o1), the hd columns of head h) takes their place, 16 bytes per
    // thread and copy, followed by the K/V rows of the earlier positions past
    // the first round in the free part of the region (after the wo slice and
    // the value sums), so later rounds read shared memory; positions beyond
    // its capacity are read from global memory in their round. (The same
    // copies as bulk copies issued by one warp measured 199 -> 227 us/token:
    // their issue waits behind the FFN block's bulk copies on the SM's copy
    // engine, and the cluster barrier waits for that warp.)
    float *s_o = stage + (size_t)(dim / AC) * hd;   // value sums [ngrp][hd], after the wo slice
    float *kv2 = s_o + (size_t)ngrp * hd;           // K rows [n2][hd], then V rows [n2][hd]
    const int p2 = t0 + AT_ROUND;
    const int kv2_cap = (a.stage_floats - (dim / AC) * hd - ngrp * hd) / (2 * hd);
    const int n2 = max(0, min(min(t1, pos), p2 + kv2_cap) - p2);
    {
        const float *wo_base = m.wo + (size_t)l * dim * dim + (size_t)h * hd;
        for (int f = tid; f < (o1 - o0) * hd4; f += AT_THREADS) {
            const int row = f / hd4, c = f - row * hd4;
            cp_async16_pol(stage + (size_t)row * hd + 4 * c, wo_base + (size_t)(o0 + row) * dim + 4 * c, pkw, polw);
        }
        if (n2 > 0) {
            const float *kb = m.kc + (head_base + p2) * hd, *vb = m.vc + (head_base + p2) * hd;
            for (int f = tid; f < n2 * hd4; f += AT_THREADS) {
                cp_async16_pol(kv2 + 4 * f, kb + 4 * f, pkk, polk);
                cp_async16_pol(kv2 + (size_t)n2 * hd + 4 * f, vb + 4 * f, pkk, polk);
            }
        }
        cp_async_commit();
    }
    trace_ev(m, tr, pos, 2 * l, 9);
    asm volatile("barrier.cluster.wait.aligned;" ::: "memory");   // s_qkv complete
    trace_ev(m, tr, pos, 2 * l, 4);
    // 2. attention over [t0, t1): online softmax in rounds of AT_ROUND
    const float scale = __fdiv_rn(1.0f, pt_sqrtf((float)hd));
    float4 qv[QK];
#pragma unroll
    for (int i = 0; i < QK; i++) {
        const int cc = sub + 4 * i;
        qv[i] = (cc < hd4) ? reinterpret_cast<const float4 *>(s_qkv)[cc] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float m_run = -3.4028235e+38f, l_run = 0.f, o_run = 0.f;   // o_run: element tid of the output (tid < hd)
    for (int rt0 = t0; rt0 < t1; rt0 += AT_ROUND) {
        const int n = min(AT_ROUND, t1 - rt0);
        if (rt0 != t0) {   // later rounds: staged rows from shared memory, the rest from L2 (warmed)
            cp_async_wait_all();
            __syncthreads();
            const float4 *kb = reinterpret_cast<const float4 *>(m.kc + (head_base + rt0) * hd);
            const float4 *vb = reinterpret_cast<const float4 *>(m.vc + (head_base + rt0) * hd);
            const float4 *ks = reinterpret_cast<const float4 *>(kv2);
            const float4 *vs = reinterpret_cast<const float4 *>(kv2 + (size_t)n2 * hd);
#pragma unroll
            for (int i = 0; i < QK; i++) {
                const int cc = sub + 4 * i, p = rt0 + js;
                float4 val = make_float4(0.f, 0.f, 0.f, 0.f);
                if (cc < hd4 && js < n && p != pos)
                    val = (p - p2 < n2) ? ks[(size_t)(p - p2) * hd4 + cc] : ldcg_pol(kb + (size_t)js * hd4 + cc, pkk, polk);
                kv[i] = val;
            }
#pragma unroll
            for (int k = 0; k < VP; k++) {
                const int j = grp + ngrp * k, p = rt0 + j;
                float4 val = make_float4(0.f, 0.f, 0.f, 0.f);
                if (grp < ngrp && j < n && p != pos)
                    val = (p - p2 < n2) ? vs[(size_t)(p - p2) * hd4 + d4] : ldcg_pol(vb + (size_t)j * hd4 + d4, pkk, polk);
                vpre[k] = val;
            }
        }
        // the current position's row is this kernel's own (post-RoPE) k and v
        if (js < n && rt0 + js == pos) {
#pragma unroll
            for (int i = 0; i < QK; i++) {
                const int cc = sub + 4 * i;
                if (cc < hd4) kv[i] = reinterpret_cast<const float4 *>(s_qkv + hd)[cc];
            }
        }
#pragma unroll
        for (int k = 0; k < VP; k++) {
            const int j = grp + ngrp * k;
            if (grp < ngrp && j < n && rt0 + j == pos) vpre[k] = reinterpret_cast<const float4 *>(s_qkv + 2 * hd)[d4];
        }
        {
            float acc = 0.f;
#pragma unroll
            for (int i = 0; i < QK; i++) acc = dot4(kv[i], qv[i], acc);
            acc += __shfl_xor_sync(0xffffffffu, acc, 1);
            acc += __shfl_xor_sync(0xffffffffu, acc, 2);
            if (js < n && sub == 0) s_sc[js] = __fmul_rn(acc, scale);
        }
        __syncthreads();
        // Every warp reduces the round's scores itself (same lanes, same
        // order, so all threads hold identical values): no serial section
        // and no broadcast through shared memory.
        float mx = -3.4028235e+38f;
        for (int j = lane; j < n; j += 32) mx = fmaxf(mx, s_sc[j]);
        mx = warp_max(mx);
        const float m_new = fmaxf(m_run, mx);
        float sum = 0.f;
        for (int j = lane; j < n; j += 32) sum += pt_expf(__fsub_rn(s_sc[j], m_new));
        sum = warp_sum(sum);
        const float alpha = pt_expf(__fsub_rn(m_run, m_new));
        l_run = fmaf(l_run, alpha, sum);
        m_run = m_new;
        if (grp < ngrp) {
            float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int k = 0; k < VP; k++) {
                const int j = grp + ngrp * k;
                if (j < n) {
                    const float e = pt_expf(__fsub_rn(s_sc[j], m_new));
                    o.x = fmaf(e, vpre[k].x, o.x); o.y = fmaf(e, vpre[k].y, o.y);
                    o.z = fmaf(e, vpre[k].z, o.z); o.w = fmaf(e, vpre[k].w, o.w);
                }
            }
            reinterpret_cast<float4 *>(s_o)[grp * hd4 + d4] = o;
        }
        __syncthreads();
        if (tid < hd) {
            float o = 0.f;
            for (int g = 0; g < ngrp; g++) o += s_o[g * hd + tid];
            o_run = fmaf(o_run, alpha, o);
        }
        if (rt0 + AT_ROUND < t1) __syncthreads();   // s_sc and s_o are reused by the next round
    }
    trace_ev(m, tr, pos, 2 * l, 5);
    // partial of this CTA -> slot r of every CTA
    if (tid < hd)
        for (int k = 0; k < AC; k++) cluster.map_shared_rank(&s_part[0][0], k)[r * (AT_MAX_HD + 4) + tid] = o_run;
    if (tid == 0)
        for (int k = 0; k < AC; k++) {
            float *p = cluster.map_shared_rank(&s_part[0][0], k) + r * (AT_MAX_HD + 4);
            p[AT_MAX_HD] = m_run;
            p[AT_MAX_HD + 1] = l_run;
        }
    cluster.sync();
    trace_ev(m, tr, pos, 2 * l, 6);

    // 3. merge the AC partials (every output thread, same order in every
    // CTA), then wo
    if (tid < hd) {
        float M = -3.4028235e+38f;
        for (int k = 0; k < AC; k++) M = fmaxf(M, s_part[k][AT_MAX_HD]);
        float L = 0.f, o = 0.f;
        for (int k = 0; k < AC; k++) {
            const float w = pt_expf(__fsub_rn(s_part[k][AT_MAX_HD], M));
            L = fmaf(w, s_part[k][AT_MAX_HD + 1], L);
            o = fmaf(w, s_part[k][tid], o);
        }
        s_att[tid] = o * __fdiv_rn(1.0f, L);
    }
    trace_ev(m, tr, pos, 2 * l, 10);
    cp_async_wait_all();
    __syncthreads();   // s_att and the wo slice
    trace_ev(m, tr, pos, 2 * l, 11);
    // wo rows in quads: lane 8e + k reduces row 4qd + e over float4 columns
    // k, k + 8, ...; lane 0 gathers the quad and adds it at L2.
    const int e8 = lane >> 3, k8 = lane & 7;
    const float4 *att4 = reinterpret_cast<const float4 *>(s_att);
    for (int qd = warp; qd < (o1 - o0) / 4; qd += NW) {
        const float4 *w4 = reinterpret_cast<const float4 *>(stage + (size_t)(4 * qd + e8) * hd);
        float acc = 0.f;
        for (int c = k8; c < hd4; c += 8) acc = dot4(w4[c], att4[c], acc);
        acc += __shfl_xor_sync(0xffffffffu, acc, 1);
        acc += __shfl_xor_sync(0xffffffffu, acc, 2);
        acc += __shfl_xor_sync(0xffffffffu, acc, 4);
        const float y1 = __shfl_sync(0xffffffffu, acc, 8);
        const float y2 = __shfl_sync(0xffffffffu, acc, 16);
        const float y3 = __shfl_sync(0xffffffffu, acc, 24);
        if (lane == 0) {
            float4 out = make_float4(acc, y1, y2, y3);
            if (h == 0) {
                const float4 rr = reinterpret_cast<const float4 *>(s_res)[qd];
                out.x = __fadd_rn(rr.x, out.x); out.y = __fadd_rn(rr.y, out.y);
                out.z = __fadd_rn(rr.z, out.z); out.w = __fadd_rn(rr.w, out.w);
            }
            red_add_v4(a.xout + o0 + 4 * qd, out);
        }
    }
    // the new K/V row, needed only by later tokens (written after the
    // cluster barriers, whose release would otherwise wait for it)
    if (r == 0 && pos_ok && tid < 2 * hd) {
        const int d = tid % hd;
        float *dst = (tid < hd ? m.kc : m.vc) + (head_base + pos) * hd + d;
        *dst = s_qkv[(tid < hd ? hd : 2 * hd) + d];
    }
    trace_ev(m, tr, pos, 2 * l, 7);
    if (tid == AT_THREADS - 1) s_last = (ticket == gridDim.x - 1);
    __syncthreads();
    if (s_last) {
        for (int i = tid; i < c4; i += AT_THREADS)
            reinterpret_cast<float4 *>(a.xclear)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (tid == 0) m.tickets[0] = 0u;
    }
    if (bad && tid == 0) mbar_wait_bounded(&bars[0], 0u, nullptr, 0);   // let the copy land before exiting
}

// Host-side launchers --------------------------------------------------------

#define PTC_NV_SWITCH(nv, KERNEL_CALL)                                                \
    switch (nv) {                                                                     \
        case 1: { constexpr int NV = 1; KERNEL_CALL; } break;                         \
        case 2: { constexpr int NV = 2; KERNEL_CALL; } break;                         \
        case 3: { constexpr int NV = 3; KERNEL_CALL; } break;                         \
        case 4: { constexpr int NV = 4; KERNEL_CALL; } break;                         \
        case 5: { constexpr int NV = 5; KERNEL_CALL; } break;                         \
        case 6: { constexpr int NV = 6; KERNEL_CALL; } break;                         \
        case 7: { constexpr int NV = 7; KERNEL_CALL; } break;                         \
        case 8: { constexpr int NV = 8; KERNEL_CALL; } break;                         \
        case 9: { constexpr int NV = 9; KERNEL_CALL; } break;                         \
        case 10: { constexpr int NV = 10; KERNEL_CALL; } break;                       \
        case 11: { constexpr int NV = 11; KERNEL_CALL; } break;                       \
        case 12: { constexpr int NV = 12; KERNEL_CALL; } break;                       \
        case 13: { constexpr int NV = 13; KERNEL_CALL; } break;                       \
        case 14: { constexpr int NV = 14; KERNEL_CALL; } break;                       \
        case 15: { constexpr int NV = 15; KERNEL_CALL; } break;                       \
        case 16: { constexpr int NV = 16; KERNEL_CALL; } break;                       \
        default: PTC_FATAL("decode: row width %d floats exceeds 2048", (nv) * 128);   \
    }

static inline int nv_of(int cols) { return (cols / 4 + 31) / 32; }

// Launch with the programmatic-stream-serialization attribute so that
// consecutive decode kernels overlap (prologue of N+1 with tail of N).
// PTC_NO_PDL=1 disables programmatic dependent launch (for A/B timing).
static bool pdl_on() {
    static int on = -1;
    if (on < 0) {
        const char *e = getenv("PTC_NO_PDL");
        on = (e && e[0] == '1') ? 0 : 1;
    }
    return on == 1;
}

template <typename... KArgs, typename... Args>
static void launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                       Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_on() ? 1 : 0;
    PTC_CHECK(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...));
}

// The same, for a kernel launched in clusters of `cluster` CTAs.
template <typename... KArgs, typename... Args>
static void launch_cluster_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, int cluster,
                               cudaStream_t s, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cluster;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_on() ? 2 : 1;
    PTC_CHECK(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...));
}

__global__ void k_embed(DecodeModel m);


template <int NV, int MODE>
static void launch_mv(const DecodeModel &m, MvArgs a, int n_sm, cudaStream_t s) {
    const int stage_bytes = MODE == MV_CLS ? CLS_STAGE_BYTES : MV_STAGE_BYTES;
    const int n_stages = MODE == MV_CLS ? CLS_STAGES : MV_STAGES;
    const int item_bytes = a.slots * a.cols * 4;
    a.per_stage = stage_bytes / item_bytes;
    if (a.per_stage < 1) PTC_FATAL("decode row of %d floats does not fit a staging buffer", a.cols);
    const int grid = a.n_items < n_sm ? a.n_items : n_sm;
    // Only the stages a CTA can fill are reserved, so that the next kernels
    // of the chain fit beside this one on an SM and start their weight
    // streams early.
    const int items_max = (a.n_items + grid - 1) / grid;
    int stages = (items_max + a.per_stage - 1) / a.per_stage;
    if (stages > n_stages) stages = n_stages;
    const size_t smem = (size_t)MV_BAR_BYTES + (MODE == MV_CLS ? 0 : vec_smem_bytes(a.cols)) +
                        (size_t)stages * stage_bytes;
    // Every decode kernel gets the same (maximal) shared-memory carveout, so
    // consecutive kernels co-reside on an SM without reconfiguring L1.
    if constexpr (MODE == MV_CLS) {
        if (m.trace) {
            ensure_kernel_smem((const void *)k_mv<NV, MODE, true>, smem);
            launch_pdl(k_mv<NV, MODE, true>, dim3(grid), dim3(MV_THREADS), smem, s, m, a);
            return;
        }
    }
    ensure_kernel_smem((const void *)k_mv<NV, MODE, false>, smem);
    launch_pdl(k_mv<NV, MODE, false>, dim3(grid), dim3(MV_THREADS), smem, s, m, a);
}

static MvArgs mv_args(int n_items, int cols, int slots, int l) {
    MvArgs a;
    memset(&a, 0, sizeof(a));
    a.n_items = n_items;
    a.cols = cols;
    a.slots = slots;
    a.l = l;
    return a;
}

template <int NV>
static void launch_ffn(const DecodeModel &m, FfnArgs a, int n_sm, cudaStream_t s) {
    const int grid = m.hidden < n_sm ? m.hidden : n_sm;
    const size_t smem = (size_t)MV_BAR_BYTES + vec_smem_bytes(m.dim) + 3 * (size_t)m.ffn_rows * m.dim * 4;
    auto kern = m.trace ? k_ffn<NV, true> : k_ffn<NV, false>;
    ensure_kernel_smem((const void *)kern, smem);
    launch_pdl(kern, dim3(grid), dim3(FF_THREADS), smem, s, m, a);
}

template <int NV>
static void launch_attn_fused(const DecodeModel &m, AttnArgs a, cudaStream_t s) {
    const size_t smem = (size_t)MV_BAR_BYTES + vec_smem_bytes(m.dim) + (size_t)m.attn_stage * 4;
    auto kern = m.trace ? k_attn_fused<NV, true> : k_attn_fused<NV, false>;
    ensure_kernel_smem((const void *)kern, smem);
    a.stage_floats = m.attn_stage;
    launch_cluster_pdl(kern, dim3(m.nh * AC), dim3(AT_THREADS), smem, AC, s, m, a);
}

// Staging floats of k_attn_fused for this model, or 0 when the fused
// attention does not apply: one K/V head per query head, head_dim <= 64 and
// a multiple of 4, dim a multiple of 4 * AC (whole wo row quads per CTA).
int decode_attn_stage(int dim, int nh, int nkv, int seq) {
    if (nh != nkv || dim % nh) return 0;
    const int hd = dim / nh;
    if (hd > AT_MAX_HD || hd % 4 || dim % (4 * AC) || dim / AC > AT_MAX_OUT || dim > 2048) return 0;
    // whole row pairs per CTA (RoPE pairs stay in one warp), at most
    // AT_PAIRS pairs per warp
    if ((3 * hd) % (2 * AC) || 3 * hd / AC > 2 * AT_PAIRS * (AT_THREADS / 32)) return 0;
    (void)seq;   // positions are processed in rounds: no limit from seq_len
    const int qkv_rows = (3 * hd + AC - 1) / AC;
    const int ngrp = AT_THREADS / (hd / 4);
    const int stage_a = qkv_rows * dim;                  // q/k/v rows
    const int stage_b = (dim / AC) * hd + ngrp * hd;      // wo slice + value sums
    const int stage = stage_a > stage_b ? stage_a : stage_b;
    if ((size_t)stage * 4 > 160 * 1024) return 0;
    return stage;
}

// Hidden units per k_ffn CTA for this model and grid, or 0 when the fused
// FFN does not fit (rows in shared memory, output columns per thread).
int decode_ffn_rows(int dim, int hidden, int n_sm) {
    const int grid = hidden < n_sm ? hidden : n_sm;
    const int rows = (hidden + grid - 1) / grid;
    if (rows > FF_MAX_ROWS || dim / 4 > 2 * FF_THREADS) return 0;
    if (3 * (size_t)rows * dim * 4 + vec_smem_bytes(dim) > (size_t)FF_MAX_SMEM) return 0;
    return rows;
}

// One layer with explicit residual-stream buffers: the layer reads x_in
// (rmsnorm input and attention residual) and leaves its output in x_out.
// Fused FFN: wo writes xm = x_in + wo.att and clears x_in behind it, k_ffn
// accumulates xm + w2.hb into x_out, which is zero on entry.
static void launch_layer(const DecodeModel &m, int l, bool from_embedding, float *x_in, float *x_out, int n_sm,
                         cudaStream_t s, bool recv = false) {
    const int nvd = nv_of(m.dim), nvh = nv_of(m.hidden);
    if (m.fused_attn) {
        // two kernels: attention block -> xm, FFN block -> x_out; each clears
        // the input it consumed once all its CTAs have read it
        AttnArgs at;
        memset(&at, 0, sizeof(at));
        at.xin = from_embedding ? nullptr : x_in;
        at.xout = m.xm;
        at.xclear = x_in;
        at.l = l;
        at.recv = recv ? 1 : 0;
        PTC_NV_SWITCH(nvd, (launch_attn_fused<NV>(m, at, s)));
        FfnArgs f;
        f.xin = m.xm;
        f.xout = x_out;
        f.xclear = m.xm;
        f.l = l;
        PTC_NV_SWITCH(nvd, (launch_ffn<NV>(m, f, n_sm, s)));
        return;
    }
    if (recv) PTC_FATAL("pipeline links need the fused attention block (PTC_DECODE_FUSED unset)");
    MvArgs a = mv_args((m.dim + 2 * m.kvd) / 2, m.dim, 2, l);
    a.from_embedding = from_embedding ? 1 : 0;
    a.in = x_in;
    PTC_NV_SWITCH(nvd, (launch_mv<NV, MV_QKV>(m, a, n_sm, s)));
    ensure_kernel_smem((const void *)k_attn, 0);
    ensure_kernel_smem((const void *)k_embed, 0);
    launch_pdl(k_attn, dim3(m.nh, m.n_chunks), dim3(ATT_THREADS), 0, s, m, l);
    a = mv_args(m.dim, m.dim, 1, l);
    a.W = m.wo + (size_t)l * m.dim * m.dim;
    a.in = m.att;
    if (m.fused_ffn) {
        a.res_in = x_in;
        a.res_out = m.xm;
        a.zero_res_in = 1;
        PTC_NV_SWITCH(nvd, (launch_mv<NV, MV_RESID>(m, a, n_sm, s)));
        FfnArgs f;
        f.xin = m.xm;
        f.xout = x_out;
        f.xclear = nullptr;   // wo overwrites xm whole
        f.l = l;
        PTC_NV_SWITCH(nvd, (launch_ffn<NV>(m, f, n_sm, s)));
        return;
    }
    // unfused: x_in == x_out, updated in place
    a.res_in = x_in;
    a.res_out = x_in;
    PTC_NV_SWITCH(nvd, (launch_mv<NV, MV_RESID>(m, a, n_sm, s)));
    a = mv_args(m.hidden, m.dim, 2, l);
    a.in = x_in;
    PTC_NV_SWITCH(nvd, (launch_mv<NV, MV_FFN13>(m, a, n_sm, s)));
    a = mv_args(m.dim, m.hidden, 1, l);
    a.W = m.w2 + (size_t)l * m.dim * m.hidden;
    a.in = m.hb;
    a.res_in = x_in;
    a.res_out = x_in;
    PTC_NV_SWITCH(nvh, (launch_mv<NV, MV_RESID>(m, a, n_sm, s)));
}

// One block of layer l (kind 0: attention, 1: FFN) on the buffers a full
// [0, L) decode uses -- for timing single kernels.
void launch_block(const DecodeModel &m, int kind, int l, int n_sm, cudaStream_t s) {
    float *x_in = m.x, *x_out = m.x;
    if (m.fused_ffn) {
        x_in = (l == 0) ? m.x : m.xo + (size_t)(l - 1) * m.dim;
        x_out = (l == m.L - 1) ? m.x : m.xo + (size_t)l * m.dim;
    }
    const int nvd = nv_of(m.dim);
    if (kind == 0 && m.fused_attn) {
        AttnArgs at;
        memset(&at, 0, sizeof(at));
        at.xin = x_in;
        at.xout = m.xm;
        at.xclear = x_in;
        at.l = l;
        PTC_NV_SWITCH(nvd, (launch_attn_fused<NV>(m, at, s)));
    } else if (kind == 1 && m.fused_ffn) {
        FfnArgs f;
        f.xin = m.xm;
        f.xout = x_out;
        f.xclear = m.fused_attn ? m.xm : nullptr;
        f.l = l;
        PTC_NV_SWITCH(nvd, (launch_ffn<NV>(m, f, n_sm, s)));
    } else {
        launch_layer(m, l, false, x_in, x_out, n_sm, s);   // unfused layouts: the whole layer
    }
}

// Layers [l0, l1): the range reads m.x and leaves its output in m.x. With
// the fused FFN, layer l < l1-1 hands over through xo[l] (zeroed again by
// the next layer's wo once read); the last layer accumulates into m.x,
// which the first layer's wo cleared.
void launch_layers(const DecodeModel &m, int l0, int l1, bool from_embedding, int n_sm, cudaStream_t s) {
    for (int l = l0; l < l1; l++) {
        float *x_in = m.x, *x_out = m.x;
        if (m.fused_ffn) {
            x_in = (l == l0) ? m.x : m.xo + (size_t)(l - 1) * m.dim;
            x_out = (l == l1 - 1) ? m.x : m.xo + (size_t)l * m.dim;
        }
        launch_layer(m, l, from_embedding && l == 0, x_in, x_out, n_sm, s, m.link_mode && m.link_recv && l == l0);
    }
}

void launch_head(const DecodeModel &m, int n_sm, cudaStream_t s, int *host_next) {
    const bool vp = m.link_mode && m.vp_rows > 0;
    MvArgs a = mv_args(vp ? m.vp_rows : m.V, m.dim, 1, 0);
    a.W = vp ? m.vp_W : m.wcls;
    a.row0 = vp ? m.vp_row0 : 0;
    a.host_next = host_next;
    a.recv = m.link_mode && !vp ? 1 : 0;
    a.send_next = m.link_mode && !vp ? 1 : 0;
    a.vp = vp ? 1 : 0;
    a.vp_cls = vp && !m.vp_x_local ? 1 : 0;
    a.adv_recvd = vp && m.L > 0 && m.link_recv ? 1 : 0;
    PTC_NV_SWITCH(nv_of(m.dim), (launch_mv<NV, MV_CLS>(m, a, n_sm, s)));
}

// x = token_embedding[tok] (llama2.c:220-222) for a decoder whose layer 0
// does not fold the lookup in (the pipeline's embed+head rank).
__global__ void k_embed(DecodeModel m) {
    pdl_trigger();
    pdl_wait();
    const int tok = __ldcg(&m.step->tok);
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < m.dim; i += gridDim.x * blockDim.x)
        m.x[i] = __ldg(m.emb + (size_t)tok * m.dim + i);
}

void launch_embed(const DecodeModel &m, cudaStream_t s) {
    launch_pdl(k_embed, dim3((m.dim + 255) / 256), dim3(256), 0, s, m);
}

// dst[c][r] = src[r][c] for a rows x cols matrix, through a padded 32x32 tile.
__global__ void k_transpose(float *dst, const float *src, int rows, int cols) {
    __shared__ float tile[32][33];
    const int bx = blockIdx.x * 32, by = blockIdx.y * 32;
    for (int j = threadIdx.y; j < 32; j += blockDim.y) {
        const int r = by + j, c = bx + threadIdx.x;
        if (r < rows && c < cols) tile[j][threadIdx.x] = src[(size_t)r * cols + c];
    }
    __syncthreads();
    for (int j = threadIdx.y; j < 32; j += blockDim.y) {
        const int c = bx + j, r = by + threadIdx.x;
        if (c < cols && r < rows) dst[(size_t)c * rows + r] = tile[threadIdx.x][j];
    }
}

// w2t[l] = w2[l]^T for each layer ([dim, hidden] -> [hidden, dim]): the FFN
// block reads the w2 column of each of its hidden units as one contiguous row.
void transpose_w2(const DecodeModel &m, float *w2t, cudaStream_t s) {
    for (int l = 0; l < m.L; l++)
        k_transpose<<<dim3((m.hidden + 31) / 32, (m.dim + 31) / 32), dim3(32, 8), 0, s>>>(
            w2t + (size_t)l * m.hidden * m.dim, m.w2 + (size_t)l * m.dim * m.hidden, m.dim, m.hidden);
    PTC_CHECK(cudaGetLastError());
}

// RoPE factors (cos, sin) of every (position, pair) with pitorch's angle and
// trigonometry (pt_ops.c:33-49), computed once per decoder.
__global__ void k_rope_table(float2 *t, int seq, int hd) {
    const int half = hd / 2;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < seq * half; i += gridDim.x * blockDim.x) {
        const int p = i / half, j = 2 * (i % half);
        const float th = rope_theta(j, hd, p);
        t[i] = make_float2(pt_cosf(th), pt_sinf(th));
    }
}

void build_rope_table(float2 *t, int seq, int hd, cudaStream_t s) {
    const int n = seq * (hd / 2);
    k_rope_table<<<(n + 255) / 256, 256, 0, s>>>(t, seq, hd);
    PTC_CHECK(cudaGetLastError());
}

int decode_attn_limits_ok(int hd, int chunk, int n_chunks) {
    // scores: 4 threads per position, <= 4 float4 each (hd <= 64); values:
    // ATT_THREADS / (hd/4) position groups, <= 4 positions per thread
    return hd <= 64 && hd % 4 == 0 && chunk * 4 == ATT_THREADS && n_chunks <= ATT_MAX_CHUNKS &&
           chunk <= 4 * (ATT_THREADS / (hd / 4)) && n_chunks <= ATT_MERGE_PER_THREAD * (ATT_THREADS / (hd / 4));
}

}  // namespace ptc
