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

#include <utility>

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
__device__ __forceinline__ void store_vec(float *dst, const float4 (&x)[NV], int c4, int lane) {
    float4 *d4 = reinterpret_cast<float4 *>(dst);
#pragma unroll
    for (int v = 0; v < NV; v++) {
        int c = lane + 32 * v;
        if (c < c4) d4[c] = x[v];
    }
}

__device__ __forceinline__ const float *qkv_row(const DecodeModel &m, int l, int r) {
    size_t D = m.dim, K = m.kvd;
    if (r < m.dim) return m.wq + (size_t)l * D * D + (size_t)r * D;
    r -= m.dim;
    if (r < m.kvd) return m.wk + (size_t)l * K * D + (size_t)r * D;
    r -= m.kvd;
    return m.wv + (size_t)l * K * D + (size_t)r * D;
}

// ---------------------------------------------------------------------------
// k_qkv: one warp per row pair (2j, 2j+1) of [wq; wk; wv]. Pairs never
// straddle q/k/v (dim and kv_dim are even), so RoPE (pt_ops.c:33-49) is
// applied in the epilogue and k/v go straight into the cache slot of pos.
// Layer 0 reads its input from the token's embedding row and publishes it
// as the residual stream x (llama2.c:220-222).
// ---------------------------------------------------------------------------
template <int NV>
__global__ void __launch_bounds__(256) k_qkv(DecodeModel m, int l, int from_embedding) {
    pdl_trigger();
    const int lane = threadIdx.x & 31;
    const int pair = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int c4 = m.dim >> 2;
    const int r0 = 2 * pair;
    const bool active = r0 < m.dim + 2 * m.kvd;
    float4 w0[NV], w1[NV];
    if (active) {
        load_row<NV>(w0, qkv_row(m, l, r0), c4, lane);
        load_row<NV>(w1, qkv_row(m, l, r0 + 1), c4, lane);
    }
    pdl_wait();
    if (!active) return;
    const int pos = __ldcg(&m.step->pos);
    if (pos < 0 || pos >= m.seq) return;  // stepped past the cache: no writes
    float4 xr[NV];
    if (from_embedding) {
        const int tok = __ldcg(&m.step->tok);
        load_act<NV>(xr, m.emb + (size_t)tok * m.dim, c4, lane);
        if (pair == 0) store_vec<NV>(m.x, xr, c4, lane);
    } else {
        load_act<NV>(xr, m.x, c4, lane);
    }
    rmsnorm_regs<NV>(xr, m.rms_att + (size_t)l * m.dim, m.dim, lane);
    const float a0 = row_dot<NV>(w0, xr);
    const float a1 = row_dot<NV>(w1, xr);
    if (lane != 0) return;
    const int hd = m.hd;
    if (r0 < m.dim + m.kvd) {
        const bool is_q = r0 < m.dim;
        const int i = is_q ? r0 : r0 - m.dim;
        const float th = rope_theta(i, hd, pos);
        const float c = pt_cosf(th), s = pt_sinf(th);
        const float o0 = __fsub_rn(__fmul_rn(a0, c), __fmul_rn(a1, s));
        const float o1 = __fadd_rn(__fmul_rn(a0, s), __fmul_rn(a1, c));
        if (is_q) {
            m.q[i] = o0;
            m.q[i + 1] = o1;
        } else {
            float *dst = m.kc + (((size_t)l * m.nkv + i / hd) * m.seq + pos) * hd + (i % hd);
            dst[0] = o0;
            dst[1] = o1;
        }
    } else {
        const int i = r0 - m.dim - m.kvd;
        float *dst = m.vc + (((size_t)l * m.nkv + i / hd) * m.seq + pos) * hd + (i % hd);
        dst[0] = a0;
        dst[1] = a1;
    }
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
constexpr int ATT_MAX_HD = 256;
constexpr int ATT_MAX_CHUNKS = 256;

__global__ void __launch_bounds__(ATT_THREADS) k_attn(DecodeModel m, int l) {
    pdl_trigger();
    __shared__ __align__(16) float s_q[ATT_MAX_HD];
    __shared__ float s_p[ATT_MAX_CHUNKS];
    __shared__ __align__(16) float s_o[ATT_THREADS * 4];
    __shared__ float s_stat[2];
    __shared__ int s_last;

    const int h = blockIdx.x, c = blockIdx.y;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int hd = m.hd, hd4 = hd >> 2, CH = m.att_chunk;
    const int kvh = h / (m.nh / m.nkv);
    const int ngrp = ATT_THREADS / hd4;      // position groups for the value pass
    const int d4 = tid % hd4, grp = tid / hd4;
    pdl_wait();
    const int pos = min(__ldcg(&m.step->pos), m.seq - 1);
    const int t0 = c * CH;
    const size_t head_base = ((size_t)l * m.nkv + kvh) * m.seq;
    const float scale = __fdiv_rn(1.0f, pt_sqrtf((float)hd));
    float *part = m.att_part + ((size_t)h * m.n_chunks + c) * (hd + 2);

    if (t0 <= pos) {
        const int n = min(CH, pos + 1 - t0);
        for (int d = tid; d < hd; d += ATT_THREADS) s_q[d] = __ldcg(m.q + h * hd + d);
        __syncthreads();
        {   // scores: 4 threads per position, float4 loads
            const int j = tid >> 2, sub = tid & 3;
            float acc = 0.f;
            if (j < n) {
                const float4 *kr = reinterpret_cast<const float4 *>(m.kc + (head_base + t0 + j) * hd);
                const float4 *q4 = reinterpret_cast<const float4 *>(s_q);
#pragma unroll 16
                for (int k = sub; k < hd4; k += 4) acc = dot4(__ldcg(kr + k), q4[k], acc);
            }
            acc += __shfl_xor_sync(0xffffffffu, acc, 1);
            acc += __shfl_xor_sync(0xffffffffu, acc, 2);
            if (j < n && sub == 0) s_p[j] = __fmul_rn(acc, scale);
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
        {   // values: thread (float4 column d4, position group grp)
            float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
            if (grp < ngrp) {
                const float4 *vb = reinterpret_cast<const float4 *>(m.vc + (head_base + t0) * hd);
#pragma unroll 4
                for (int j = grp; j < n; j += ngrp) {
                    const float4 v = __ldcg(vb + (size_t)j * hd4 + d4);
                    const float e = s_p[j];
                    o.x = fmaf(e, v.x, o.x); o.y = fmaf(e, v.y, o.y);
                    o.z = fmaf(e, v.z, o.z); o.w = fmaf(e, v.w, o.w);
                }
                reinterpret_cast<float4 *>(s_o)[grp * hd4 + d4] = o;
            }
        }
        __syncthreads();
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
        s_last = (ticket == gridDim.y - 1);
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    // Merge the nc chunk partials of this head.
    const int nc = pos / CH + 1;
    const float *hp = m.att_part + (size_t)h * m.n_chunks * (hd + 2);
    for (int k = tid; k < nc; k += ATT_THREADS) s_p[k] = __ldcg(hp + (size_t)k * (hd + 2) + hd);
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
        for (int k = 0; k < nc; k++) L = fmaf(s_p[k], __ldcg(hp + (size_t)k * (hd + 2) + hd + 1), L);
        s_stat[1] = __fdiv_rn(1.0f, L);
    }
    {
        float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
        if (grp < ngrp) {
            for (int k = grp; k < nc; k += ngrp) {
                const float *pk = hp + (size_t)k * (hd + 2) + 4 * d4;
                const float w = s_p[k];
                o.x = fmaf(w, __ldcg(pk + 0), o.x); o.y = fmaf(w, __ldcg(pk + 1), o.y);
                o.z = fmaf(w, __ldcg(pk + 2), o.z); o.w = fmaf(w, __ldcg(pk + 3), o.w);
            }
            reinterpret_cast<float4 *>(s_o)[grp * hd4 + d4] = o;
        }
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
// k_resid: x[r] += W[r] . in, one warp per row (wo with in = att, w2 with
// in = hb); the residual add of llama2.c:277 / :287.
// ---------------------------------------------------------------------------
template <int NV>
__global__ void __launch_bounds__(128) k_resid(DecodeModel m, const float *W, const float *in,
                                               int rows, int cols) {
    pdl_trigger();
    const int lane = threadIdx.x & 31;
    const int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int c4 = cols >> 2;
    const bool active = r < rows;
    float4 w[NV];
    if (active) load_row<NV>(w, W + (size_t)r * cols, c4, lane);
    pdl_wait();
    if (!active) return;
    float4 xr[NV];
    load_act<NV>(xr, in, c4, lane);
    const float a = row_dot<NV>(w, xr);
    if (lane == 0) m.x[r] = __fadd_rn(__ldcg(m.x + r), a);
}

// ---------------------------------------------------------------------------
// k_ffn13: one warp per hidden unit i: rmsnorm(x) . w1[i] and . w3[i], then
// hb[i] = silu(h1) * h3 (llama2.c:280-285).
// ---------------------------------------------------------------------------
template <int NV>
__global__ void __launch_bounds__(256) k_ffn13(DecodeModel m, int l) {
    pdl_trigger();
    const int lane = threadIdx.x & 31;
    const int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int c4 = m.dim >> 2;
    const bool active = i < m.hidden;
    float4 wa[NV], wb[NV];
    if (active) {
        const size_t off = (size_t)l * m.hidden * m.dim + (size_t)i * m.dim;
        load_row<NV>(wa, m.w1 + off, c4, lane);
        load_row<NV>(wb, m.w3 + off, c4, lane);
    }
    pdl_wait();
    if (!active) return;
    float4 xr[NV];
    load_act<NV>(xr, m.x, c4, lane);
    rmsnorm_regs<NV>(xr, m.rms_ffn + (size_t)l * m.dim, m.dim, lane);
    const float h1 = row_dot<NV>(wa, xr);
    const float h3 = row_dot<NV>(wb, xr);
    if (lane == 0) m.hb[i] = silu_mul(h1, h3);
}

// ---------------------------------------------------------------------------
// k_cls: final rmsnorm + logits = wcls . x over the vocab rows, with the
// greedy argmax folded in (pitorch/pt.c:267-271). Warps stride over row
// pairs; each CTA publishes its best (value, index) key with one 64-bit
// atomicMax; the last CTA to finish records the token and, in device-loop
// mode, advances the position (teacher-forcing prompt tokens as the
// reference's decode loops do, pitorch/text/pt_text.c:343-347).
// ---------------------------------------------------------------------------
template <int NV>
__global__ void __launch_bounds__(256) k_cls(DecodeModel m) {
    pdl_trigger();
    __shared__ unsigned long long s_best[8];
    __shared__ int s_last;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int nw = (gridDim.x * blockDim.x) >> 5;
    const int c4 = m.dim >> 2;
    const int V = m.V;
    float4 w0[NV], w1[NV];
    int r = 2 * gw;
    if (r < V) {
        load_row<NV>(w0, m.wcls + (size_t)r * m.dim, c4, lane);
        if (r + 1 < V) load_row<NV>(w1, m.wcls + (size_t)(r + 1) * m.dim, c4, lane);
    }
    pdl_wait();
    float4 xr[NV];
    load_act<NV>(xr, m.x, c4, lane);
    rmsnorm_regs<NV>(xr, m.rms_final, m.dim, lane);
    if (gw == 0) store_vec<NV>(m.xn, xr, c4, lane);

    unsigned long long best = 0ull;
    while (r < V) {
        const float a0 = row_dot<NV>(w0, xr);
        const float a1 = (r + 1 < V) ? row_dot<NV>(w1, xr) : 0.f;
        if (lane == 0) {
            m.logits[r] = a0;
            unsigned long long k0 = argmax_key(a0, r);
            if (k0 > best) best = k0;
            if (r + 1 < V) {
                m.logits[r + 1] = a1;
                unsigned long long k1 = argmax_key(a1, r + 1);
                if (k1 > best) best = k1;
            }
        }
        r += 2 * nw;
        if (r < V) {
            load_row<NV>(w0, m.wcls + (size_t)r * m.dim, c4, lane);
            if (r + 1 < V) load_row<NV>(w1, m.wcls + (size_t)(r + 1) * m.dim, c4, lane);
        }
    }
    if (lane == 0) s_best[warp] = best;
    __syncthreads();
    StepState *st = m.step;
    if (threadIdx.x == 0) {
        unsigned long long b = 0ull;
        for (int w = 0; w < (int)(blockDim.x >> 5); w++) b = (s_best[w] > b) ? s_best[w] : b;
        if (b) atomicMax(&st->amax, b);
        __threadfence();
        unsigned ticket = atomicAdd(&st->done, 1u);
        s_last = (ticket == gridDim.x - 1);
    }
    __syncthreads();
    if (!s_last || threadIdx.x != 0) return;
    __threadfence();
    const unsigned long long k = atomicAdd(&st->amax, 0ull);
    const int next = argmax_key_index(k);
    st->next = next;
    st->amax = 0ull;
    st->done = 0u;
    if (st->mode == 1 && st->pos < m.seq) {
        const int p = st->pos;
        int t = next;
        if (p + 1 < st->n_prompt) t = st->tokens[p + 1];
        else st->tokens[p + 1] = next;
        st->tok = t;
        st->pos = p + 1;
    }
    __threadfence();
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
template <typename... KArgs, typename... Args>
static void launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, cudaStream_t s,
                       Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = 0;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    PTC_CHECK(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...));
}

void launch_layer(const DecodeModel &m, int l, bool from_embedding, cudaStream_t s) {
    const int nvd = nv_of(m.dim), nvh = nv_of(m.hidden);
    const int pairs = (m.dim + 2 * m.kvd) / 2;
    PTC_NV_SWITCH(nvd, launch_pdl(k_qkv<NV>, dim3((pairs + 7) / 8), dim3(256), s, m, l,
                                  from_embedding ? 1 : 0));
    launch_pdl(k_attn, dim3(m.nh, m.n_chunks), dim3(ATT_THREADS), s, m, l);
    const float *wo = m.wo + (size_t)l * m.dim * m.dim;
    PTC_NV_SWITCH(nvd, launch_pdl(k_resid<NV>, dim3((m.dim + 3) / 4), dim3(128), s, m, wo,
                                  (const float *)m.att, m.dim, m.dim));
    PTC_NV_SWITCH(nvd, launch_pdl(k_ffn13<NV>, dim3((m.hidden + 7) / 8), dim3(256), s, m, l));
    const float *w2 = m.w2 + (size_t)l * m.dim * m.hidden;
    PTC_NV_SWITCH(nvh, launch_pdl(k_resid<NV>, dim3((m.dim + 3) / 4), dim3(128), s, m, w2,
                                  (const float *)m.hb, m.dim, m.hidden));
}

void launch_head(const DecodeModel &m, int n_sm, cudaStream_t s) {
    const int nvd = nv_of(m.dim);
    int blocks = (m.V / 2 + 7) / 8;
    if (blocks > 2 * n_sm) blocks = 2 * n_sm;
    PTC_NV_SWITCH(nvd, launch_pdl(k_cls<NV>, dim3(blocks), dim3(256), s, m));
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
    launch_pdl(k_embed, dim3((m.dim + 255) / 256), dim3(256), s, m);
}

int decode_attn_limits_ok(int hd, int chunk, int n_chunks) {
    return hd <= ATT_MAX_HD && hd % 4 == 0 && chunk * 4 == ATT_THREADS && n_chunks <= ATT_MAX_CHUNKS;
}

}  // namespace ptc
