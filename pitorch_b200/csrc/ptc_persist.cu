// ptc_persist.cu -- the decode step as ONE persistent kernel.
//
// A chain of ~61 dependent kernels per token costs ~5 us per kernel on B200
// (launch, ramp and drain dominate the 0.3-12 MB each one moves), so the
// token is instead run by a single cooperative kernel with one CTA per SM
// and grid-wide barriers between the data-dependent phases of
// pitorch/model/llama2.c:224-303:
//
//   per layer l:
//     QKV   rmsnorm(x) . [wq;wk;wv] + RoPE, k/v into the KV cache  | barrier
//     ATT   attention partials over (head, position chunk) items   | barrier
//     WO    merge the partials, x1 = x0 = x0 + wo . att             | barrier
//     FFN   rmsnorm(x1) . w1/w3 -> silu*gate for this CTA's hidden
//           block, then x0 += w2[:, block] . hb[block] (split over
//           hidden blocks, atomics into x0, which already holds x1) | barrier
//   head:
//     CLS   rmsnorm(x0) . wcls + argmax                             | barrier
//
// Weights never depend on activations, so a producer warp in each CTA
// streams the CTA's weight slices for every phase, in phase order, through a
// ring of shared-memory stages with bulk (TMA) copies, running ahead across
// barriers as far as the ring allows; the 15 consumer warps only wait for a
// stage to be full. w2 is read through a transposed device copy so a CTA's
// hidden block is contiguous. In device-loop mode one launch decodes many
// positions: the argmax feeds the next position's embedding lookup without
// leaving the GPU (teacher-forcing prompt tokens as pitorch/text/pt_text.c
// :343-347 does).
//
// Every wait (grid barrier, stage full/empty) is bounded; on expiry the
// kernel records an error code and returns.
#include <string.h>

#include "../../include/ptc.h"
#include "ptc_common.cuh"
#include "ptc_decode.cuh"
#include "ptc_internal.h"
#include "ptc_persist.h"

namespace ptc {

constexpr int PS_THREADS = 512;
constexpr int PS_WARPS = PS_THREADS / 32;
constexpr int PS_CONS_WARPS = PS_WARPS - 1;   // warp PS_WARPS-1 is the producer
constexpr int PS_CONS_THREADS = PS_CONS_WARPS * 32;
constexpr int PS_ATT_THREADS = 256;           // warps 0..7 work attention items
constexpr int ERR_GRID_BARRIER = 2;
constexpr int ERR_STAGE_EMPTY = 3;
constexpr int ERR_STAGE_FULL = 4;
constexpr long WAIT_LIMIT = 1L << 24;

// Named barriers: 1 = all consumer warps, 2 = attention workers.
__device__ __forceinline__ void cons_sync() { asm volatile("bar.sync 1, %0;" ::"r"(PS_CONS_THREADS) : "memory"); }
__device__ __forceinline__ void att_sync() { asm volatile("bar.sync 2, %0;" ::"r"(PS_ATT_THREADS) : "memory"); }

__device__ __forceinline__ unsigned ld_acquire(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ bool err_set(const PersistArgs &a) { return *((volatile int *)a.m.err) != 0; }

// Grid barrier among the consumer warps of all CTAs (monotonic counter
// reset to 0 before each launch; the k-th barrier waits for k*G arrivals).
__device__ __forceinline__ unsigned long long globaltimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ bool grid_barrier(const PersistArgs &a, unsigned &epoch, int *s_abort) {
    cons_sync();
    const bool tr = a.trace && blockIdx.x == 0 && threadIdx.x == 0 && (int)(2 * epoch + 1) < a.trace_cap;
    if (tr) a.trace[2 * epoch] = globaltimer();
    if (threadIdx.x == 0) {
        __threadfence();
        asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(a.bar), "r"(1u) : "memory");
        const unsigned target = (epoch + 1) * gridDim.x;
        long it = 0;
        while (ld_acquire(a.bar) < target) {
            if (++it > WAIT_LIMIT || ((it & 1023) == 0 && err_set(a))) {
                atomicExch(a.m.err, ERR_GRID_BARRIER);
                *s_abort = 1;
                break;
            }
        }
    }
    if (tr) a.trace[2 * epoch + 1] = globaltimer();
    epoch++;
    cons_sync();
    return *((volatile int *)s_abort) == 0;
}

// ---- the weight schedule shared by producer and consumers ----------------

enum PsPhase { PH_QKV = 0, PH_WO = 1, PH_FFN13 = 2, PH_W2T = 3, PH_CLS = 4 };

struct Block {
    int it0, it1;  // this CTA's items
    int ps;        // items per stage
    int cols;      // floats per row
    int slots;     // rows per item
};

__device__ __forceinline__ Block phase_block(const PersistArgs &a, int ph) {
    const DecodeModel &m = a.m;
    int n = 0, cols = m.dim, slots = 1;
    switch (ph) {
        case PH_QKV: n = (m.dim + 2 * m.kvd) / 2; slots = 2; break;
        case PH_WO: n = m.dim; break;
        case PH_FFN13: n = m.hidden; slots = 2; break;
        case PH_W2T: n = m.hidden; break;
        default: n = m.V; break;
    }
    Block b;
    b.it0 = (int)((long)n * blockIdx.x / gridDim.x);
    b.it1 = (int)((long)n * (blockIdx.x + 1) / gridDim.x);
    b.cols = cols;
    b.slots = slots;
    b.ps = MV_STAGE_BYTES / (slots * cols * 4);
    return b;
}

__device__ __forceinline__ int n_chunks(const Block &b) { return (b.it1 - b.it0 + b.ps - 1) / b.ps; }

// Issue the bulk copies of chunk k of phase `ph` (layer l) into `stage`.
__device__ __forceinline__ void issue_chunk(const PersistArgs &a, int ph, int l, const Block &b, int k, float *stage,
                                            uint64_t *full) {
    const DecodeModel &m = a.m;
    const int c0 = b.it0 + k * b.ps, c1 = min(b.it1, c0 + b.ps);
    const int n = c1 - c0;
    const size_t rb = (size_t)b.cols * 4;
    if (ph == PH_QKV) {
        const size_t D = m.dim, K = m.kvd;
        const float *base[3] = {m.wq + (size_t)l * D * D, m.wk + (size_t)l * K * D, m.wv + (size_t)l * K * D};
        const int edge[4] = {0, m.dim, m.dim + m.kvd, m.dim + 2 * m.kvd};
        mbar_expect_tx(full, (unsigned)(2 * n * rb));
        const int r0 = 2 * c0, r1 = 2 * c1;
        for (int s = 0; s < 3; s++) {
            const int lo = max(r0, edge[s]), hi = min(r1, edge[s + 1]);
            if (lo < hi)
                bulk_g2s(stage + (size_t)(lo - r0) * b.cols, base[s] + (size_t)(lo - edge[s]) * b.cols,
                         (unsigned)((hi - lo) * rb), full);
        }
    } else if (ph == PH_FFN13) {
        const size_t off = (size_t)l * m.hidden * m.dim + (size_t)c0 * m.dim;
        mbar_expect_tx(full, (unsigned)(2 * n * rb));
        bulk_g2s(stage, m.w1 + off, (unsigned)(n * rb), full);
        bulk_g2s(stage + (size_t)b.ps * b.cols, m.w3 + off, (unsigned)(n * rb), full);
    } else {
        const float *W = (ph == PH_WO)    ? m.wo + (size_t)l * m.dim * m.dim
                         : (ph == PH_W2T) ? a.w2t + (size_t)l * m.hidden * m.dim
                                          : m.wcls;
        mbar_expect_tx(full, (unsigned)(n * rb));
        bulk_g2s(stage, W + (size_t)c0 * b.cols, (unsigned)(n * rb), full);
    }
}

// Ring cursor: chunk counter c -> stage c % NS, use c / NS.
struct Ring {
    float *stages;
    uint64_t *full, *empty;
    unsigned c;
};

__device__ __forceinline__ float *ring_stage(const Ring &r) { return r.stages + (r.c % PS_STAGES) * (MV_STAGE_BYTES / 4); }

// ---- producer warp ------------------------------------------------------------
__device__ void producer(const PersistArgs &a, Ring r) {
    if ((threadIdx.x & 31) != 0) return;
    const int L = a.m.L;
    for (int step = 0; step < a.n_steps; step++) {
        for (int l = 0; l < L; l++) {
            for (int ph = PH_QKV; ph <= PH_W2T; ph++) {
                const Block b = phase_block(a, ph);
                const int nk = n_chunks(b);
                for (int k = 0; k < nk; k++, r.c++) {
                    const unsigned s = r.c % PS_STAGES, u = r.c / PS_STAGES;
                    if (u > 0 && !mbar_wait_bounded(&r.empty[s], (u - 1) & 1, a.m.err, ERR_STAGE_EMPTY)) return;
                    if (err_set(a)) return;
                    issue_chunk(a, ph, l, b, k, ring_stage(r), &r.full[s]);
                }
            }
        }
        if (a.has_head) {
            const Block b = phase_block(a, PH_CLS);
            const int nk = n_chunks(b);
            for (int k = 0; k < nk; k++, r.c++) {
                const unsigned s = r.c % PS_STAGES, u = r.c / PS_STAGES;
                if (u > 0 && !mbar_wait_bounded(&r.empty[s], (u - 1) & 1, a.m.err, ERR_STAGE_EMPTY)) return;
                if (err_set(a)) return;
                issue_chunk(a, PH_CLS, 0, b, k, ring_stage(r), &r.full[s]);
            }
        }
    }
}

// Consumer side of one chunk: wait full, run f(stage, c0, c1), release.
template <typename F>
__device__ __forceinline__ bool consume(const PersistArgs &a, Ring &r, const Block &b, int k, int *s_abort, F f) {
    const unsigned s = r.c % PS_STAGES, u = r.c / PS_STAGES;
    const bool got = mbar_wait_bounded(&r.full[s], u & 1, a.m.err, ERR_STAGE_FULL);
    if (!got) *s_abort = 1;
    if (got) {
        const int c0 = b.it0 + k * b.ps, c1 = min(b.it1, c0 + b.ps);
        f(ring_stage(r), c0, c1);
    }
    __syncwarp();
    if ((threadIdx.x & 31) == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&r.empty[s])) : "memory");
    r.c++;
    return got;
}

template <int NV>
__device__ __forceinline__ void load_vec(float4 (&x)[NV], const float *src, int c4, int lane) {
    const float4 *s4 = reinterpret_cast<const float4 *>(src);
#pragma unroll
    for (int v = 0; v < NV; v++) {
        const int c = lane + 32 * v;
        x[v] = (c < c4) ? __ldcg(s4 + c) : make_float4(0.f, 0.f, 0.f, 0.f);
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

// o = (x * s) * g with s = 1 / sqrt(mean(x^2) + 1e-5) (pitorch/ops/core/pt_ops.c:5-12);
// the gain vector is loaded by the caller together with x (one round trip).
template <int NV>
__device__ __forceinline__ void rmsnorm_vec(float4 (&x)[NV], const float4 (&g)[NV], int dim) {
    float ss = 0.f;
#pragma unroll
    for (int v = 0; v < NV; v++) ss += x[v].x * x[v].x + x[v].y * x[v].y + x[v].z * x[v].z + x[v].w * x[v].w;
    ss = warp_sum(ss);
    const float sc = rms_scale(ss, dim);
#pragma unroll
    for (int v = 0; v < NV; v++) {
        x[v].x = __fmul_rn(__fmul_rn(x[v].x, sc), g[v].x);
        x[v].y = __fmul_rn(__fmul_rn(x[v].y, sc), g[v].y);
        x[v].z = __fmul_rn(__fmul_rn(x[v].z, sc), g[v].z);
        x[v].w = __fmul_rn(__fmul_rn(x[v].w, sc), g[v].w);
    }
}

template <int NV>
__device__ __forceinline__ float dot_smem(const float *row, const float4 (&x)[NV], int c4, int lane) {
    const float4 *r4 = reinterpret_cast<const float4 *>(row);
    float acc = 0.f;
#pragma unroll
    for (int v = 0; v < NV; v++) {
        const int c = lane + 32 * v;
        if (c < c4) acc = dot4(r4[c], x[v], acc);
    }
    return warp_sum(acc);
}

// ---- attention item: (head h, positions [t0, t1)) -> partial ---------------
// q, the K rows of the first 64 positions and the first V rows of every
// value thread are all loaded before any of them is used, so the item costs
// one memory round trip for n <= 64 positions (hd <= 64).
__device__ void att_item(const PersistArgs &a, int l, int h, int t0, int t1, float *part, float *sm_p,
                         float *sm_o, float *sm_stat) {
    const DecodeModel &m = a.m;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int hd = m.hd, hd4 = hd >> 2;
    const int kvh = h / (m.nh / m.nkv);
    const size_t head_base = ((size_t)l * m.nkv + kvh) * m.seq;
    const float scale = __fdiv_rn(1.0f, pt_sqrtf((float)hd));
    const int ngrp = PS_ATT_THREADS / hd4;
    const int d4 = tid % hd4, grp = tid / hd4;
    const int n = t1 - t0;
    const int js = tid >> 2, sub = tid & 3;
    const float4 *q4 = reinterpret_cast<const float4 *>(m.q + h * hd);
    const float4 *vb = reinterpret_cast<const float4 *>(m.vc + (head_base + t0) * hd);
    constexpr int QK = 4;   // float4 chunks of q per scores thread (hd <= 64)
    constexpr int VP = 4;   // prefetched V rows per value thread
    float4 qv[QK], kv[QK], vpre[VP];
#pragma unroll
    for (int i = 0; i < QK; i++) {
        const int c = sub + 4 * i;
        qv[i] = (c < hd4) ? __ldcg(q4 + c) : make_float4(0.f, 0.f, 0.f, 0.f);
        const float4 *kr = reinterpret_cast<const float4 *>(m.kc + (head_base + t0 + js) * hd);
        kv[i] = (c < hd4 && js < n) ? __ldcg(kr + c) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int k = 0; k < VP; k++) {
        const int j = grp + ngrp * k;
        vpre[k] = (grp < ngrp && j < n) ? __ldcg(vb + (size_t)j * hd4 + d4) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    for (int j0 = 0; j0 < n; j0 += PS_ATT_THREADS / 4) {
        const int j = j0 + js;
        if (j0 > 0) {
#pragma unroll
            for (int i = 0; i < QK; i++) {
                const int c = sub + 4 * i;
                const float4 *kr = reinterpret_cast<const float4 *>(m.kc + (head_base + t0 + j) * hd);
                kv[i] = (c < hd4 && j < n) ? __ldcg(kr + c) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
        float acc = 0.f;
#pragma unroll
        for (int i = 0; i < QK; i++) acc = dot4(kv[i], qv[i], acc);
        acc += __shfl_xor_sync(0xffffffffu, acc, 1);
        acc += __shfl_xor_sync(0xffffffffu, acc, 2);
        if (j < n && sub == 0) sm_p[j] = __fmul_rn(acc, scale);
    }
    att_sync();
    if (warp == 0) {
        float mx = -3.4028235e+38f;
        for (int j = lane; j < n; j += 32) mx = fmaxf(mx, sm_p[j]);
        mx = warp_max(mx);
        float sum = 0.f;
        for (int j = lane; j < n; j += 32) {
            const float e = pt_expf(__fsub_rn(sm_p[j], mx));
            sm_p[j] = e;
            sum += e;
        }
        sum = warp_sum(sum);
        if (lane == 0) { sm_stat[0] = mx; sm_stat[1] = sum; }
    }
    att_sync();
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
    if (grp < ngrp) {
#pragma unroll
        for (int k = 0; k < VP; k++) {
            const int j = grp + ngrp * k;
            if (j < n) {
                const float e = sm_p[j];
                o.x = fmaf(e, vpre[k].x, o.x); o.y = fmaf(e, vpre[k].y, o.y);
                o.z = fmaf(e, vpre[k].z, o.z); o.w = fmaf(e, vpre[k].w, o.w);
            }
        }
        for (int j = grp + ngrp * VP; j < n; j += ngrp) {
            const float4 v = __ldcg(vb + (size_t)j * hd4 + d4);
            const float e = sm_p[j];
            o.x = fmaf(e, v.x, o.x); o.y = fmaf(e, v.y, o.y);
            o.z = fmaf(e, v.z, o.z); o.w = fmaf(e, v.w, o.w);
        }
        reinterpret_cast<float4 *>(sm_o)[grp * hd4 + d4] = o;
    }
    att_sync();
    for (int d = tid; d < hd; d += PS_ATT_THREADS) {
        float acc = 0.f;
        for (int g = 0; g < ngrp; g++) acc += sm_o[g * hd + d];
        part[d] = acc;
    }
    if (tid == 0) { part[hd] = sm_stat[0]; part[hd + 1] = sm_stat[1]; }
    att_sync();
}

// ---- the kernel --------------------------------------------------------------------
template <int NVD>
__global__ void __launch_bounds__(PS_THREADS, 1) k_persist(PersistArgs a) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    const DecodeModel &m = a.m;
    Ring r;
    r.stages = reinterpret_cast<float *>(smem_raw);
    r.full = reinterpret_cast<uint64_t *>(smem_raw + PS_STAGES * MV_STAGE_BYTES);
    r.empty = r.full + PS_STAGES;
    r.c = 0;
    float *sm_vec = reinterpret_cast<float *>(r.empty + PS_STAGES);   // [max(dim, hidden-block)] + extras
    float *sm_att = sm_vec;                      // [dim] merged attention output
    float *sm_hb = sm_vec + PS_MAX_DIM;          // [hidden block]
    float *sm_q = sm_hb + PS_MAX_HBLOCK;         // [hd]
    float *sm_p = sm_q + 256;                    // [positions per item]
    float *sm_o = sm_p + PS_MAX_ITEM_POS;        // [PS_ATT_THREADS * 4]
    float *sm_stat = sm_o + PS_ATT_THREADS * 4;  // [2 + 2*nh*maxc]
    float *sm_part = sm_stat + PS_STAT_FLOATS;   // [nh * nch * (hd + 2)] staged partials
    float *sm_xrow = sm_part + PS_PART_FLOATS;   // [wo rows of this CTA]
    __shared__ int s_abort;
    __shared__ int s_next;
    __shared__ unsigned long long s_best[PS_CONS_WARPS];

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        for (int s = 0; s < PS_STAGES; s++) {
            mbar_init(&r.full[s], 1);
            mbar_init(&r.empty[s], PS_CONS_WARPS);
        }
        mbar_init_fence();
        s_abort = 0;
    }
    __syncthreads();
    if (warp == PS_WARPS - 1) {
        producer(a, r);
        return;
    }

    const int G = gridDim.x, D = m.dim, H = m.hidden;
    const int c4d = D >> 2;
    (void)H;
    unsigned epoch = 0;
    StepState *st = m.step;
    int pos = __ldcg(&st->pos);
    int tok = __ldcg(&st->tok);
    const int mode = st->mode;
    const int n_prompt = st->n_prompt;

    for (int step = 0; step < a.n_steps; step++) {
        if (pos < 0 || pos >= m.seq) break;
        for (int l = 0; l < m.L; l++) {
            // ---------------- QKV ----------------
            {
                const Block b = phase_block(a, PH_QKV);
                float4 xr[NVD], gr[NVD];
                const bool from_emb = a.has_embed && l == 0;
                const float *xsrc = from_emb ? m.emb + (size_t)tok * D : m.x;
                load_gain<NVD>(gr, m.rms_att + (size_t)l * D, c4d, lane);
                load_vec<NVD>(xr, xsrc, c4d, lane);
                if (from_emb && blockIdx.x == 0 && warp == 0) {
                    float4 *x4 = reinterpret_cast<float4 *>(m.x);
#pragma unroll
                    for (int v = 0; v < NVD; v++) if (lane + 32 * v < c4d) x4[lane + 32 * v] = xr[v];
                }
                rmsnorm_vec<NVD>(xr, gr, D);
                const int nk = n_chunks(b);
                for (int k = 0; k < nk; k++) {
                    consume(a, r, b, k, &s_abort, [&](const float *stage, int c0, int c1) {
                        for (int i = c0 + warp; i < c1; i += PS_CONS_WARPS) {
                            const int li = i - c0;
                            const float a0 = dot_smem<NVD>(stage + (size_t)(2 * li) * D, xr, c4d, lane);
                            const float a1 = dot_smem<NVD>(stage + (size_t)(2 * li + 1) * D, xr, c4d, lane);
                            if (lane == 0) {
                                const int r0 = 2 * i, hd = m.hd;
                                if (r0 < D + m.kvd) {
                                    const bool is_q = r0 < D;
                                    const int j = is_q ? r0 : r0 - D;
                                    const float th = rope_theta(j, hd, pos);
                                    const float cs = pt_cosf(th), sn = pt_sinf(th);
                                    const float o0 = __fsub_rn(__fmul_rn(a0, cs), __fmul_rn(a1, sn));
                                    const float o1 = __fadd_rn(__fmul_rn(a0, sn), __fmul_rn(a1, cs));
                                    if (is_q) { m.q[j] = o0; m.q[j + 1] = o1; }
                                    else {
                                        float *dst = m.kc + (((size_t)l * m.nkv + j / hd) * m.seq + pos) * hd + (j % hd);
                                        dst[0] = o0; dst[1] = o1;
                                    }
                                } else {
                                    const int j = r0 - D - m.kvd;
                                    float *dst = m.vc + (((size_t)l * m.nkv + j / hd) * m.seq + pos) * hd + (j % hd);
                                    dst[0] = a0; dst[1] = a1;
                                }
                            }
                        }
                    });
                }
                if (!grid_barrier(a, epoch, &s_abort)) return;
            }
            // the previous token's argmax key has been read by every CTA
            if (l == 0 && blockIdx.x == 0 && tid == 0) st->amax = 0ull;
            // ---------------- ATT ----------------
            const int nh = m.nh;
            int nch = (pos + 1 + 15) / 16;
            const int maxc = max(1, G / nh);
            if (nch > maxc) nch = maxc;
            {
                const int per = (pos + 1 + nch - 1) / nch;
                if (warp < PS_ATT_THREADS / 32) {
                    for (int item = blockIdx.x; item < nh * nch; item += G) {
                        const int h = item / nch, c = item % nch;
                        const int t0 = c * per, t1 = min(pos + 1, t0 + per);
                        float *part = a.att_part + ((size_t)h * a.max_chunks + c) * (m.hd + 2);
                        if (t0 < t1) {
                            att_item(a, l, h, t0, t1, part, sm_p, sm_o, sm_stat);
                        } else if (tid == 0) {
                            part[m.hd] = -3.4028235e+38f;
                            part[m.hd + 1] = 0.f;
                        }
                    }
                }
                if (!grid_barrier(a, epoch, &s_abort)) return;
            }
            // ---------------- WO ----------------
            {
                const int hd = m.hd;
                // merge: stage every partial record (and this CTA's residual rows)
                // with one round of independent loads, then work in shared memory
                const int rec = hd + 2;
                const Block b = phase_block(a, PH_WO);
                for (int e = tid; e < nh * nch * rec; e += PS_CONS_THREADS) {
                    const int t = e / rec, j = e % rec;
                    const int h = t / nch, c = t % nch;
                    sm_part[e] = __ldcg(a.att_part + ((size_t)h * a.max_chunks + c) * rec + j);
                }
                for (int i = b.it0 + tid; i < b.it1; i += PS_CONS_THREADS) sm_xrow[i - b.it0] = __ldcg(m.x + i);
                cons_sync();
                float *sm_w = sm_stat + 2;
                float *sm_inv = sm_w + nh * maxc;
                for (int h = tid; h < nh; h += PS_CONS_THREADS) {
                    float M = -3.4028235e+38f;
                    for (int c = 0; c < nch; c++) M = fmaxf(M, sm_part[(h * nch + c) * rec + hd]);
                    float Ls = 0.f;
                    for (int c = 0; c < nch; c++) {
                        const float w = pt_expf(__fsub_rn(sm_part[(h * nch + c) * rec + hd], M));
                        sm_w[h * nch + c] = w;
                        Ls = fmaf(w, sm_part[(h * nch + c) * rec + hd + 1], Ls);
                    }
                    sm_inv[h] = __fdiv_rn(1.0f, Ls);
                }
                cons_sync();
                for (int t = tid; t < D; t += PS_CONS_THREADS) {
                    const int h = t / hd, d = t % hd;
                    float o = 0.f;
                    for (int c = 0; c < nch; c++) o = fmaf(sm_w[h * nch + c], sm_part[(h * nch + c) * rec + d], o);
                    sm_att[t] = o * sm_inv[h];
                }
                cons_sync();
                float4 ar[NVD];
                {
                    const float4 *a4 = reinterpret_cast<const float4 *>(sm_att);
#pragma unroll
                    for (int v = 0; v < NVD; v++) {
                        const int c = lane + 32 * v;
                        ar[v] = (c < c4d) ? a4[c] : make_float4(0.f, 0.f, 0.f, 0.f);
                    }
                }
                const int nk = n_chunks(b);
                for (int k = 0; k < nk; k++) {
                    consume(a, r, b, k, &s_abort, [&](const float *stage, int c0, int c1) {
                        for (int i = c0 + warp; i < c1; i += PS_CONS_WARPS) {
                            const float v = dot_smem<NVD>(stage + (size_t)(i - c0) * D, ar, c4d, lane);
                            if (lane == 0) {
                                const float xv = __fadd_rn(sm_xrow[i - b.it0], v);
                                m.x[i] = xv;
                                a.x1[i] = xv;
                            }
                        }
                    });
                }
                if (!grid_barrier(a, epoch, &s_abort)) return;
            }
            // ---------------- FFN ----------------
            {
                const Block b13 = phase_block(a, PH_FFN13);
                float4 xr[NVD], gr[NVD];
                load_gain<NVD>(gr, m.rms_ffn + (size_t)l * D, c4d, lane);
                load_vec<NVD>(xr, a.x1, c4d, lane);
                rmsnorm_vec<NVD>(xr, gr, D);
                const int nk = n_chunks(b13);
                for (int k = 0; k < nk; k++) {
                    consume(a, r, b13, k, &s_abort, [&](const float *stage, int c0, int c1) {
                        for (int i = c0 + warp; i < c1; i += PS_CONS_WARPS) {
                            const int li = i - c0;
                            const float h1 = dot_smem<NVD>(stage + (size_t)li * D, xr, c4d, lane);
                            const float h3 = dot_smem<NVD>(stage + (size_t)(b13.ps + li) * D, xr, c4d, lane);
                            if (lane == 0) sm_hb[i - b13.it0] = silu_mul(h1, h3);
                        }
                    });
                }
                cons_sync();
                // x0 += w2[:, block] . hb[block]: thread t owns row quads t, t+480, ...
                const Block b2 = phase_block(a, PH_W2T);
                constexpr int NQ = (PS_MAX_DIM / 4 + PS_CONS_THREADS - 1) / PS_CONS_THREADS;
                float4 acc[NQ];
#pragma unroll
                for (int q = 0; q < NQ; q++) acc[q] = make_float4(0.f, 0.f, 0.f, 0.f);
                const int nk2 = n_chunks(b2);
                for (int k = 0; k < nk2; k++) {
                    consume(a, r, b2, k, &s_abort, [&](const float *stage, int c0, int c1) {
#pragma unroll
                        for (int q = 0; q < NQ; q++) {
                            const int g4 = tid + q * PS_CONS_THREADS;
                            if (g4 < c4d) {
                                float4 s4 = acc[q];
                                for (int i = c0; i < c1; i++) {
                                    const float4 w = reinterpret_cast<const float4 *>(stage + (size_t)(i - c0) * D)[g4];
                                    const float h = sm_hb[i - b2.it0];
                                    s4.x = fmaf(w.x, h, s4.x); s4.y = fmaf(w.y, h, s4.y);
                                    s4.z = fmaf(w.z, h, s4.z); s4.w = fmaf(w.w, h, s4.w);
                                }
                                acc[q] = s4;
                            }
                        }
                    });
                }
                if (b2.it1 > b2.it0) {
#pragma unroll
                    for (int q = 0; q < NQ; q++) {
                        const int g4 = tid + q * PS_CONS_THREADS;
                        if (g4 < c4d)
                            asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(m.x + 4 * g4),
                                         "f"(acc[q].x), "f"(acc[q].y), "f"(acc[q].z), "f"(acc[q].w)
                                         : "memory");
                    }
                }
                if (!grid_barrier(a, epoch, &s_abort)) return;
            }
        }
        if (!a.has_head) break;   // layer-only decoder: one position per launch
        // ---------------- CLS ----------------
        {
            const Block b = phase_block(a, PH_CLS);
            float4 xr[NVD], gr[NVD];
            load_gain<NVD>(gr, m.rms_final, c4d, lane);
            load_vec<NVD>(xr, m.x, c4d, lane);
            rmsnorm_vec<NVD>(xr, gr, D);
            if (blockIdx.x == 0 && warp == 0) {
                float4 *x4 = reinterpret_cast<float4 *>(m.xn);
#pragma unroll
                for (int v = 0; v < NVD; v++) if (lane + 32 * v < c4d) x4[lane + 32 * v] = xr[v];
            }
            unsigned long long best = 0ull;
            const int nk = n_chunks(b);
            for (int k = 0; k < nk; k++) {
                consume(a, r, b, k, &s_abort, [&](const float *stage, int c0, int c1) {
                    for (int i = c0 + warp; i < c1; i += PS_CONS_WARPS) {
                        const float v = dot_smem<NVD>(stage + (size_t)(i - c0) * D, xr, c4d, lane);
                        if (lane == 0) {
                            m.logits[i] = v;
                            const unsigned long long key = argmax_key(v, i);
                            if (key > best) best = key;
                        }
                    }
                });
            }
            if (lane == 0) s_best[warp] = best;
            cons_sync();
            if (tid == 0) {
                unsigned long long bb = 0ull;
                for (int w = 0; w < PS_CONS_WARPS; w++) bb = s_best[w] > bb ? s_best[w] : bb;
                if (bb) atomicMax(&st->amax, bb);
            }
            if (!grid_barrier(a, epoch, &s_abort)) return;
            if (tid == 0) s_next = argmax_key_index(atomicAdd(&st->amax, 0ull));
            cons_sync();
            const int next = s_next;
            if (blockIdx.x == 0 && tid == 0) {
                st->next = next;
                if (mode == 1) {
                    if (pos + 1 >= n_prompt && pos + 1 <= m.seq) st->tokens[pos + 1] = next;
                }
            }
            if (mode == 1) {
                tok = (pos + 1 < n_prompt) ? __ldcg(st->tokens + pos + 1) : next;
                pos = pos + 1;
                if (blockIdx.x == 0 && tid == 0) { st->pos = pos; st->tok = tok; }
            }
        }
    }
}

// ---- host side -------------------------------------------------------------------

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

// w2t[l] = w2[l]^T for each layer ([dim, hidden] -> [hidden, dim]).
void persist_transpose_w2(const DecodeModel &m, float *w2t, cudaStream_t s) {
    for (int l = 0; l < m.L; l++)
        k_transpose<<<dim3((m.hidden + 31) / 32, (m.dim + 31) / 32), dim3(32, 8), 0, s>>>(
            w2t + (size_t)l * m.hidden * m.dim, m.w2 + (size_t)l * m.dim * m.hidden, m.dim, m.hidden);
    PTC_CHECK(cudaGetLastError());
}

size_t persist_smem_bytes(const DecodeModel &m) {
    (void)m;
    return (size_t)PS_STAGES * MV_STAGE_BYTES + 2 * PS_STAGES * 8 +
           4 * (size_t)(PS_MAX_DIM + PS_MAX_HBLOCK + 256 + PS_MAX_ITEM_POS + PS_ATT_THREADS * 4 + PS_STAT_FLOATS +
                        PS_PART_FLOATS + PS_MAX_WO_ROWS);
}

bool persist_supported(const DecodeModel &m, int n_sm) {
    const int hblock = (m.hidden + n_sm - 1) / n_sm;
    const int maxc = n_sm / m.nh > 0 ? n_sm / m.nh : 1;
    const int item_pos = (m.seq + maxc - 1) / maxc;
    return m.dim <= PS_MAX_DIM && m.hidden <= 2048 && m.dim % 4 == 0 && m.hidden % 4 == 0 && m.hd % 4 == 0 &&
           m.hd <= 64 && hblock <= PS_MAX_HBLOCK && item_pos <= PS_MAX_ITEM_POS &&
           2 + 2 * m.nh * maxc <= PS_STAT_FLOATS && m.nh <= n_sm &&
           m.nh * maxc * (m.hd + 2) <= PS_PART_FLOATS && (m.dim + n_sm - 1) / n_sm <= PS_MAX_WO_ROWS &&
           MV_STAGE_BYTES / (2 * m.dim * 4) >= 1;
}

#define PS_NV_CASES(X) X(1) X(2) X(3) X(4) X(5) X(6) X(7) X(8) X(9) X(10) X(11) X(12) X(13) X(14) X(15) X(16)

void persist_launch(const PersistArgs &a, int n_sm, cudaStream_t s) {
    const int nvd = (a.m.dim / 4 + 31) / 32;
    const size_t smem = persist_smem_bytes(a.m);
    void (*kern)(PersistArgs) = nullptr;
    switch (nvd) {
#define PS_CASE(N) \
    case N: kern = k_persist<N>; break;
        PS_NV_CASES(PS_CASE)
#undef PS_CASE
        default: PTC_FATAL("persistent decode: dim %d too large", a.m.dim);
    }
    ensure_kernel_smem((const void *)kern, smem);
    PTC_CHECK(cudaMemsetAsync(a.bar, 0, sizeof(unsigned), s));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(n_sm);
    cfg.blockDim = dim3(PS_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    PTC_CHECK(cudaLaunchKernelEx(&cfg, kern, a));
}

}  // namespace ptc
