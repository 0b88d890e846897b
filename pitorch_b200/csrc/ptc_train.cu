// ptc_train.cu -- pt_train_step on the GPU: batched forward with saved
// activations, cross-entropy, the 7-operator backward and SGD.
//
// Follows pitorch/train/pt_train.c (forward :171-329, backward :549-866,
// SGD :870-942, staged variants :946-1383) and the primitives of
// pitorch/train/pt_backward_ops.c. The reference runs T per-position matvecs
// per linear layer and a CPU outer-product loop for weight gradients; here
// every linear layer is one fp32 GEMM over all positions (ptc_gemm.cu) and
// the elementwise/normalisation/attention work runs as small kernels.
// Position T-1 carries no loss and is skipped by every backward GEMM, as in
// pt_train.c:596-605.
//
// Buffers (device, sized for max_T and the context's local layers L) use the
// reference's activation layout (pt_train.h:19-32), e.g. residuals
// [(L+1), T, dim], att [L, n_heads, T, T], and its gradient layout
// (pt_train.c:334-371). All are carved from the context arena at creation;
// a step allocates nothing.
#include <string.h>

#include "../../include/ptc.h"
#include "ptc_common.cuh"
#include "ptc_gemm.h"
#include "ptc_internal.h"

using ptc::GemmArgs;

namespace ptc {

// ---------------------------------------------------------------------------
// Elementwise / row kernels
// ---------------------------------------------------------------------------

// residuals[0][t] = emb[tokens[t]] (pt_train.c:189-191)
__global__ void k_tr_embed(float *res, const float *emb, const int *tokens, int T, int D) {
    for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < T * D; e += gridDim.x * blockDim.x) {
        const int t = e / D, i = e % D;
        res[e] = emb[(size_t)tokens[t] * D + i];
    }
}

// One warp per row: out = (x * s) * w, s = 1/sqrt(mean(x^2)+eps) (pt_ops.c:5-12).
__global__ void k_tr_rmsnorm(float *__restrict__ out, const float *__restrict__ x, const float *__restrict__ w,
                             int rows, int D) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= rows) return;
    const float *xr = x + (size_t)warp * D;
    float ss = 0.f;
    // unrolled so that a lane's loads are in flight together (the sums keep
    // their order)
#pragma unroll 8
    for (int i = lane; i < D; i += 32) ss = fmaf(xr[i], xr[i], ss);
    ss = warp_sum(ss);
    const float s = rms_scale(ss, D);
    float *o = out + (size_t)warp * D;
#pragma unroll 8
    for (int i = lane; i < D; i += 32) o[i] = __fmul_rn(__fmul_rn(xr[i], s), w[i]);
}

// Causal attention forward, one CTA per (head, t) (pt_train.c:224-259):
// att row = softmax(q_t . k_s * scale) for s <= t (zeros after t), and
// att_out[t, h] = sum_s att[s] v_s.
__global__ void __launch_bounds__(128) k_tr_attn_fwd(const float *q, const float *k, const float *v,
                                                     float *att, float *out, int T, int nh, int nkv,
                                                     int hd) {
    extern __shared__ float sm[];
    float *s_q = sm;          // [hd]
    float *s_p = sm + hd;     // [T]
    __shared__ float s_red[2];
    const int h = blockIdx.x, t = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarp = blockDim.x >> 5;
    const int D = nh * hd, K = nkv * hd, koff = (h / (nh / nkv)) * hd;
    const float scale = __fdiv_rn(1.0f, pt_sqrtf((float)hd));
    for (int d = threadIdx.x; d < hd; d += blockDim.x) s_q[d] = q[(size_t)t * D + h * hd + d];
    __syncthreads();
    // one thread per position: independent 128-bit loads of k_s
    for (int s = threadIdx.x; s <= t; s += blockDim.x) {
        const float4 *kr = reinterpret_cast<const float4 *>(k + (size_t)s * K + koff);
        const float4 *q4 = reinterpret_cast<const float4 *>(s_q);
        float acc = 0.f;
        for (int d4 = 0; d4 < hd / 4; d4++) acc = dot4(__ldg(kr + d4), q4[d4], acc);
        s_p[s] = __fmul_rn(acc, scale);
    }
    __syncthreads();
    if (warp == 0) {
        float mx = -3.4028235e+38f;
        for (int s = lane; s <= t; s += 32) mx = fmaxf(mx, s_p[s]);
        mx = warp_max(mx);
        float sum = 0.f;
        for (int s = lane; s <= t; s += 32) {
            const float e = pt_expf(__fsub_rn(s_p[s], mx));
            s_p[s] = e;
            sum += e;
        }
        sum = warp_sum(sum);
        if (lane == 0) s_red[0] = __fdiv_rn(1.0f, sum);
    }
    __syncthreads();
    const float inv = s_red[0];
    float *arow = att + ((size_t)h * T + t) * T;
    for (int s = threadIdx.x; s < T; s += blockDim.x) {
        const float p = (s <= t) ? __fmul_rn(s_p[s], inv) : 0.f;
        if (s <= t) s_p[s] = p;
        arow[s] = p;
    }
    __syncthreads();
    // weighted values: warp w sums positions s = w (mod 4) for columns
    // lane and lane + 32; the four partial sums are added in warp order
    __shared__ float s_part[4][64];
    float o0 = 0.f, o1 = 0.f;
    for (int s = warp; s <= t; s += nwarp) {
        const float p = s_p[s];
        const float *vr = v + (size_t)s * K + koff;
        if (lane < hd) o0 = fmaf(p, vr[lane], o0);
        if (lane + 32 < hd) o1 = fmaf(p, vr[lane + 32], o1);
    }
    s_part[warp][lane] = o0;
    s_part[warp][lane + 32] = o1;
    __syncthreads();
    for (int d = threadIdx.x; d < hd; d += blockDim.x) {
        float o = 0.f;
        for (int w = 0; w < nwarp; w++) o += s_part[w][d];
        out[(size_t)t * D + h * hd + d] = o;
    }
}

// Row-block variants of the two per-row attention kernels, for T <= TB_T:
// one CTA per (head, TB_R consecutive query rows), one warp per row. The
// head's K and V rows 0..n_s-1 (n_s = last row of the block + 1) are staged
// once per CTA in shared memory with a row stride of hd + 4 floats (16-byte
// rows; the float4 reads of 8 consecutive rows then hit distinct banks).
// Lane j of a warp owns positions j, j + 32, ... of its row.
constexpr int TB_R = 8;
constexpr int TB_J = 8;
constexpr int TB_T = 32 * TB_J;

size_t attn_block_smem(int T, int hd) {
    return ((size_t)2 * T * (hd + 4) + (size_t)TB_R * hd + (size_t)TB_R * T) * 4;
}

__device__ __forceinline__ void stage_kv_rows(float *sK, float *sV, const float *k, const float *v, int n_s,
                                              int K, int koff, int hd) {
    const int hd4 = hd >> 2, ks = hd + 4;
    for (int f = threadIdx.x; f < n_s * hd4; f += blockDim.x) {
        const int s = f / hd4, c = f - s * hd4;
        reinterpret_cast<float4 *>(sK + (size_t)s * ks)[c] =
            __ldg(reinterpret_cast<const float4 *>(k + (size_t)s * K + koff) + c);
        reinterpret_cast<float4 *>(sV + (size_t)s * ks)[c] =
            __ldg(reinterpret_cast<const float4 *>(v + (size_t)s * K + koff) + c);
    }
}

// Forward (pt_train.c:224-259): att row t = softmax(q_t . k_s * scale) over
// s <= t (zeros after t), att_out[t, h] = sum_s att[s] v_s.
__global__ void __launch_bounds__(TB_R * 32) k_tr_attn_fwd_blk(const float *q, const float *k, const float *v,
                                                              float *att, float *out, int T, int nh, int nkv,
                                                              int hd) {
    extern __shared__ __align__(16) float sm[];
    const int h = blockIdx.x, t0 = blockIdx.y * TB_R;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int D = nh * hd, K = nkv * hd, koff = (h / (nh / nkv)) * hd, hd4 = hd >> 2, ks = hd + 4;
    const int n_s = min(T, t0 + TB_R);
    float *sK = sm, *sV = sm + (size_t)T * ks, *sQ = sV + (size_t)T * ks, *sP = sQ + TB_R * hd;
    stage_kv_rows(sK, sV, k, v, n_s, K, koff, hd);
    const int t = t0 + warp;
    if (t < T)
        for (int d = lane; d < hd; d += 32) sQ[warp * hd + d] = q[(size_t)t * D + h * hd + d];
    __syncthreads();
    if (t >= T) return;   // no block barrier follows
    const float scale = __fdiv_rn(1.0f, pt_sqrtf((float)hd));
    const float4 *q4 = reinterpret_cast<const float4 *>(sQ + warp * hd);
    float sc[TB_J];
    float mx = -3.4028235e+38f;
#pragma unroll
    for (int j = 0; j < TB_J; j++) {
        const int sp = lane + 32 * j;
        sc[j] = 0.f;
        if (sp <= t) {
            const float4 *k4 = reinterpret_cast<const float4 *>(sK + (size_t)sp * ks);
            float acc = 0.f;
            for (int c = 0; c < hd4; c++) acc = dot4(k4[c], q4[c], acc);
            sc[j] = __fmul_rn(acc, scale);
            mx = fmaxf(mx, sc[j]);
        }
    }
    mx = warp_max(mx);
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < TB_J; j++) {
        if (lane + 32 * j <= t) {
            sc[j] = pt_expf(__fsub_rn(sc[j], mx));
            sum += sc[j];
        }
    }
    sum = warp_sum(sum);
    const float inv = __fdiv_rn(1.0f, sum);
    float *arow = att + ((size_t)h * T + t) * T, *prow = sP + warp * T;
#pragma unroll
    for (int j = 0; j < TB_J; j++) {
        const int sp = lane + 32 * j;
        if (sp < T) {
            const float pv = (sp <= t) ? __fmul_rn(sc[j], inv) : 0.f;
            arow[sp] = pv;
            prow[sp] = pv;
        }
    }
    __syncwarp();
    float o0 = 0.f, o1 = 0.f;
    for (int sp = 0; sp <= t; sp++) {
        const float pv = prow[sp];
        const float *vr = sV + (size_t)sp * ks;
        if (lane < hd) o0 = fmaf(pv, vr[lane], o0);
        if (lane + 32 < hd) o1 = fmaf(pv, vr[lane + 32], o1);
    }
    float *orow = out + (size_t)t * D + h * hd;
    if (lane < hd) orow[lane] = o0;
    if (lane + 32 < hd) orow[lane + 32] = o1;
}

// Backward part 1 (pt_train.c:780-812) for rows t < n_rows: dP = d_ao . v,
// dS[t][s] = P[t][s] (dP[s] - <dP, P[t]>) * scale, d_q[t] = sum_s dS[t][s] k_s.
__global__ void __launch_bounds__(TB_R * 32) k_tr_attn_bwd_q_blk(const float *d_ao, const float *att,
                                                                const float *k, const float *v, float *dS,
                                                                float *d_q, int T, int n_rows, int nh, int nkv,
                                                                int hd) {
    extern __shared__ __align__(16) float sm[];
    const int h = blockIdx.x, t0 = blockIdx.y * TB_R;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int D = nh * hd, K = nkv * hd, koff = (h / (nh / nkv)) * hd, hd4 = hd >> 2, ks = hd + 4;
    const int n_s = min(n_rows, t0 + TB_R);
    float *sK = sm, *sV = sm + (size_t)T * ks, *sD = sV + (size_t)T * ks, *sP = sD + TB_R * hd;
    stage_kv_rows(sK, sV, k, v, n_s, K, koff, hd);
    const int t = t0 + warp;
    if (t < n_rows)
        for (int d = lane; d < hd; d += 32) sD[warp * hd + d] = d_ao[(size_t)t * D + h * hd + d];
    __syncthreads();
    if (t >= n_rows) return;   // no block barrier follows
    const float scale = __fdiv_rn(1.0f, pt_sqrtf((float)hd));
    const float4 *d4 = reinterpret_cast<const float4 *>(sD + warp * hd);
    const float *P = att + ((size_t)h * T + t) * T;
    float dp[TB_J], pr[TB_J];
    float dot = 0.f;
#pragma unroll
    for (int j = 0; j < TB_J; j++) {
        const int sp = lane + 32 * j;
        dp[j] = 0.f;
        pr[j] = 0.f;
        if (sp <= t) {
            const float4 *v4 = reinterpret_cast<const float4 *>(sV + (size_t)sp * ks);
            float acc = 0.f;
            for (int c = 0; c < hd4; c++) acc = dot4(v4[c], d4[c], acc);
            dp[j] = acc;
            pr[j] = P[sp];
            dot = fmaf(acc, pr[j], dot);
        }
    }
    dot = warp_sum(dot);
    float *dsr = dS + ((size_t)h * T + t) * T, *xrow = sP + warp * T;
#pragma unroll
    for (int j = 0; j < TB_J; j++) {
        const int sp = lane + 32 * j;
        if (sp < T) {
            const float x = (sp <= t) ? __fmul_rn(__fmul_rn(pr[j], __fsub_rn(dp[j], dot)), scale) : 0.f;
            dsr[sp] = x;
            xrow[sp] = x;
        }
    }
    __syncwarp();
    float a0 = 0.f, a1 = 0.f;
    for (int sp = 0; sp <= t; sp++) {
        const float x = xrow[sp];
        const float *kr = sK + (size_t)sp * ks;
        if (lane < hd) a0 = fmaf(x, kr[lane], a0);
        if (lane + 32 < hd) a1 = fmaf(x, kr[lane + 32], a1);
    }
    float *qrow = d_q + (size_t)t * D + h * hd;
    if (lane < hd) qrow[lane] = a0;
    if (lane + 32 < hd) qrow[lane + 32] = a1;
}

// sh = silu(h1) * h3 with the training form (h1 * sig) * h3 (pt_train.c:281-284).
__global__ void k_tr_silu_gate(float *sh, const float *h1, const float *h3, size_t n) {
    for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < n; e += (size_t)gridDim.x * blockDim.x) {
        const float a = h1[e];
        const float sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, pt_expf(-a)));
        sh[e] = __fmul_rn(__fmul_rn(a, sig), h3[e]);
    }
}

// Per-row cross-entropy (pt_train.c:309-325): one CTA per row t < T-1.
// Also keeps each row's max and exponential sum (row_max, row_sum) for the
// backward, which then needs one pass over the logits instead of three.
__global__ void k_tr_ce_rows(const float *__restrict__ logits, const int *tokens, int V, float *loss_rows,
                             float *row_max, float *row_sum) {
    __shared__ float s_r[32];
    const int t = blockIdx.x;
    const float *__restrict__ lg = logits + (size_t)t * V;
    float mx = -3.4028235e+38f;
#pragma unroll 8
    for (int v = threadIdx.x; v < V; v += blockDim.x) mx = fmaxf(mx, lg[v]);
    mx = warp_max(mx);
    if ((threadIdx.x & 31) == 0) s_r[threadIdx.x >> 5] = mx;
    __syncthreads();
    if (threadIdx.x < 32) {
        float m = threadIdx.x < (blockDim.x >> 5) ? s_r[threadIdx.x] : -3.4028235e+38f;
        m = warp_max(m);
        if (threadIdx.x == 0) s_r[0] = m;
    }
    __syncthreads();
    mx = s_r[0];
    __syncthreads();
    float sum = 0.f;
#pragma unroll 8
    for (int v = threadIdx.x; v < V; v += blockDim.x) sum += pt_expf(__fsub_rn(lg[v], mx));
    sum = warp_sum(sum);
    if ((threadIdx.x & 31) == 0) s_r[threadIdx.x >> 5] = sum;
    __syncthreads();
    if (threadIdx.x == 0) {
        float s = 0.f;
        for (int w = 0; w < (int)(blockDim.x >> 5); w++) s += s_r[w];
        const float tgt = lg[tokens[t + 1]];
        loss_rows[t] = -(__fsub_rn(__fsub_rn(tgt, mx), pt_logf(s)));
        row_max[t] = mx;
        row_sum[t] = s;
    }
}

// loss = (sum_t loss_t) / (T-1), summed in position order as the reference does.
__global__ void k_tr_loss_sum(const float *loss_rows, int n, float *loss) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    float l = 0.f;
    for (int t = 0; t < n; t++) l = __fadd_rn(l, loss_rows[t]);
    *loss = __fdiv_rn(l, (float)n);
}

// d_logit rows (pt_train.c:609-621): softmax * (1/(T-1)), minus 1/(T-1) at the
// target. The row's max and exponential sum are the forward's (k_tr_ce_rows
// computed them with the same reductions), so one pass writes
// exp(l - max) * (1/sum * 1/(T-1)) -- the same bits as storing the
// exponentials and scaling them afterwards.
__global__ void k_tr_ce_backward(const float *__restrict__ logits, const int *tokens, int V, float invn,
                                 const float *row_max, const float *row_sum, float *__restrict__ dl_all) {
    const int t = blockIdx.x;
    const float *__restrict__ lg = logits + (size_t)t * V;
    float *__restrict__ dl = dl_all + (size_t)t * V;
    const float mx = row_max[t];
    const float f = __fmul_rn(__fdiv_rn(1.0f, row_sum[t]), invn);
    const int tgt = tokens[t + 1];
#pragma unroll 8
    for (int v = threadIdx.x; v < V; v += blockDim.x) {
        float x = __fmul_rn(pt_expf(__fsub_rn(lg[v], mx)), f);
        if (v == tgt) x = __fsub_rn(x, invn);
        dl[v] = x;
    }
}

// rmsnorm backward, one warp per row (pt_backward_ops.c:4-30): dx += ..., and
// the row's weight-grad contribution d_o * x * inv into dw_rows.
// d_o is the sum of up to three products computed side by side (d_o2, d_o3
// null when absent), added here in the order in which accumulating them into
// one buffer would have: (d_o + d_o2) + d_o3.
__device__ __forceinline__ float sum3(const float *__restrict__ a, const float *__restrict__ b,
                                      const float *__restrict__ c, size_t i) {
    float v = a[i];
    if (b) v = __fadd_rn(v, b[i]);
    if (c) v = __fadd_rn(v, c[i]);
    return v;
}

__global__ void k_tr_rmsnorm_bwd(float *__restrict__ dx, float *__restrict__ dw_rows, const float *__restrict__ d_o,
                                 const float *__restrict__ d_o2, const float *__restrict__ d_o3,
                                 const float *__restrict__ x, const float *__restrict__ w, int rows, int D) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= rows) return;
    const float *xr = x + (size_t)warp * D;
    const size_t ro = (size_t)warp * D;
    float ss = 0.f, dot = 0.f;
    // unrolled so that a lane's loads are in flight together (the sums keep
    // their order)
#pragma unroll 8
    for (int i = lane; i < D; i += 32) {
        ss = fmaf(xr[i], xr[i], ss);
        dot = fmaf(__fmul_rn(sum3(d_o, d_o2, d_o3, ro + i), w[i]), xr[i], dot);
    }
    ss = warp_sum(ss);
    dot = warp_sum(dot);
    const float inv = __fdiv_rn(1.0f, pt_sqrtf(__fadd_rn(__fdiv_rn(ss, (float)D), 1e-5f)));
    const float coeff = __fdiv_rn(__fmul_rn(__fmul_rn(inv, inv), inv), (float)D);
    float *dxr = dx + (size_t)warp * D;
    float *dwr = dw_rows + (size_t)warp * D;
#pragma unroll 8
    for (int i = lane; i < D; i += 32) {
        const float di = sum3(d_o, d_o2, d_o3, ro + i);
        dwr[i] = __fmul_rn(__fmul_rn(di, xr[i]), inv);
        const float a = __fmul_rn(__fmul_rn(inv, di), w[i]);
        const float b = __fmul_rn(__fmul_rn(coeff, dot), xr[i]);
        dxr[i] = __fadd_rn(dxr[i], __fsub_rn(a, b));
    }
}

// g[i] += sum over rows of dw_rows[t][i]: CTA = 32 columns, warp w sums
// rows w, w + 8, ... (lane = column), the 8 partials are added in warp order.
__global__ void __launch_bounds__(256) k_tr_colsum_accum(float *g, const float *rows_, int n_rows, int D) {
    __shared__ float s_part[8][33];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int i = blockIdx.x * 32 + lane;
    float acc = 0.f;
    if (i < D)
#pragma unroll 8
        for (int t = warp; t < n_rows; t += 8) acc = __fadd_rn(acc, rows_[(size_t)t * D + i]);
    s_part[warp][lane] = acc;
    __syncthreads();
    if (warp == 0 && i < D) {
        float sum = g[i];
        for (int w = 0; w < 8; w++) sum = __fadd_rn(sum, s_part[w][lane]);
        g[i] = sum;
    }
}

// silu*gate backward (pt_train.c:715-721).
__global__ void k_tr_silu_bwd(float *d_hid, float *d_hid2, const float *h1, const float *h3, size_t n) {
    for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < n; e += (size_t)gridDim.x * blockDim.x) {
        const float a = h1[e];
        const float sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, pt_expf(-a)));
        const float sv = __fmul_rn(a, sig);
        const float dh = d_hid[e];
        const float ds = __fmul_rn(dh, h3[e]);
        d_hid2[e] = __fmul_rn(dh, sv);
        d_hid[e] = __fmul_rn(__fmul_rn(ds, sig), __fadd_rn(1.0f, __fmul_rn(a, __fsub_rn(1.0f, sig))));
    }
}

// Attention backward part 1, one CTA per (head, t < T-1) (pt_train.c:780-812):
// dS[t][s] = P[t][s] (dP[t][s] - <dP[t], P[t]>) * scale with dP = d_ao . v,
// and d_q[t] = sum_s dS[t][s] k_s.
__global__ void __launch_bounds__(128) k_tr_attn_bwd_q(const float *d_ao, const float *att, const float *q,
                                                       const float *k, const float *v, float *dS,
                                                       float *d_q, int T, int nh, int nkv, int hd) {
    extern __shared__ float sm[];
    float *s_do = sm;         // [hd]
    float *s_dp = sm + hd;    // [T]
    __shared__ float s_dot;
    const int h = blockIdx.x, t = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarp = blockDim.x >> 5;
    const int D = nh * hd, K = nkv * hd, koff = (h / (nh / nkv)) * hd;
    const float scale = __fdiv_rn(1.0f, pt_sqrtf((float)hd));
    const float *P = att + ((size_t)h * T + t) * T;
    for (int d = threadIdx.x; d < hd; d += blockDim.x) s_do[d] = d_ao[(size_t)t * D + h * hd + d];
    __syncthreads();
    for (int s = threadIdx.x; s <= t; s += blockDim.x) {
        const float4 *vr = reinterpret_cast<const float4 *>(v + (size_t)s * K + koff);
        const float4 *d4p = reinterpret_cast<const float4 *>(s_do);
        float acc = 0.f;
        for (int d4 = 0; d4 < hd / 4; d4++) acc = dot4(__ldg(vr + d4), d4p[d4], acc);
        s_dp[s] = acc;
    }
    __syncthreads();
    if (warp == 0) {
        float dot = 0.f;
        for (int s = lane; s <= t; s += 32) dot = fmaf(s_dp[s], P[s], dot);
        dot = warp_sum(dot);
        if (lane == 0) s_dot = dot;
    }
    __syncthreads();
    float *dsr = dS + ((size_t)h * T + t) * T;
    for (int s = threadIdx.x; s < T; s += blockDim.x) {
        float x = 0.f;
        if (s <= t) x = __fmul_rn(__fmul_rn(P[s], __fsub_rn(s_dp[s], s_dot)), scale);
        dsr[s] = x;
        if (s <= t) s_dp[s] = x;
    }
    __syncthreads();
    __shared__ float s_part[4][64];
    float a0 = 0.f, a1 = 0.f;
    for (int s = warp; s <= t; s += nwarp) {
        const float x = s_dp[s];
        const float *kr = k + (size_t)s * K + koff;
        if (lane < hd) a0 = fmaf(x, kr[lane], a0);
        if (lane + 32 < hd) a1 = fmaf(x, kr[lane + 32], a1);
    }
    s_part[warp][lane] = a0;
    s_part[warp][lane + 32] = a1;
    __syncthreads();
    for (int d = threadIdx.x; d < hd; d += blockDim.x) {
        float acc = 0.f;
        for (int w = 0; w < nwarp; w++) acc += s_part[w][d];
        d_q[(size_t)t * D + h * hd + d] = acc;
    }
}

// Attention backward part 2, one CTA per (kv head, s): d_k[s] = sum_t dS[t][s] q_t,
// d_v[s] = sum_t P[t][s] d_ao_t over t in [s, n_rows) and the query heads of
// this kv head.
__global__ void __launch_bounds__(128) k_tr_attn_bwd_kv(const float *d_ao, const float *att, const float *q,
                                                        const float *dS, float *d_k, float *d_v, int T,
                                                        int n_rows, int nh, int nkv, int hd) {
    // warp w takes rows t = s + w (mod warps); lanes own columns lane and
    // lane + 32 (hd <= 64); partial sums are added in warp order
    const int kh = blockIdx.x, s = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarp = blockDim.x >> 5;
    const int D = nh * hd, K = nkv * hd, group = nh / nkv;
    __shared__ float s_k[4][64], s_v[4][64];
    float ak0 = 0.f, ak1 = 0.f, av0 = 0.f, av1 = 0.f;
    for (int hh = 0; hh < group; hh++) {
        const int h = kh * group + hh;
        for (int t = s + warp; t < n_rows; t += nwarp) {
            const size_t rowoff = ((size_t)h * T + t) * T + s;
            const float ds = dS[rowoff], p = att[rowoff];
            const float *qr = q + (size_t)t * D + h * hd, *dr = d_ao + (size_t)t * D + h * hd;
            if (lane < hd) {
                ak0 = fmaf(ds, qr[lane], ak0);
                av0 = fmaf(p, dr[lane], av0);
            }
            if (lane + 32 < hd) {
                ak1 = fmaf(ds, qr[lane + 32], ak1);
                av1 = fmaf(p, dr[lane + 32], av1);
            }
        }
    }
    s_k[warp][lane] = ak0;
    s_k[warp][lane + 32] = ak1;
    s_v[warp][lane] = av0;
    s_v[warp][lane + 32] = av1;
    __syncthreads();
    for (int d = threadIdx.x; d < hd; d += blockDim.x) {
        float ak = 0.f, av = 0.f;
        for (int w = 0; w < nwarp; w++) {
            ak += s_k[w][d];
            av += s_v[w][d];
        }
        d_k[(size_t)s * K + kh * hd + d] = ak;
        d_v[(size_t)s * K + kh * hd + d] = av;
    }
}

// RoPE backward (pt_backward_ops.c:52-69) into fresh d_qpre / d_kpre.
__global__ void k_tr_rope_bwd(float *dq_pre, float *dk_pre, const float *dq, const float *dk, int rows,
                              int D, int K, int hd) {
    const int half = D / 2;
    for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < rows * half; e += gridDim.x * blockDim.x) {
        const int t = e / half, i = 2 * (e % half);
        const float th = rope_theta(i, hd, t);
        const float c = pt_cosf(th), s = pt_sinf(th);
        const float *a = dq + (size_t)t * D + i;
        float *o = dq_pre + (size_t)t * D + i;
        o[0] = __fadd_rn(__fmul_rn(a[0], c), __fmul_rn(a[1], s));
        o[1] = __fadd_rn(__fmul_rn(-a[0], s), __fmul_rn(a[1], c));
        if (i < K) {
            const float *b = dk + (size_t)t * K + i;
            float *ok = dk_pre + (size_t)t * K + i;
            ok[0] = __fadd_rn(__fmul_rn(b[0], c), __fmul_rn(b[1], s));
            ok[1] = __fadd_rn(__fmul_rn(-b[0], s), __fmul_rn(b[1], c));
        }
    }
}

// g_emb[tokens[t]] += d_res[t] (pt_train.c:862-863); repeated tokens collide,
// hence atomics.
__global__ void k_tr_embed_bwd(float *g_emb, const float *d_res, const int *tokens, int rows, int D) {
    for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < rows * D; e += gridDim.x * blockDim.x) {
        const int t = e / D, i = e % D;
        atomicAdd(g_emb + (size_t)tokens[t] * D + i, d_res[e]);
    }
}

// w -= lr * g (pt_train.c:870-873)
__global__ void k_tr_sgd(float *w, const float *g, size_t n, float lr) {
    for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < n; e += (size_t)gridDim.x * blockDim.x)
        w[e] = __fsub_rn(w[e], __fmul_rn(lr, g[e]));
}

}  // namespace ptc

// ---------------------------------------------------------------------------
// Trainer object
// ---------------------------------------------------------------------------
// One microbatch's forward state: everything the backward of that microbatch
// reads. The trainer works on the selected set (its fields below mirror it).
struct ActSet {
    float *res, *res_att, *xb_att, *q, *k, *v, *att, *att_out, *xb_ffn, *hb, *hb2, *x_final, *logits;
    int *tokens;
    float *loss_rows, *loss;
    float *dres_save;   // this microbatch's d_res, kept across a pipeline schedule
    int T;
};
constexpr int PTC_MAX_MICROBATCHES = 16;

// Events of the second stream: forks after the producers of a product's
// inputs, joins after the products. Forward (ptc_trainer_fwd_layers): k / v
// beside q, w3 beside w1. Backward (ptc_trainer_bwd_layers): the weight
// gradients beside the input gradients.
enum { EV_FFN2, EV_FFN13, EV_WO, EV_QKV, EV_J_FFN2, EV_J_FFN13, EV_J_WO, EV_J_QKV,
       EV_F_KV, EV_F_W3, EV_J_F_KV, EV_J_F_W3, EV_J_X3, EV_J_XK, EV_J_XV, EV_RMS, EV_J_CS, EV_HEAD, EV_J_HEAD,
       N_EV };

struct ptc_trainer {
    ptc_ctx *ctx;
    cudaStream_t s;
    cudaStream_t s2;      // independent products beside those on s
    cudaStream_t s3;      // the backward's second and third input-gradient products
    cudaEvent_t ev[N_EV];
    int n_sm;
    int D, H, L, nh, nkv, V, seq, hd, K, maxT, T;
    int has_embed, has_head;
    ptc_weights w;  // device weights (mutable through casts)
    // activations
    float *res, *res_att, *xb_att, *q, *k, *v, *att, *att_out, *xb_ffn, *hb, *hb2, *x_final, *logits;
    // backward
    float *d_res, *d_aout, *d_q, *d_k, *d_v, *d_logit, *d_xb, *d_hid, *d_hid2, *sh, *dS, *d_qpre,
        *d_kpre, *dw_rows, *partial;
    float *partial2;      // split-K workspace of the second stream
    float *partial3;      // ... and of the third
    float *d_xb2, *d_xb3; // the input-gradient products computed beside d_xb
    size_t partial_cap;
    int *tokens;
    float *loss_rows, *loss;
    float *loss_host;  // pinned
    // gradients (pt_train.c:334-371 layout, absent parts empty)
    float *g_mem;
    size_t n_params;
    float *g_emb, *g_rms_att, *g_wq, *g_wk, *g_wv, *g_wo, *g_rms_ffn, *g_w1, *g_w2, *g_w3, *g_rms_final,
        *g_wcls;
    // microbatch activation sets (set 0 = the buffers above at creation)
    ActSet sets[PTC_MAX_MICROBATCHES];
    int n_sets, cur;
};

static void save_set(ptc_trainer *tr, int i) {
    ActSet &a = tr->sets[i];
    a.res = tr->res; a.res_att = tr->res_att; a.xb_att = tr->xb_att; a.q = tr->q; a.k = tr->k; a.v = tr->v;
    a.att = tr->att; a.att_out = tr->att_out; a.xb_ffn = tr->xb_ffn; a.hb = tr->hb; a.hb2 = tr->hb2;
    a.x_final = tr->x_final; a.logits = tr->logits; a.tokens = tr->tokens; a.loss_rows = tr->loss_rows;
    a.loss = tr->loss; a.T = tr->T;
}
static void load_set(ptc_trainer *tr, int i) {
    const ActSet &a = tr->sets[i];
    tr->res = a.res; tr->res_att = a.res_att; tr->xb_att = a.xb_att; tr->q = a.q; tr->k = a.k; tr->v = a.v;
    tr->att = a.att; tr->att_out = a.att_out; tr->xb_ffn = a.xb_ffn; tr->hb = a.hb; tr->hb2 = a.hb2;
    tr->x_final = a.x_final; tr->logits = a.logits; tr->tokens = a.tokens; tr->loss_rows = a.loss_rows;
    tr->loss = a.loss; tr->T = a.T;
}

// Every pass needs the selected activation set's sequence length. A set that
// has had neither tokens nor a length (ptc_trainer_set_tokens /
// ptc_trainer_set_T) has T = 0, and its kernels would index row T - 1 = -1:
// refuse on the host instead. (A pipeline schedule's layer rank selecting
// microbatch 1 without giving it a length did exactly that.)
static void require_T(const ptc_trainer *tr, const char *pass) {
    if (tr->T < 2 || tr->T > tr->maxT)
        PTC_FATAL("%s on microbatch set %d with T=%d: set the tokens or the length first (max_T=%d)", pass, tr->cur,
                  tr->T, tr->maxT);
}

static int blocks_for(size_t n, int threads, int n_sm) {
    size_t b = (n + threads - 1) / threads;
    size_t cap = (size_t)n_sm * 8;
    return (int)(b < 1 ? 1 : (b > cap ? cap : b));
}

extern "C" ptc_trainer *ptc_trainer_create(ptc_ctx *c, const ptc_config *cfg, const ptc_weights *w,
                                           int max_T, int has_embed, int has_head) {
    ptc_trainer *tr = new ptc_trainer();
    memset(tr, 0, sizeof(*tr));
    tr->ctx = c;
    PTC_CHECK(cudaSetDevice(ptc_device(c)));
    tr->s = ptc_ctx_stream(c);
    PTC_CHECK(cudaStreamCreateWithFlags(&tr->s2, cudaStreamNonBlocking));
    PTC_CHECK(cudaStreamCreateWithFlags(&tr->s3, cudaStreamNonBlocking));
    for (int i = 0; i < N_EV; i++) PTC_CHECK(cudaEventCreateWithFlags(&tr->ev[i], cudaEventDisableTiming));
    tr->n_sm = ptc_sm_count(c);
    tr->D = cfg->dim;
    tr->H = cfg->hidden_dim;
    tr->L = cfg->n_layers;
    tr->nh = cfg->n_heads;
    tr->nkv = cfg->n_kv_heads;
    tr->V = cfg->vocab_size;
    tr->seq = cfg->seq_len;
    tr->hd = tr->D / tr->nh;
    tr->K = tr->nkv * tr->hd;
    tr->maxT = max_T;
    tr->has_embed = has_embed;
    tr->has_head = has_head;
    tr->w = *w;
    if (max_T < 2) PTC_FATAL("training needs max_T >= 2 (got %d)", max_T);
    if (tr->D % 2 || tr->hd % 2) PTC_FATAL("training needs even dim and head_dim");
    if (tr->hd > 64 || tr->hd % 4) PTC_FATAL("training attention supports head_dim <= 64, a multiple of 4 (got %d)", tr->hd);

    const size_t T = max_T, D = tr->D, H = tr->H, L = tr->L, K = tr->K, V = tr->V, nh = tr->nh;
    auto A = [&](size_t n) { return (float *)ptc_alloc(c, (n ? n : 1) * 4); };
    tr->res = A((L + 1) * T * D);
    tr->res_att = A(L * T * D);
    tr->xb_att = A(L * T * D);
    tr->q = A(L * T * D);
    tr->k = A(L * T * K);
    tr->v = A(L * T * K);
    tr->att = A(L * nh * T * T);
    tr->att_out = A(L * T * D);
    tr->xb_ffn = A(L * T * D);
    tr->hb = A(L * T * H);
    tr->hb2 = A(L * T * H);
    tr->x_final = A(T * D);
    tr->logits = has_head ? A(T * V) : nullptr;
    tr->d_res = A(T * D);
    tr->d_aout = A(T * D);
    tr->d_q = A(T * D);
    tr->d_k = A(T * K);
    tr->d_v = A(T * K);
    tr->d_logit = has_head ? A(T * V) : nullptr;
    tr->d_xb = A(T * D);
    tr->d_hid = A(T * H);
    tr->d_hid2 = A(T * H);
    tr->sh = A(T * H);
    tr->dS = A(nh * T * T);
    tr->d_qpre = A(T * D);
    tr->d_kpre = A(T * K);
    tr->dw_rows = A(T * D);
    tr->partial_cap = 8 * T * (D > H ? D : H);
    tr->partial = A(tr->partial_cap);
    tr->partial2 = A(tr->partial_cap);
    tr->partial3 = A(tr->partial_cap);
    tr->d_xb2 = A(T * D);
    tr->d_xb3 = A(T * D);
    tr->tokens = (int *)ptc_alloc(c, T * 4);
    tr->loss_rows = A(3 * T);   // loss per row, then the rows' max and exponential sum
    tr->loss = A(1);
    tr->loss_host = (float *)ptc_host_alloc(4);

    // gradient layout of pt_train.c:334-371 for the owned parts
    const size_t Ve = has_embed ? V : 0;
    size_t n = Ve * D + L * D + L * D * D + 2 * L * K * D + L * D * D + L * D + 3 * L * H * D +
               (has_head ? D : 0);
    const bool untied = has_head && w->wcls && w->wcls != w->token_embedding;
    if (untied) n += V * D;
    tr->n_params = n;
    tr->g_mem = A(n);
    float *p = tr->g_mem;
    tr->g_emb = has_embed ? p : nullptr; p += Ve * D;
    tr->g_rms_att = p; p += L * D;
    tr->g_wq = p; p += L * D * D;
    tr->g_wk = p; p += L * K * D;
    tr->g_wv = p; p += L * K * D;
    tr->g_wo = p; p += L * D * D;
    tr->g_rms_ffn = p; p += L * D;
    tr->g_w1 = p; p += L * H * D;
    tr->g_w2 = p; p += L * D * H;
    tr->g_w3 = p; p += L * H * D;
    tr->g_rms_final = has_head ? p : nullptr; p += has_head ? D : 0;
    tr->g_wcls = untied ? p : (has_head ? tr->g_emb : nullptr);
    if (has_head && !untied && !has_embed) PTC_FATAL("tied classifier needs the embedding on the same rank");
    PTC_CHECK(cudaMemsetAsync(tr->g_mem, 0, n * 4, tr->s));
    PTC_CHECK(cudaStreamSynchronize(tr->s));
    tr->n_sets = 1;
    tr->cur = 0;
    save_set(tr, 0);
    tr->sets[0].dres_save = A(T * D);
    return tr;
}

extern "C" void ptc_trainer_destroy(ptc_trainer *tr) {
    if (!tr) return;
    cudaStreamSynchronize(tr->s);
    cudaStreamSynchronize(tr->s2);
    cudaStreamSynchronize(tr->s3);
    for (int i = 0; i < N_EV; i++) cudaEventDestroy(tr->ev[i]);
    cudaStreamDestroy(tr->s2);
    cudaStreamDestroy(tr->s3);
    ptc_host_free(tr->loss_host);
    delete tr;
}

extern "C" size_t ptc_trainer_n_params(ptc_trainer *tr) { return tr->n_params; }
extern "C" float *ptc_trainer_grads(ptc_trainer *tr) { return tr->g_mem; }
extern "C" float *ptc_trainer_residual(ptc_trainer *tr, int l) {
    return tr->res + (size_t)l * tr->T * tr->D;
}
extern "C" float *ptc_trainer_dres(ptc_trainer *tr) { return tr->d_res; }

// Microbatch activation sets for pipeline schedules: n sets in all (set 0
// exists from creation), each a full copy of the forward state for max_T
// tokens. Selecting a set makes the forward/backward calls use it.
extern "C" void ptc_trainer_set_microbatches(ptc_trainer *tr, int n) {
    if (n < 1 || n > PTC_MAX_MICROBATCHES) PTC_FATAL("microbatches %d outside [1, %d]", n, PTC_MAX_MICROBATCHES);
    save_set(tr, tr->cur);
    const size_t T = tr->maxT, D = tr->D, H = tr->H, L = tr->L, K = tr->K, V = tr->V, nh = tr->nh;
    auto A = [&](size_t e) { return (float *)ptc_alloc(tr->ctx, (e ? e : 1) * 4); };
    for (int i = tr->n_sets; i < n; i++) {
        ActSet &a = tr->sets[i];
        a.res = A((L + 1) * T * D);
        a.res_att = A(L * T * D);
        a.xb_att = A(L * T * D);
        a.q = A(L * T * D);
        a.k = A(L * T * K);
        a.v = A(L * T * K);
        a.att = A(L * nh * T * T);
        a.att_out = A(L * T * D);
        a.xb_ffn = A(L * T * D);
        a.hb = A(L * T * H);
        a.hb2 = A(L * T * H);
        a.x_final = A(T * D);
        a.logits = tr->has_head ? A(T * V) : nullptr;
        a.tokens = (int *)ptc_alloc(tr->ctx, T * 4);
        a.loss_rows = A(3 * T);
        a.loss = A(1);
        a.dres_save = A(T * D);
        a.T = 0;   // no length until its tokens or length are set
    }
    if (n > tr->n_sets) tr->n_sets = n;
}

extern "C" void ptc_trainer_select(ptc_trainer *tr, int m) {
    if (m < 0 || m >= tr->n_sets) PTC_FATAL("microbatch %d outside [0, %d)", m, tr->n_sets);
    if (m == tr->cur) return;
    save_set(tr, tr->cur);
    load_set(tr, m);
    tr->cur = m;
}

// The selected microbatch's d_res keeping buffer ([T, dim]).
extern "C" float *ptc_trainer_dres_save(ptc_trainer *tr) { return tr->sets[tr->cur].dres_save; }

static GemmArgs G(int M, int N, int K, const float *A, int lda, bool akc, const float *B, int ldb, bool bkc,
                  float *C, int ldc, int epi) {
    GemmArgs g;
    memset(&g, 0, sizeof(g));
    g.M = M; g.N = N; g.K = K;
    g.A = A; g.lda = lda; g.a_kcontig = akc;
    g.B = B; g.ldb = ldb; g.b_kcontig = bkc;
    g.C = C; g.ldc = ldc; g.epi = epi;
    return g;
}

static void run_gemm(ptc_trainer *tr, GemmArgs g) {
    g.partial = tr->partial;
    g.partial_cap = tr->partial_cap;
    ptc::gemm(g, tr->n_sm, tr->s);
}

// A weight-gradient product on the second stream, with its own split-K
// workspace; kept on the SIMT kernel (no_alloc), whose launches own no state
// that a product on the first stream could share.
static void run_gemm2(ptc_trainer *tr, GemmArgs g) {
    g.partial = tr->partial2;
    g.partial_cap = tr->partial_cap;
    g.no_alloc = 1;
    ptc::gemm(g, tr->n_sm, tr->s2);
}

// The same on the third stream (its own workspace).
static void run_gemm3(ptc_trainer *tr, GemmArgs g) {
    g.partial = tr->partial3;
    g.partial_cap = tr->partial_cap;
    g.no_alloc = 1;
    ptc::gemm(g, tr->n_sm, tr->s3);
}

static void fork_to_s2(ptc_trainer *tr, int e) {
    PTC_CHECK(cudaEventRecord(tr->ev[e], tr->s));
    PTC_CHECK(cudaStreamWaitEvent(tr->s2, tr->ev[e], 0));
}
static void mark_s2(ptc_trainer *tr, int e) { PTC_CHECK(cudaEventRecord(tr->ev[e], tr->s2)); }
static void join_s2(ptc_trainer *tr, int e) { PTC_CHECK(cudaStreamWaitEvent(tr->s, tr->ev[e], 0)); }

extern "C" void ptc_trainer_set_tokens(ptc_trainer *tr, const int *tokens, int T) {
    if (T < 2 || T > tr->maxT) PTC_FATAL("T=%d outside [2, max_T=%d]", T, tr->maxT);
    if (T > tr->seq) PTC_FATAL("T=%d exceeds seq_len %d", T, tr->seq);
    for (int t = 0; t < T; t++)
        if (tokens[t] < 0 || tokens[t] >= tr->V) PTC_FATAL("token %d outside [0, %d)", tokens[t], tr->V);
    tr->T = T;
    PTC_CHECK(cudaMemcpyAsync(tr->tokens, tokens, (size_t)T * 4, cudaMemcpyHostToDevice, tr->s));
}

extern "C" void ptc_trainer_set_T(ptc_trainer *tr, int T) {
    if (T < 2 || T > tr->maxT) PTC_FATAL("T=%d outside [2, max_T=%d]", T, tr->maxT);
    if (T > tr->seq) PTC_FATAL("T=%d exceeds seq_len %d", T, tr->seq);
    tr->T = T;
}

extern "C" void ptc_trainer_zero_grads(ptc_trainer *tr) {
    PTC_CHECK(cudaMemsetAsync(tr->g_mem, 0, tr->n_params * 4, tr->s));
}

// pt_forward_train_embed (pt_train.c:946-952)
extern "C" void ptc_trainer_fwd_embed(ptc_trainer *tr) {
    if (!tr->has_embed) PTC_FATAL("trainer has no embedding");
    require_T(tr, "forward embedding");
    const int n = tr->T * tr->D;
    ptc::k_tr_embed<<<blocks_for(n, 256, tr->n_sm), 256, 0, tr->s>>>(tr->res, tr->w.token_embedding,
                                                                       tr->tokens, tr->T, tr->D);
    PTC_CHECK(cudaGetLastError());
}

// pt_forward_train_layers_range (pt_train.c:954-1061)
// The row-block attention kernels need T <= TB_T, whole float4 head rows and
// their shared-memory staging within a CTA's limit; otherwise the per-row
// kernels run.
static bool attn_blocked(ptc_trainer *tr, int T) {
    if (T > ptc::TB_T || tr->hd % 4 || tr->hd > 64) return false;
    const size_t smem = ptc::attn_block_smem(T, tr->hd);
    if (smem > 200 * 1024) return false;
    ptc::ensure_kernel_smem((const void *)ptc::k_tr_attn_fwd_blk, smem);
    ptc::ensure_kernel_smem((const void *)ptc::k_tr_attn_bwd_q_blk, smem);
    return true;
}

extern "C" void ptc_trainer_fwd_layers(ptc_trainer *tr, int l0, int l1) {
    require_T(tr, "forward layers");
    if (l0 < 0 || l1 > tr->L || l0 > l1) PTC_FATAL("layer range [%d, %d) outside [0, %d)", l0, l1, tr->L);
    const int T = tr->T, D = tr->D, H = tr->H, K = tr->K, nh = tr->nh;
    cudaStream_t s = tr->s;
    for (int l = l0; l < l1; l++) {
        const size_t LD = (size_t)l * T * D, LK = (size_t)l * T * K, LH = (size_t)l * T * H;
        float *rin = tr->res + LD, *rmid = tr->res_att + LD, *rout = tr->res + (size_t)(l + 1) * T * D;
        float *xa = tr->xb_att + LD, *xf = tr->xb_ffn + LD;
        ptc::k_tr_rmsnorm<<<(T + 7) / 8, 256, 0, s>>>(xa, rin, tr->w.rms_att_weight + (size_t)l * D, T, D);
        // k and v on the second stream beside q (all read xa)
        fork_to_s2(tr, EV_F_KV);
        GemmArgs g = G(T, K, D, xa, D, true, tr->w.wk + (size_t)l * K * D, D, true, tr->k + LK, K, ptc::EPI_ROPE);
        g.rope_hd = tr->hd;
        run_gemm2(tr, g);
        run_gemm2(tr, G(T, K, D, xa, D, true, tr->w.wv + (size_t)l * K * D, D, true, tr->v + LK, K, ptc::EPI_STORE));
        mark_s2(tr, EV_J_F_KV);
        g = G(T, D, D, xa, D, true, tr->w.wq + (size_t)l * D * D, D, true, tr->q + LD, D, ptc::EPI_ROPE);
        g.rope_hd = tr->hd;
        run_gemm(tr, g);
        join_s2(tr, EV_J_F_KV);
        if (attn_blocked(tr, T)) {
            ptc::k_tr_attn_fwd_blk<<<dim3(nh, (T + ptc::TB_R - 1) / ptc::TB_R), ptc::TB_R * 32,
                                     ptc::attn_block_smem(T, tr->hd), s>>>(
                tr->q + LD, tr->k + LK, tr->v + LK, tr->att + (size_t)l * nh * T * T, tr->att_out + LD, T, nh,
                tr->nkv, tr->hd);
        } else {
            const size_t smem = (size_t)(tr->hd + T) * 4;
            ptc::k_tr_attn_fwd<<<dim3(nh, T), 128, smem, s>>>(tr->q + LD, tr->k + LK, tr->v + LK,
                                                              tr->att + (size_t)l * nh * T * T, tr->att_out + LD,
                                                              T, nh, tr->nkv, tr->hd);
        }
        PTC_CHECK(cudaGetLastError());
        g = G(T, D, D, tr->att_out + LD, D, true, tr->w.wo + (size_t)l * D * D, D, true, rmid, D, ptc::EPI_RESID);
        g.R = rin;
        g.ldr = D;
        run_gemm(tr, g);
        ptc::k_tr_rmsnorm<<<(T + 7) / 8, 256, 0, s>>>(xf, rmid, tr->w.rms_ffn_weight + (size_t)l * D, T, D);
        // w3 on the second stream beside w1 (both read xf)
        fork_to_s2(tr, EV_F_W3);
        run_gemm2(tr, G(T, H, D, xf, D, true, tr->w.w3 + (size_t)l * H * D, D, true, tr->hb2 + LH, H, ptc::EPI_STORE));
        mark_s2(tr, EV_J_F_W3);
        run_gemm(tr, G(T, H, D, xf, D, true, tr->w.w1 + (size_t)l * H * D, D, true, tr->hb + LH, H, ptc::EPI_STORE));
        join_s2(tr, EV_J_F_W3);
        ptc::k_tr_silu_gate<<<blocks_for((size_t)T * H, 256, tr->n_sm), 256, 0, s>>>(tr->sh, tr->hb + LH,
                                                                                      tr->hb2 + LH, (size_t)T * H);
        g = G(T, D, H, tr->sh, H, true, tr->w.w2 + (size_t)l * D * H, H, true, rout, D, ptc::EPI_RESID);
        g.R = rmid;
        g.ldr = D;
        run_gemm(tr, g);
    }
    PTC_CHECK(cudaGetLastError());
}

// pt_forward_train_head (pt_train.c:1063-1099): returns the loss (synchronises).
// Head forward with the loss copied to pinned memory asynchronously: the
// caller reads tr->loss_host after synchronising the stream.
static void fwd_head_enqueue(ptc_trainer *tr) {
    if (!tr->has_head) PTC_FATAL("trainer has no head");
    const int T = tr->T, D = tr->D, V = tr->V;
    cudaStream_t s = tr->s;
    const float *rfin = tr->res + (size_t)tr->L * T * D;
    ptc::k_tr_rmsnorm<<<(T + 7) / 8, 256, 0, s>>>(tr->x_final, rfin, tr->w.rms_final_weight, T, D);
    run_gemm(tr, G(T, V, D, tr->x_final, D, true, tr->w.wcls, D, true, tr->logits, V, ptc::EPI_STORE));
    ptc::k_tr_ce_rows<<<T - 1, 512, 0, s>>>(tr->logits, tr->tokens, V, tr->loss_rows, tr->loss_rows + tr->maxT,
                                            tr->loss_rows + 2 * (size_t)tr->maxT);
    ptc::k_tr_loss_sum<<<1, 32, 0, s>>>(tr->loss_rows, T - 1, tr->loss);
    PTC_CHECK(cudaGetLastError());
    PTC_CHECK(cudaMemcpyAsync(tr->loss_host, tr->loss, 4, cudaMemcpyDeviceToHost, s));
}

extern "C" float ptc_trainer_fwd_head(ptc_trainer *tr) {
    require_T(tr, "forward head");
    fwd_head_enqueue(tr);
    PTC_CHECK(cudaStreamSynchronize(tr->s));
    return *tr->loss_host;
}

// pt_backward_head (pt_train.c:1103-1171)
extern "C" void ptc_trainer_bwd_head(ptc_trainer *tr) {
    require_T(tr, "backward head");
    const int T = tr->T, D = tr->D, V = tr->V, n = T - 1;
    cudaStream_t s = tr->s;
    PTC_CHECK(cudaMemsetAsync(tr->d_res, 0, (size_t)T * D * 4, s));
    const float invn = 1.0f / (float)(T - 1);
    ptc::k_tr_ce_backward<<<n, 512, 0, s>>>(tr->logits, tr->tokens, V, invn, tr->loss_rows + tr->maxT,
                                            tr->loss_rows + 2 * (size_t)tr->maxT, tr->d_logit);
    // dWcls += d_logit^T . x_final   [V x D], K = n -- on the second stream
    // (its own split-K and tensor-core workspaces), beside the input gradient
    fork_to_s2(tr, EV_HEAD);
    {
        GemmArgs g = G(V, D, n, tr->d_logit, V, false, tr->x_final, D, false, tr->g_wcls, D, ptc::EPI_ACCUM);
        g.partial = tr->partial2;
        g.partial_cap = tr->partial_cap;
        ptc::gemm(g, tr->n_sm, tr->s2);
    }
    mark_s2(tr, EV_J_HEAD);
    // d_xb = d_logit . Wcls   [n x D], K = V
    run_gemm(tr, G(n, D, V, tr->d_logit, V, true, tr->w.wcls, D, false, tr->d_xb, D, ptc::EPI_STORE));
    const float *rfin = tr->res + (size_t)tr->L * T * D;
    ptc::k_tr_rmsnorm_bwd<<<(n + 7) / 8, 256, 0, s>>>(tr->d_res, tr->dw_rows, tr->d_xb, nullptr, nullptr, rfin,
                                                      tr->w.rms_final_weight, n, D);
    ptc::k_tr_colsum_accum<<<(D + 31) / 32, 256, 0, s>>>(tr->g_rms_final, tr->dw_rows, n, D);
    join_s2(tr, EV_J_HEAD);   // the classifier gradient (tied: the embedding's) is complete
    PTC_CHECK(cudaGetLastError());
}

// pt_backward_layers_range (pt_train.c:1173-1377)
extern "C" void ptc_trainer_bwd_layers(ptc_trainer *tr, int l0, int l1) {
    require_T(tr, "backward layers");
    if (l0 < 0 || l1 > tr->L || l0 > l1) PTC_FATAL("layer range [%d, %d) outside [0, %d)", l0, l1, tr->L);
    const int T = tr->T, D = tr->D, H = tr->H, K = tr->K, nh = tr->nh, n = T - 1;
    cudaStream_t s = tr->s;
    for (int l = l1 - 1; l >= l0; l--) {
        const size_t LD = (size_t)l * T * D, LK = (size_t)l * T * K, LH = (size_t)l * T * H;
        const float *W1 = tr->w.w1 + (size_t)l * H * D, *W2 = tr->w.w2 + (size_t)l * D * H;
        const float *W3 = tr->w.w3 + (size_t)l * H * D, *Wo = tr->w.wo + (size_t)l * D * D;
        const float *Wq = tr->w.wq + (size_t)l * D * D, *Wk = tr->w.wk + (size_t)l * K * D;
        const float *Wv = tr->w.wv + (size_t)l * K * D;
        // FFN. sh is the previous layer's g_w2 input: that product has been
        // joined before this layer's first write of d_res' successor below
        ptc::k_tr_silu_gate<<<blocks_for((size_t)n * H, 256, tr->n_sm), 256, 0, s>>>(tr->sh, tr->hb + LH,
                                                                                      tr->hb2 + LH, (size_t)n * H);
        fork_to_s2(tr, EV_FFN2);   // d_res, sh ready
        run_gemm2(tr, G(D, H, n, tr->d_res, D, false, tr->sh, H, false, tr->g_w2 + (size_t)l * D * H, H,
                        ptc::EPI_ACCUM));
        mark_s2(tr, EV_J_FFN2);
        join_s2(tr, EV_J_FFN13);   // the previous layer's g_w1 / g_w3 read d_hid, d_hid2
        run_gemm(tr, G(n, H, D, tr->d_res, D, true, W2, H, false, tr->d_hid, H, ptc::EPI_STORE));
        ptc::k_tr_silu_bwd<<<blocks_for((size_t)n * H, 256, tr->n_sm), 256, 0, s>>>(
            tr->d_hid, tr->d_hid2, tr->hb + LH, tr->hb2 + LH, (size_t)n * H);
        fork_to_s2(tr, EV_FFN13);   // d_hid, d_hid2 ready
        run_gemm2(tr, G(H, D, n, tr->d_hid, H, false, tr->xb_ffn + LD, D, false, tr->g_w1 + (size_t)l * H * D, D,
                        ptc::EPI_ACCUM));
        run_gemm2(tr, G(H, D, n, tr->d_hid2, H, false, tr->xb_ffn + LD, D, false, tr->g_w3 + (size_t)l * H * D, D,
                        ptc::EPI_ACCUM));
        mark_s2(tr, EV_J_FFN13);
        // d_xb = d_hid.W1 + d_hid2.W3: the second product on the third stream
        // into its own buffer, summed in the rmsnorm backward
        PTC_CHECK(cudaStreamWaitEvent(tr->s3, tr->ev[EV_FFN13], 0));
        run_gemm3(tr, G(n, D, H, tr->d_hid2, H, true, W3, D, false, tr->d_xb2, D, ptc::EPI_STORE));
        PTC_CHECK(cudaEventRecord(tr->ev[EV_J_X3], tr->s3));
        run_gemm(tr, G(n, D, H, tr->d_hid, H, true, W1, D, false, tr->d_xb, D, ptc::EPI_STORE));
        join_s2(tr, EV_J_FFN2);   // g_w2 has read d_res (and sh)
        join_s2(tr, EV_J_X3);
        ptc::k_tr_rmsnorm_bwd<<<(n + 7) / 8, 256, 0, s>>>(tr->d_res, tr->dw_rows, tr->d_xb, tr->d_xb2, nullptr,
                                                          tr->res_att + LD, tr->w.rms_ffn_weight + (size_t)l * D, n, D);
        // the gain's column sums on the third stream (dw_rows is next written
        // by the attention half's rmsnorm backward, after the join of that
        // stream's k product, which follows them)
        PTC_CHECK(cudaEventRecord(tr->ev[EV_RMS], s));
        PTC_CHECK(cudaStreamWaitEvent(tr->s3, tr->ev[EV_RMS], 0));
        ptc::k_tr_colsum_accum<<<(D + 31) / 32, 256, 0, tr->s3>>>(tr->g_rms_ffn + (size_t)l * D, tr->dw_rows, n, D);
        // wo
        fork_to_s2(tr, EV_WO);   // d_res of the attention half ready
        run_gemm2(tr, G(D, D, n, tr->d_res, D, false, tr->att_out + LD, D, false, tr->g_wo + (size_t)l * D * D, D,
                        ptc::EPI_ACCUM));
        mark_s2(tr, EV_J_WO);
        run_gemm(tr, G(n, D, D, tr->d_res, D, true, Wo, D, false, tr->d_aout, D, ptc::EPI_STORE));
        // attention (d_q, d_k, d_v, d_qpre, d_kpre are the previous layer's
        // g_wq / g_wk / g_wv inputs)
        join_s2(tr, EV_J_QKV);
        const float *att_l = tr->att + (size_t)l * nh * T * T;
        if (attn_blocked(tr, T)) {
            ptc::k_tr_attn_bwd_q_blk<<<dim3(nh, (n + ptc::TB_R - 1) / ptc::TB_R), ptc::TB_R * 32,
                                       ptc::attn_block_smem(T, tr->hd), s>>>(
                tr->d_aout, att_l, tr->k + LK, tr->v + LK, tr->dS, tr->d_q, T, n, nh, tr->nkv, tr->hd);
        } else {
            const size_t smem = (size_t)(tr->hd + T) * 4;
            ptc::k_tr_attn_bwd_q<<<dim3(nh, n), 128, smem, s>>>(tr->d_aout, att_l, tr->q + LD, tr->k + LK,
                                                                tr->v + LK, tr->dS, tr->d_q, T, nh, tr->nkv, tr->hd);
        }
        ptc::k_tr_attn_bwd_kv<<<dim3(tr->nkv, n), 128, 0, s>>>(tr->d_aout, att_l, tr->q + LD, tr->dS, tr->d_k,
                                                              tr->d_v, T, n, nh, tr->nkv, tr->hd);
        ptc::k_tr_rope_bwd<<<blocks_for((size_t)n * D / 2, 256, tr->n_sm), 256, 0, s>>>(
            tr->d_qpre, tr->d_kpre, tr->d_q, tr->d_k, n, D, K, tr->hd);
        const float *xa = tr->xb_att + LD;
        // d_xb = d_qpre.Wq + d_kpre.Wk + d_v.Wv: the k product on the third
        // stream, the v product first on the second (then its weight
        // gradients), each into its own buffer, summed in the rmsnorm backward
        fork_to_s2(tr, EV_QKV);   // d_qpre, d_kpre, d_v ready
        PTC_CHECK(cudaStreamWaitEvent(tr->s3, tr->ev[EV_QKV], 0));
        run_gemm3(tr, G(n, D, K, tr->d_kpre, K, true, Wk, D, false, tr->d_xb2, D, ptc::EPI_STORE));
        PTC_CHECK(cudaEventRecord(tr->ev[EV_J_XK], tr->s3));
        run_gemm2(tr, G(n, D, K, tr->d_v, K, true, Wv, D, false, tr->d_xb3, D, ptc::EPI_STORE));
        mark_s2(tr, EV_J_XV);
        run_gemm2(tr, G(D, D, n, tr->d_qpre, D, false, xa, D, false, tr->g_wq + (size_t)l * D * D, D, ptc::EPI_ACCUM));
        run_gemm2(tr, G(K, D, n, tr->d_kpre, K, false, xa, D, false, tr->g_wk + (size_t)l * K * D, D, ptc::EPI_ACCUM));
        run_gemm2(tr, G(K, D, n, tr->d_v, K, false, xa, D, false, tr->g_wv + (size_t)l * K * D, D, ptc::EPI_ACCUM));
        mark_s2(tr, EV_J_QKV);
        run_gemm(tr, G(n, D, D, tr->d_qpre, D, true, Wq, D, false, tr->d_xb, D, ptc::EPI_STORE));
        join_s2(tr, EV_J_WO);   // g_wo has read d_res
        join_s2(tr, EV_J_XK);
        join_s2(tr, EV_J_XV);
        ptc::k_tr_rmsnorm_bwd<<<(n + 7) / 8, 256, 0, s>>>(tr->d_res, tr->dw_rows, tr->d_xb, tr->d_xb2, tr->d_xb3,
                                                          tr->res + LD, tr->w.rms_att_weight + (size_t)l * D, n, D);
        // (dw_rows is next written by the next layer's FFN rmsnorm backward,
        // after the join of the third stream's d_hid2.W3 product)
        PTC_CHECK(cudaEventRecord(tr->ev[EV_RMS], s));
        PTC_CHECK(cudaStreamWaitEvent(tr->s3, tr->ev[EV_RMS], 0));
        ptc::k_tr_colsum_accum<<<(D + 31) / 32, 256, 0, tr->s3>>>(tr->g_rms_att + (size_t)l * D, tr->dw_rows, n, D);
        PTC_CHECK(cudaEventRecord(tr->ev[EV_J_CS], tr->s3));
    }
    // every weight-gradient product done before anything after the pass
    join_s2(tr, EV_J_FFN13);
    join_s2(tr, EV_J_QKV);
    join_s2(tr, EV_J_CS);
    PTC_CHECK(cudaGetLastError());
}

// pt_backward_embed (pt_train.c:1379-1383)
extern "C" void ptc_trainer_bwd_embed(ptc_trainer *tr) {
    if (!tr->has_embed) PTC_FATAL("trainer has no embedding");
    require_T(tr, "backward embedding");
    const int n = tr->T - 1;
    ptc::k_tr_embed_bwd<<<blocks_for((size_t)n * tr->D, 256, tr->n_sm), 256, 0, tr->s>>>(
        tr->g_emb, tr->d_res, tr->tokens, n, tr->D);
    PTC_CHECK(cudaGetLastError());
}

static void sgd_range(ptc_trainer *tr, const float *w, const float *g, size_t n, float lr) {
    if (!n || !w || !g) return;
    ptc::k_tr_sgd<<<blocks_for(n, 256, tr->n_sm), 256, 0, tr->s>>>((float *)w, g, n, lr);
}

// pt_sgd_update_layers (pt_train.c:902-929)
extern "C" void ptc_trainer_sgd_layers(ptc_trainer *tr, float lr, int l0, int l1) {
    const size_t D = tr->D, H = tr->H, K = tr->K, n = (size_t)(l1 - l0);
    if (n == 0) return;
    sgd_range(tr, tr->w.rms_att_weight + l0 * D, tr->g_rms_att + l0 * D, n * D, lr);
    sgd_range(tr, tr->w.wq + l0 * D * D, tr->g_wq + l0 * D * D, n * D * D, lr);
    sgd_range(tr, tr->w.wk + l0 * K * D, tr->g_wk + l0 * K * D, n * K * D, lr);
    sgd_range(tr, tr->w.wv + l0 * K * D, tr->g_wv + l0 * K * D, n * K * D, lr);
    sgd_range(tr, tr->w.wo + l0 * D * D, tr->g_wo + l0 * D * D, n * D * D, lr);
    sgd_range(tr, tr->w.rms_ffn_weight + l0 * D, tr->g_rms_ffn + l0 * D, n * D, lr);
    sgd_range(tr, tr->w.w1 + l0 * H * D, tr->g_w1 + l0 * H * D, n * H * D, lr);
    sgd_range(tr, tr->w.w2 + l0 * D * H, tr->g_w2 + l0 * D * H, n * D * H, lr);
    sgd_range(tr, tr->w.w3 + l0 * H * D, tr->g_w3 + l0 * H * D, n * H * D, lr);
    PTC_CHECK(cudaGetLastError());
}

// pt_sgd_update_head (pt_train.c:935-942)
extern "C" void ptc_trainer_sgd_head(ptc_trainer *tr, float lr) {
    const size_t D = tr->D, V = tr->V;
    if (tr->has_embed) sgd_range(tr, tr->w.token_embedding, tr->g_emb, V * D, lr);
    if (tr->has_head) {
        sgd_range(tr, tr->w.rms_final_weight, tr->g_rms_final, D, lr);
        if (tr->g_wcls && tr->g_wcls != tr->g_emb) sgd_range(tr, tr->w.wcls, tr->g_wcls, V * D, lr);
    }
    PTC_CHECK(cudaGetLastError());
}

// pt_sgd_update over every parameter (pt_train.c:875-896). When the weights
// sit in device memory in the order and spacing of the gradient buffer (the
// uploaded .bin image: embedding, per-layer tensors, final norm), one launch
// covers all of them instead of one per tensor.
static void sgd_all(ptc_trainer *tr, float lr) {
    const float *w0 = tr->w.token_embedding, *g0 = tr->g_emb;
    const float *pw[] = {tr->w.rms_att_weight, tr->w.wq, tr->w.wk, tr->w.wv, tr->w.wo, tr->w.rms_ffn_weight,
                         tr->w.w1, tr->w.w2, tr->w.w3, tr->w.rms_final_weight};
    const float *pg[] = {tr->g_rms_att, tr->g_wq, tr->g_wk, tr->g_wv, tr->g_wo, tr->g_rms_ffn,
                         tr->g_w1, tr->g_w2, tr->g_w3, tr->g_rms_final};
    bool packed = w0 && g0;
    for (int i = 0; i < 10 && packed; i++) packed = pw[i] - w0 == pg[i] - g0;
    if (!packed) {
        ptc_trainer_sgd_head(tr, lr);
        ptc_trainer_sgd_layers(tr, lr, 0, tr->L);
        return;
    }
    sgd_range(tr, w0, g0, (size_t)(tr->g_rms_final + tr->D - g0), lr);
    if (tr->g_wcls && tr->g_wcls != tr->g_emb) sgd_range(tr, tr->w.wcls, tr->g_wcls, (size_t)tr->V * tr->D, lr);
    PTC_CHECK(cudaGetLastError());
}

// pt_train_step (pitorch/pt.c:339-364) on a full-model trainer.
extern "C" float ptc_trainer_step(ptc_trainer *tr, const int *tokens, int T, float lr) {
    if (!tr->has_embed || !tr->has_head) PTC_FATAL("ptc_trainer_step needs embedding and head");
    ptc_trainer_set_tokens(tr, tokens, T);
    ptc_trainer_zero_grads(tr);
    ptc_trainer_fwd_embed(tr);
    ptc_trainer_fwd_layers(tr, 0, tr->L);
    fwd_head_enqueue(tr);   // the loss is read once the whole step ran
    ptc_trainer_bwd_head(tr);
    ptc_trainer_bwd_layers(tr, 0, tr->L);
    ptc_trainer_bwd_embed(tr);
    sgd_all(tr, lr);
    PTC_CHECK(cudaStreamSynchronize(tr->s));
    return *tr->loss_host;
}

extern "C" void ptc_trainer_sync(ptc_trainer *tr) { PTC_CHECK(cudaStreamSynchronize(tr->s)); }
