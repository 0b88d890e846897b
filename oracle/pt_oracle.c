/*
 * pt_oracle.c -- TEST INFRASTRUCTURE ONLY (see pt_oracle.h).
 *
 * A plain-C restatement of pitorch's host decode and training arithmetic.
 * Loops keep the reference's accumulation order so that, compiled with
 * gcc -O2 -ffp-contract=off, results are bit-identical to the reference's
 * host build; tests/test_oracle_pins.py checks exactly that.
 *
 * Paths in citations are relative to the pitorch project root.
 */
#include "pt_oracle.h"

#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* ======================================================================
 * Math: pitorch/ops/core/pt_math.c
 * ====================================================================== */

static float bits_to_float(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static uint32_t float_to_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

/* pt_math.c:8-25 -- n = round-half-away(x/ln2), r = x - n ln2,
 * degree-5 Taylor in Horner form, times 2^n built in the exponent field. */
float or_expf(float x) {
    if (x > 88.7f) return 3.4028235e+38f;
    if (x < -87.3f) return 0.0f;
    float t = x * 1.4426950408889634f;
    int n = (int)(t + (t >= 0 ? 0.5f : -0.5f));
    float r = x - (float)n * 0.6931471805599453f;
    float poly = 0.0083333333f;
    poly = 0.0416666667f + r * poly;
    poly = 0.1666666667f + r * poly;
    poly = 0.5f + r * poly;
    poly = 1.0f + r * poly;
    poly = 1.0f + r * poly;
    return poly * bits_to_float((uint32_t)(n + 127) << 23);
}

/* pt_math.c:31-44 -- split exponent/mantissa, fold mantissa to
 * [sqrt(1/2), sqrt(2)), 9-term series for ln(1+f). */
float or_logf(float x) {
    if (x <= 0.0f) return -3.4028235e+38f;
    uint32_t u = float_to_bits(x);
    int e = (int)((u >> 23) & 0xFF) - 127;
    float m = bits_to_float((u & 0x007FFFFFu) | 0x3F800000u);
    if (m > 1.41421356f) { m *= 0.5f; e++; }
    float f = m - 1.0f;
    float s = 0.11111111f;
    s = -0.125f + f * s;
    s = 0.14285714f + f * s;
    s = -0.16666667f + f * s;
    s = 0.2f + f * s;
    s = -0.25f + f * s;
    s = 0.33333333f + f * s;
    s = -0.5f + f * s;
    s = 1.0f + f * s;
    return f * s + (float)e * 0.69314718f;
}

/* pt_math.c:58-62 -- reduce to [-pi, pi] with a rounded multiple of 2 pi. */
static float reduce_2pi(float x) {
    float k = x * 0.15915494309190f;
    k = (float)(int)(k + (k >= 0 ? 0.5f : -0.5f));
    return x - k * 6.28318530717959f;
}

/* pt_math.c:64-74 -- fold into [-pi/2, pi/2], odd degree-9 polynomial. */
float or_sinf(float x) {
    x = reduce_2pi(x);
    if (x > 1.57079632679490f) x = 3.14159265358979f - x;
    else if (x < -1.57079632679490f) x = -3.14159265358979f - x;
    float z = x * x;
    float s = 0.00000275573f;
    s = -0.00019841270f + z * s;
    s = 0.00833333333f + z * s;
    s = -0.16666666667f + z * s;
    s = 1.0f + z * s;
    return x * s;
}

/* pt_math.c:76-87 -- fold with sign flip, even degree-8 polynomial. */
float or_cosf(float x) {
    x = reduce_2pi(x);
    float sign = 1.0f;
    if (x > 1.57079632679490f) { x = 3.14159265358979f - x; sign = -1.0f; }
    else if (x < -1.57079632679490f) { x = -3.14159265358979f - x; sign = -1.0f; }
    float z = x * x;
    float c = 0.00002480159f;
    c = -0.00138888889f + z * c;
    c = 0.04166666667f + z * c;
    c = -0.50000000000f + z * c;
    c = 1.0f + z * c;
    return sign * c;
}

/* pt_math.c:92-102 -- exponent-halving bit trick, three Newton steps. */
float or_sqrtf(float x) {
    if (x <= 0.0f) return 0.0f;
    float y = bits_to_float(0x1fbd1df5u + (float_to_bits(x) >> 1));
    for (int it = 0; it < 3; it++) y = 0.5f * (y + x / y);
    return y;
}

/* ======================================================================
 * Elementwise ops: pitorch/ops/core/pt_ops.c
 * ====================================================================== */

/* pt_ops.c:5-12 */
void or_rmsnorm(float *o, const float *x, const float *w, int dim) {
    float acc = 0.0f;
    for (int i = 0; i < dim; i++) acc += x[i] * x[i];
    float scale = 1.0f / or_sqrtf(acc / dim + 1e-5f);
    for (int i = 0; i < dim; i++) o[i] = x[i] * scale * w[i];
}

/* pt_ops.c:14-26 */
void or_softmax(float *x, int n) {
    float mx = x[0];
    for (int i = 1; i < n; i++) if (x[i] > mx) mx = x[i];
    float total = 0.0f;
    for (int i = 0; i < n; i++) { x[i] = or_expf(x[i] - mx); total += x[i]; }
    float r = 1.0f / total;
    for (int i = 0; i < n; i++) x[i] *= r;
}

/* pt_ops.c:28-31 */
void or_silu(float *x, int n) {
    for (int i = 0; i < n; i++) x[i] = x[i] / (1.0f + or_expf(-x[i]));
}

/* pt_ops.c:33-49 -- pairs (i, i+1) rotated by pos * 10000^(-(i mod hd)/hd),
 * the base written as exp(-9.210340372 * i / hd). k is rotated over dim too. */
void or_rope(float *q, float *k, int dim, int head_dim, int pos) {
    for (int i = 0; i < dim; i += 2) {
        float theta = (float)pos *
            or_expf(-9.210340372f * (float)(i % head_dim) / (float)head_dim);
        float c = or_cosf(theta), s = or_sinf(theta);
        float a = q[i], b = q[i + 1];
        q[i] = a * c - b * s;
        q[i + 1] = a * s + b * c;
        a = k[i]; b = k[i + 1];
        k[i] = a * c - b * s;
        k[i + 1] = a * s + b * c;
    }
}

/* pt_ops.c:65-70 -- first maximum wins (strict >). */
int or_argmax(const float *x, int n) {
    int best = 0;
    for (int i = 1; i < n; i++) if (x[i] > x[best]) best = i;
    return best;
}

/* pt_ops.c:72-80 -- y[i] = sum_j W[i][j] x[j], j ascending. */
void or_matvec(const float *W, const float *x, float *y, int rows, int cols) {
    for (int i = 0; i < rows; i++) {
        const float *row = W + (size_t)i * cols;
        float acc = 0.0f;
        for (int j = 0; j < cols; j++) acc += row[j] * x[j];
        y[i] = acc;
    }
}

/* ======================================================================
 * Backward primitives: pitorch/train/pt_backward_ops.c
 * ====================================================================== */

/* pt_backward_ops.c:4-30 */
void or_rmsnorm_backward(float *dx, float *dw, const float *dout,
                         const float *x, const float *w, int dim) {
    float acc = 0.0f;
    for (int i = 0; i < dim; i++) acc += x[i] * x[i];
    acc = acc / dim + 1e-5f;
    float inv = 1.0f / or_sqrtf(acc);
    for (int i = 0; i < dim; i++) dw[i] += dout[i] * x[i] * inv;
    float dot = 0.0f;
    for (int i = 0; i < dim; i++) dot += dout[i] * w[i] * x[i];
    float coeff = inv * inv * inv / (float)dim;
    for (int i = 0; i < dim; i++) dx[i] += inv * dout[i] * w[i] - coeff * dot * x[i];
}

/* pt_backward_ops.c:52-69 -- inverse rotation, accumulated into dq/dk. */
void or_rope_backward(float *dq, float *dk, const float *dq_out,
                      const float *dk_out, int dim, int head_dim, int pos) {
    for (int i = 0; i < dim; i += 2) {
        float theta = (float)pos *
            or_expf(-9.210340372f * (float)(i % head_dim) / (float)head_dim);
        float c = or_cosf(theta), s = or_sinf(theta);
        dq[i]     +=  dq_out[i] * c + dq_out[i + 1] * s;
        dq[i + 1] += -dq_out[i] * s + dq_out[i + 1] * c;
        dk[i]     +=  dk_out[i] * c + dk_out[i + 1] * s;
        dk[i + 1] += -dk_out[i] * s + dk_out[i + 1] * c;
    }
}

/* pt_backward_ops.c:71-79 */
void or_softmax_backward(float *dx, const float *dy, const float *y, int n) {
    float dot = 0.0f;
    for (int i = 0; i < n; i++) dot += dy[i] * y[i];
    for (int i = 0; i < n; i++) dx[i] += y[i] * (dy[i] - dot);
}

/* dx[j] = sum_{i<rows} W[i][j] dy[i], i ascending: the order of
 * pt_backward_ops.c:32-41 and of the transposed matvec the host build takes
 * (pt_train.c:442-453 with smatvec_cpu); both give the same bits. */
static void matvec_t(const float *W, const float *dy, float *dx, int rows, int cols) {
    for (int j = 0; j < cols; j++) {
        float acc = 0.0f;
        for (int i = 0; i < rows; i++) acc += W[(size_t)i * cols + j] * dy[i];
        dx[j] = acc;
    }
}

/* pt_train.c:475-492 -- dW[i][j] += sum_t dy_t[i] x_t[j], t ascending per
 * element (the row tiling does not change the per-element order). */
static void weight_grad(float *dW, const float *dy_all, const float *x_all,
                        int rows, int cols, int n) {
    for (int t = 0; t < n; t++) {
        const float *dy = dy_all + (size_t)t * rows;
        const float *x = x_all + (size_t)t * cols;
        for (int i = 0; i < rows; i++) {
            float d = dy[i];
            float *g = dW + (size_t)i * cols;
            for (int j = 0; j < cols; j++) g[j] += d * x[j];
        }
    }
}

/* ======================================================================
 * Model: pitorch/model/llama2.c, pitorch/train/pt_train.c
 * ====================================================================== */

typedef struct {
    float *emb, *rms_att, *wq, *wk, *wv, *wo, *rms_ffn, *w1, *w2, *w3,
          *rms_final, *wcls;
} or_weights;

struct or_model {
    int dim, hidden, L, nh, nkv, V, seq, hd, kvd, shared;
    char *blob;
    long blob_bytes;
    or_weights w;
    /* decode state (llama2.h:35-48) */
    float *x, *xb, *xb2, *q, *k, *v, *hb, *hb2, *att, *logits, *kc, *vc;
    /* training (pt_train.h:34-129) */
    int max_T;
    float *res, *res_att, *xb_att, *aq, *ak, *av, *aatt, *aout, *xb_ffn,
          *ahb, *ahb2, *x_final, *alogits, *scratch;
    float *g_mem;
    long n_params;
    or_weights g;
    float *d_res, *d_aout, *d_q, *d_k, *d_v, *d_xb, *d_qpre, *d_kpre,
          *d_hid, *d_hid2, *d_att_s, *d_pre_sm, *d_temp, *d_logit_all,
          *drt_wo_all, *d_qpre_all, *d_kpre_all, *sh_all, *d_hid_all,
          *d_hid2_all, *drt_ffn_all;
};

static float *fz(size_t n) { return (float *)calloc(n ? n : 1, sizeof(float)); }

/* llama2.c:49-70 layout: emb, rms_att, wq, wk, wv, wo, rms_ffn, w1, w2, w3,
 * rms_final, freq_cis (skipped), [wcls if vocab < 0]. */
static void carve(or_weights *w, float *p, const or_model *m) {
    size_t D = m->dim, H = m->hidden, L = m->L, K = m->kvd;
    w->emb = p;       p += (size_t)m->V * D;
    w->rms_att = p;   p += L * D;
    w->wq = p;        p += L * D * D;
    w->wk = p;        p += L * K * D;
    w->wv = p;        p += L * K * D;
    w->wo = p;        p += L * D * D;
    w->rms_ffn = p;   p += L * D;
    w->w1 = p;        p += L * H * D;
    w->w2 = p;        p += L * D * H;
    w->w3 = p;        p += L * H * D;
    w->rms_final = p; p += D;
    p += (size_t)m->seq * m->hd;      /* freq_cis_real + freq_cis_imag */
    w->wcls = m->shared ? w->emb : p;
}

or_model *or_open(const void *blob, long blob_bytes, int max_T) {
    const int *h = (const int *)blob;
    or_model *m = (or_model *)calloc(1, sizeof(or_model));
    m->dim = h[0]; m->hidden = h[1]; m->L = h[2]; m->nh = h[3]; m->nkv = h[4];
    m->V = h[5] > 0 ? h[5] : -h[5];
    m->shared = h[5] > 0;
    m->seq = h[6];
    m->hd = m->dim / m->nh;
    m->kvd = m->nkv * m->hd;
    m->blob = (char *)malloc((size_t)blob_bytes);
    memcpy(m->blob, blob, (size_t)blob_bytes);
    m->blob_bytes = blob_bytes;
    carve(&m->w, (float *)(m->blob + 28), m);

    size_t D = m->dim, H = m->hidden, L = m->L, K = m->kvd;
    m->x = fz(D); m->xb = fz(D); m->xb2 = fz(D); m->q = fz(D);
    m->k = fz(K); m->v = fz(K); m->hb = fz(H); m->hb2 = fz(H);
    m->att = fz((size_t)m->nh * m->seq); m->logits = fz(m->V);
    m->kc = fz(L * m->seq * K); m->vc = fz(L * m->seq * K);

    m->max_T = max_T;
    if (max_T > 0) {
        size_t T = max_T, V = m->V;
        m->res = fz((L + 1) * T * D); m->res_att = fz(L * T * D);
        m->xb_att = fz(L * T * D); m->aq = fz(L * T * D);
        m->ak = fz(L * T * K); m->av = fz(L * T * K);
        m->aatt = fz(L * m->nh * T * T); m->aout = fz(L * T * D);
        m->xb_ffn = fz(L * T * D); m->ahb = fz(L * T * H); m->ahb2 = fz(L * T * H);
        m->x_final = fz(T * D); m->alogits = fz(T * V);
        m->scratch = fz(H > D ? H : D);
        /* pt_train.c:334-371 gradient layout */
        m->n_params = (long)(V * D + L * D + L * D * D + 2 * L * K * D + L * D * D +
                             L * D + 3 * L * H * D + D + (m->shared ? 0 : V * D));
        m->g_mem = fz((size_t)m->n_params);
        float *p = m->g_mem;
        m->g.emb = p;      p += V * D;
        m->g.rms_att = p;  p += L * D;
        m->g.wq = p;       p += L * D * D;
        m->g.wk = p;       p += L * K * D;
        m->g.wv = p;       p += L * K * D;
        m->g.wo = p;       p += L * D * D;
        m->g.rms_ffn = p;  p += L * D;
        m->g.w1 = p;       p += L * H * D;
        m->g.w2 = p;       p += L * D * H;
        m->g.w3 = p;       p += L * H * D;
        m->g.rms_final = p; p += D;
        m->g.wcls = m->shared ? m->g.emb : p;
        m->d_res = fz(T * D); m->d_aout = fz(T * D); m->d_q = fz(T * D);
        m->d_k = fz(T * K); m->d_v = fz(T * K); m->d_xb = fz(D);
        m->d_qpre = fz(D); m->d_kpre = fz(K); m->d_hid = fz(H); m->d_hid2 = fz(H);
        m->d_att_s = fz(T); m->d_pre_sm = fz(T); m->d_temp = fz(H > D ? H : D);
        m->d_logit_all = fz(T * V);
        m->drt_wo_all = fz(T * D); m->d_qpre_all = fz(T * D); m->d_kpre_all = fz(T * K);
        m->sh_all = fz(T * H); m->d_hid_all = fz(T * H); m->d_hid2_all = fz(T * H);
        m->drt_ffn_all = fz(T * D);
    }
    return m;
}

void or_close(or_model *m) {
    if (!m) return;
    float *bufs[] = {m->x, m->xb, m->xb2, m->q, m->k, m->v, m->hb, m->hb2, m->att,
                     m->logits, m->kc, m->vc, m->res, m->res_att, m->xb_att, m->aq,
                     m->ak, m->av, m->aatt, m->aout, m->xb_ffn, m->ahb, m->ahb2,
                     m->x_final, m->alogits, m->scratch, m->g_mem, m->d_res,
                     m->d_aout, m->d_q, m->d_k, m->d_v, m->d_xb, m->d_qpre,
                     m->d_kpre, m->d_hid, m->d_hid2, m->d_att_s, m->d_pre_sm,
                     m->d_temp, m->d_logit_all, m->drt_wo_all, m->d_qpre_all,
                     m->d_kpre_all, m->sh_all, m->d_hid_all, m->d_hid2_all,
                     m->drt_ffn_all};
    for (size_t i = 0; i < sizeof(bufs) / sizeof(bufs[0]); i++) free(bufs[i]);
    free(m->blob);
    free(m);
}

void or_config(const or_model *m, int out[7]) {
    out[0] = m->dim; out[1] = m->hidden; out[2] = m->L; out[3] = m->nh;
    out[4] = m->nkv; out[5] = m->V; out[6] = m->seq;
}

/* pt.c:273-280 */
void or_reset_kv(or_model *m) {
    size_t n = (size_t)m->L * m->seq * m->kvd;
    memset(m->kc, 0, n * sizeof(float));
    memset(m->vc, 0, n * sizeof(float));
}

const float *or_logits(const or_model *m) { return m->logits; }
const float *or_x(const or_model *m) { return m->x; }
void or_set_x(or_model *m, const float *x) { memcpy(m->x, x, m->dim * sizeof(float)); }
const void *or_blob(const or_model *m) { return m->blob; }
long or_blob_bytes(const or_model *m) { return m->blob_bytes; }
const float *or_grads(const or_model *m, long *n_out) {
    if (n_out) *n_out = m->n_params;
    return m->g_mem;
}

/* llama2.c:220-222 */
void or_forward_embed(or_model *m, int token) {
    memcpy(m->x, m->w.emb + (size_t)token * m->dim, m->dim * sizeof(float));
}

/* llama2.c:224-289 -- one decode position through layers [l0, l1). */
void or_forward_layers_range(or_model *m, int pos, int l0, int l1) {
    const int D = m->dim, H = m->hidden, hd = m->hd, K = m->kvd;
    const int group = m->nh / m->nkv;
    const float scale = 1.0f / or_sqrtf((float)hd);
    for (int l = l0; l < l1; l++) {
        or_rmsnorm(m->xb, m->x, m->w.rms_att + (size_t)l * D, D);
        or_matvec(m->w.wq + (size_t)l * D * D, m->xb, m->q, D, D);
        or_matvec(m->w.wk + (size_t)l * K * D, m->xb, m->k, K, D);
        or_matvec(m->w.wv + (size_t)l * K * D, m->xb, m->v, K, D);
        or_rope(m->q, m->k, D, hd, pos);

        float *kl = m->kc + (size_t)l * m->seq * K;
        float *vl = m->vc + (size_t)l * m->seq * K;
        memcpy(kl + (size_t)pos * K, m->k, K * sizeof(float));
        memcpy(vl + (size_t)pos * K, m->v, K * sizeof(float));

        for (int h = 0; h < m->nh; h++) {
            const float *qh = m->q + h * hd;
            float *ah = m->att + (size_t)h * m->seq;
            int koff = (h / group) * hd;
            for (int t = 0; t <= pos; t++) {
                const float *kt = kl + (size_t)t * K + koff;
                float dot = 0.0f;
                for (int i = 0; i < hd; i++) dot += qh[i] * kt[i];
                ah[t] = dot * scale;
            }
            or_softmax(ah, pos + 1);
            float *oh = m->xb + h * hd;
            memset(oh, 0, hd * sizeof(float));
            for (int t = 0; t <= pos; t++) {
                const float *vt = vl + (size_t)t * K + koff;
                float a = ah[t];
                for (int i = 0; i < hd; i++) oh[i] += a * vt[i];
            }
        }
        or_matvec(m->w.wo + (size_t)l * D * D, m->xb, m->xb2, D, D);
        for (int i = 0; i < D; i++) m->x[i] = m->x[i] + m->xb2[i];

        or_rmsnorm(m->xb, m->x, m->w.rms_ffn + (size_t)l * D, D);
        or_matvec(m->w.w1 + (size_t)l * H * D, m->xb, m->hb, H, D);
        or_matvec(m->w.w3 + (size_t)l * H * D, m->xb, m->hb2, H, D);
        or_silu(m->hb, H);
        for (int i = 0; i < H; i++) m->hb[i] = m->hb[i] * m->hb2[i];
        or_matvec(m->w.w2 + (size_t)l * D * H, m->hb, m->xb, D, H);
        for (int i = 0; i < D; i++) m->x[i] = m->x[i] + m->xb[i];
    }
}

/* llama2.c:291-295 -- note x is normalised in place. */
void or_forward_head(or_model *m) {
    or_rmsnorm(m->x, m->x, m->w.rms_final, m->dim);
    or_matvec(m->w.wcls, m->x, m->logits, m->V, m->dim);
}

/* llama2.c:298-303 */
void or_forward(or_model *m, int token, int pos) {
    or_forward_embed(m, token);
    or_forward_layers_range(m, pos, 0, m->L);
    or_forward_head(m);
}

void or_decode_greedy(or_model *m, const int *prompt, int n_prompt, int n_pos,
                      int *tokens_out, float *logits_out) {
    or_reset_kv(m);
    int tok = prompt[0];
    for (int p = 0; p < n_pos; p++) {
        or_forward(m, tok, p);
        if (logits_out) memcpy(logits_out + (size_t)p * m->V, m->logits, m->V * sizeof(float));
        int next = (p + 1 < n_prompt) ? prompt[p + 1] : or_argmax(m->logits, m->V);
        tokens_out[p] = next;
        tok = next;
    }
}

/* ---- training -------------------------------------------------------- */

/* pt_train.c:171-329 */
float or_forward_train(or_model *m, const int *tokens, int T) {
    const int D = m->dim, H = m->hidden, hd = m->hd, K = m->kvd, nh = m->nh;
    const int L = m->L, V = m->V, group = nh / m->nkv;
    const float scale = 1.0f / or_sqrtf((float)hd);

    for (int t = 0; t < T; t++)
        memcpy(m->res + (size_t)t * D, m->w.emb + (size_t)tokens[t] * D, D * sizeof(float));

    for (int l = 0; l < L; l++) {
        float *rin = m->res + (size_t)l * T * D;
        float *rmid = m->res_att + (size_t)l * T * D;
        float *rout = m->res + (size_t)(l + 1) * T * D;
        for (int t = 0; t < T; t++) {
            float *xb = m->xb_att + ((size_t)l * T + t) * D;
            or_rmsnorm(xb, rin + (size_t)t * D, m->w.rms_att + (size_t)l * D, D);
            float *qt = m->aq + ((size_t)l * T + t) * D;
            float *kt = m->ak + ((size_t)l * T + t) * K;
            float *vt = m->av + ((size_t)l * T + t) * K;
            or_matvec(m->w.wq + (size_t)l * D * D, xb, qt, D, D);
            or_matvec(m->w.wk + (size_t)l * K * D, xb, kt, K, D);
            or_matvec(m->w.wv + (size_t)l * K * D, xb, vt, K, D);
            or_rope(qt, kt, D, hd, t);
        }
        for (int t = 0; t < T; t++) {
            const float *qt = m->aq + ((size_t)l * T + t) * D;
            float *ot = m->aout + ((size_t)l * T + t) * D;
            for (int h = 0; h < nh; h++) {
                const float *qh = qt + h * hd;
                float *ah = m->aatt + (((size_t)l * nh + h) * T + t) * T;
                int koff = (h / group) * hd;
                for (int s = 0; s <= t; s++) {
                    const float *ks = m->ak + ((size_t)l * T + s) * K + koff;
                    float dot = 0.0f;
                    for (int i = 0; i < hd; i++) dot += qh[i] * ks[i];
                    ah[s] = dot * scale;
                }
                for (int s = t + 1; s < T; s++) ah[s] = 0.0f;
                or_softmax(ah, t + 1);
                float *oh = ot + h * hd;
                memset(oh, 0, hd * sizeof(float));
                for (int s = 0; s <= t; s++) {
                    const float *vs = m->av + ((size_t)l * T + s) * K + koff;
                    float a = ah[s];
                    for (int i = 0; i < hd; i++) oh[i] += a * vs[i];
                }
            }
            or_matvec(m->w.wo + (size_t)l * D * D, ot, m->scratch, D, D);
            for (int i = 0; i < D; i++)
                rmid[(size_t)t * D + i] = rin[(size_t)t * D + i] + m->scratch[i];
        }
        for (int t = 0; t < T; t++) {
            float *xb = m->xb_ffn + ((size_t)l * T + t) * D;
            or_rmsnorm(xb, rmid + (size_t)t * D, m->w.rms_ffn + (size_t)l * D, D);
            float *h1 = m->ahb + ((size_t)l * T + t) * H;
            float *h3 = m->ahb2 + ((size_t)l * T + t) * H;
            or_matvec(m->w.w1 + (size_t)l * H * D, xb, h1, H, D);
            or_matvec(m->w.w3 + (size_t)l * H * D, xb, h3, H, D);
            for (int i = 0; i < H; i++) {
                float sig = 1.0f / (1.0f + or_expf(-h1[i]));
                m->scratch[i] = (h1[i] * sig) * h3[i];
            }
            float *o = rout + (size_t)t * D;
            or_matvec(m->w.w2 + (size_t)l * D * H, m->scratch, o, D, H);
            for (int i = 0; i < D; i++) o[i] = o[i] + rmid[(size_t)t * D + i];
        }
    }

    const float *rfin = m->res + (size_t)L * T * D;
    for (int t = 0; t < T; t++) {
        or_rmsnorm(m->x_final + (size_t)t * D, rfin + (size_t)t * D, m->w.rms_final, D);
        or_matvec(m->w.wcls, m->x_final + (size_t)t * D, m->alogits + (size_t)t * V, V, D);
    }
    float loss = 0.0f;
    for (int t = 0; t < T - 1; t++) {
        const float *lg = m->alogits + (size_t)t * V;
        float mx = lg[0];
        for (int v = 1; v < V; v++) if (lg[v] > mx) mx = lg[v];
        float total = 0.0f;
        for (int v = 0; v < V; v++) total += or_expf(lg[v] - mx);
        loss += -(lg[tokens[t + 1]] - mx - or_logf(total));
    }
    return loss / (float)(T - 1);
}

/* pt_train.c:549-866 (host build: transposed-matvec input grads). */
static void or_backward(or_model *m, const int *tokens, int T) {
    const int D = m->dim, H = m->hidden, hd = m->hd, K = m->kvd, nh = m->nh;
    const int L = m->L, V = m->V, group = nh / m->nkv;
    const float scale = 1.0f / or_sqrtf((float)hd);
    const int n = T - 1;   /* position T-1 carries no loss (pt_train.c:596-605) */

    memset(m->d_res, 0, (size_t)T * D * sizeof(float));
    const float invn = 1.0f / (float)(T - 1);

    /* loss backward (pt_train.c:609-621) */
    for (int t = 0; t < n; t++) {
        float *dl = m->d_logit_all + (size_t)t * V;
        const float *lg = m->alogits + (size_t)t * V;
        float mx = lg[0];
        for (int v = 1; v < V; v++) if (lg[v] > mx) mx = lg[v];
        float total = 0.0f;
        for (int v = 0; v < V; v++) { dl[v] = or_expf(lg[v] - mx); total += dl[v]; }
        float r = 1.0f / total;
        for (int v = 0; v < V; v++) dl[v] *= r * invn;
        dl[tokens[t + 1]] -= invn;
    }
    /* classifier input grad + final rmsnorm backward (pt_train.c:625-638) */
    for (int t = 0; t < n; t++) {
        matvec_t(m->w.wcls, m->d_logit_all + (size_t)t * V, m->d_xb, V, D);
        or_rmsnorm_backward(m->d_res + (size_t)t * D, m->g.rms_final, m->d_xb,
                            m->res + (size_t)L * T * D + (size_t)t * D, m->w.rms_final, D);
    }
    /* classifier weight grad (pt_train.c:651) */
    weight_grad(m->g.wcls, m->d_logit_all, m->x_final, V, D, n);

    for (int l = L - 1; l >= 0; l--) {
        const float *Wq = m->w.wq + (size_t)l * D * D, *Wk = m->w.wk + (size_t)l * K * D;
        const float *Wv = m->w.wv + (size_t)l * K * D, *Wo = m->w.wo + (size_t)l * D * D;
        const float *W1 = m->w.w1 + (size_t)l * H * D, *W2 = m->w.w2 + (size_t)l * D * H;
        const float *W3 = m->w.w3 + (size_t)l * H * D;

        /* FFN backward (pt_train.c:686-750) */
        for (int t = 0; t < n; t++) {
            float *drt = m->d_res + (size_t)t * D;
            const float *h1 = m->ahb + ((size_t)l * T + t) * H;
            const float *h3 = m->ahb2 + ((size_t)l * T + t) * H;
            float *sh = m->sh_all + (size_t)t * H;
            for (int i = 0; i < H; i++) {
                float sig = 1.0f / (1.0f + or_expf(-h1[i]));
                sh[i] = (h1[i] * sig) * h3[i];
            }
            memcpy(m->drt_ffn_all + (size_t)t * D, drt, D * sizeof(float));
            matvec_t(W2, drt, m->d_hid, D, H);
            for (int i = 0; i < H; i++) {
                float sig = 1.0f / (1.0f + or_expf(-h1[i]));
                float sv = h1[i] * sig;
                float ds = m->d_hid[i] * h3[i];
                m->d_hid2[i] = m->d_hid[i] * sv;
                m->d_hid[i] = ds * sig * (1.0f + h1[i] * (1.0f - sig));
            }
            memcpy(m->d_hid_all + (size_t)t * H, m->d_hid, H * sizeof(float));
            memcpy(m->d_hid2_all + (size_t)t * H, m->d_hid2, H * sizeof(float));
            matvec_t(W1, m->d_hid, m->d_xb, H, D);
            matvec_t(W3, m->d_hid2, m->d_temp, H, D);
            for (int i = 0; i < D; i++) m->d_xb[i] += m->d_temp[i];
            or_rmsnorm_backward(drt, m->g.rms_ffn + (size_t)l * D, m->d_xb,
                                m->res_att + ((size_t)l * T + t) * D,
                                m->w.rms_ffn + (size_t)l * D, D);
        }
        weight_grad(m->g.w2 + (size_t)l * D * H, m->drt_ffn_all, m->sh_all, D, H, n);
        weight_grad(m->g.w1 + (size_t)l * H * D, m->d_hid_all, m->xb_ffn + (size_t)l * T * D, H, D, n);
        weight_grad(m->g.w3 + (size_t)l * H * D, m->d_hid2_all, m->xb_ffn + (size_t)l * T * D, H, D, n);

        /* wo backward (pt_train.c:757-770) */
        memset(m->d_aout, 0, (size_t)T * D * sizeof(float));
        for (int t = 0; t < n; t++) {
            matvec_t(Wo, m->d_res + (size_t)t * D, m->d_aout + (size_t)t * D, D, D);
            memcpy(m->drt_wo_all + (size_t)t * D, m->d_res + (size_t)t * D, D * sizeof(float));
        }
        weight_grad(m->g.wo + (size_t)l * D * D, m->drt_wo_all, m->aout + (size_t)l * T * D, D, D, n);

        /* attention backward (pt_train.c:776-812) */
        memset(m->d_q, 0, (size_t)T * D * sizeof(float));
        memset(m->d_k, 0, (size_t)T * K * sizeof(float));
        memset(m->d_v, 0, (size_t)T * K * sizeof(float));
        for (int t = 0; t < n; t++) {
            for (int h = 0; h < nh; h++) {
                const float *dao = m->d_aout + (size_t)t * D + h * hd;
                const float *ah = m->aatt + (((size_t)l * nh + h) * T + t) * T;
                int koff = (h / group) * hd;
                memset(m->d_att_s, 0, (size_t)T * sizeof(float));
                for (int s = 0; s <= t; s++) {
                    const float *vs = m->av + ((size_t)l * T + s) * K + koff;
                    float a = ah[s];
                    for (int i = 0; i < hd; i++) {
                        m->d_att_s[s] += dao[i] * vs[i];
                        m->d_v[(size_t)s * K + koff + i] += a * dao[i];
                    }
                }
                memset(m->d_pre_sm, 0, (size_t)T * sizeof(float));
                or_softmax_backward(m->d_pre_sm, m->d_att_s, ah, t + 1);
                const float *qh = m->aq + ((size_t)l * T + t) * D + h * hd;
                for (int s = 0; s <= t; s++) {
                    const float *ks = m->ak + ((size_t)l * T + s) * K + koff;
                    float ds = m->d_pre_sm[s] * scale;
                    for (int i = 0; i < hd; i++) {
                        m->d_q[(size_t)t * D + h * hd + i] += ds * ks[i];
                        m->d_k[(size_t)s * K + koff + i] += ds * qh[i];
                    }
                }
            }
        }

        /* RoPE + QKV + attention rmsnorm backward (pt_train.c:818-852) */
        for (int t = 0; t < n; t++) {
            memset(m->d_qpre, 0, D * sizeof(float));
            memset(m->d_kpre, 0, K * sizeof(float));
            or_rope_backward(m->d_qpre, m->d_kpre, m->d_q + (size_t)t * D,
                             m->d_k + (size_t)t * K, D, hd, t);
            matvec_t(Wq, m->d_qpre, m->d_xb, D, D);
            matvec_t(Wk, m->d_kpre, m->d_temp, K, D);
            for (int i = 0; i < D; i++) m->d_xb[i] += m->d_temp[i];
            matvec_t(Wv, m->d_v + (size_t)t * K, m->d_temp, K, D);
            for (int i = 0; i < D; i++) m->d_xb[i] += m->d_temp[i];
            memcpy(m->d_qpre_all + (size_t)t * D, m->d_qpre, D * sizeof(float));
            memcpy(m->d_kpre_all + (size_t)t * K, m->d_kpre, K * sizeof(float));
            or_rmsnorm_backward(m->d_res + (size_t)t * D, m->g.rms_att + (size_t)l * D,
                                m->d_xb, m->res + ((size_t)l * T + t) * D,
                                m->w.rms_att + (size_t)l * D, D);
        }
        const float *xa = m->xb_att + (size_t)l * T * D;
        weight_grad(m->g.wq + (size_t)l * D * D, m->d_qpre_all, xa, D, D, n);
        weight_grad(m->g.wk + (size_t)l * K * D, m->d_kpre_all, xa, K, D, n);
        weight_grad(m->g.wv + (size_t)l * K * D, m->d_v, xa, K, D, n);
    }

    /* embedding backward (pt_train.c:862-863) */
    for (int t = 0; t < n; t++) {
        float *g = m->g.emb + (size_t)tokens[t] * D;
        const float *d = m->d_res + (size_t)t * D;
        for (int i = 0; i < D; i++) g[i] += d[i];
    }
}

/* pt_train.c:870-896 */
static void sgd(float *w, const float *g, size_t n, float lr) {
    for (size_t i = 0; i < n; i++) w[i] -= lr * g[i];
}

static void or_sgd(or_model *m, float lr) {
    size_t D = m->dim, H = m->hidden, L = m->L, K = m->kvd, V = m->V;
    sgd(m->w.emb, m->g.emb, V * D, lr);
    sgd(m->w.rms_att, m->g.rms_att, L * D, lr);
    sgd(m->w.wq, m->g.wq, L * D * D, lr);
    sgd(m->w.wk, m->g.wk, L * K * D, lr);
    sgd(m->w.wv, m->g.wv, L * K * D, lr);
    sgd(m->w.wo, m->g.wo, L * D * D, lr);
    sgd(m->w.rms_ffn, m->g.rms_ffn, L * D, lr);
    sgd(m->w.w1, m->g.w1, L * H * D, lr);
    sgd(m->w.w2, m->g.w2, L * D * H, lr);
    sgd(m->w.w3, m->g.w3, L * H * D, lr);
    sgd(m->w.rms_final, m->g.rms_final, D, lr);
    if (m->w.wcls != m->w.emb) sgd(m->w.wcls, m->g.wcls, V * D, lr);
}

/* pt.c:339-364 */
float or_train_step(or_model *m, const int *tokens, int T, float lr) {
    if (m->max_T <= 0 || T > m->max_T || T < 2) return -1.0f;
    memset(m->g_mem, 0, (size_t)m->n_params * sizeof(float));
    float loss = or_forward_train(m, tokens, T);
    or_backward(m, tokens, T);
    or_sgd(m, lr);
    return loss;
}
