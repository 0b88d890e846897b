/*
 * pt_text.c -- tokenizer, sampler and generation loop (pitorch/text/pt_text.c
 * semantics). Host string work; the forward passes of pt_generate run on the
 * GPU through the state's device twin.
 */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include "../../../include/pt_text.h"
#include "pt_device.h"


/* ---- tokenizer (pt_text.c:30-203) ------------------------------------------ */

void pt_tokenizer_init(pt_tokenizer_t *t, const void *data, int vocab_size) {
    const unsigned char *p = (const unsigned char *)data;
    unsigned max_len;
    memcpy(&max_len, p, 4);
    p += 4;
    t->vocab_size = vocab_size;
    t->max_token_length = (int)max_len;
    t->vocab = (char **)malloc((size_t)vocab_size * sizeof(char *));
    t->vocab_scores = (float *)malloc((size_t)vocab_size * sizeof(float));
    t->sorted_vocab = (pt_token_index_t *)malloc((size_t)vocab_size * sizeof(pt_token_index_t));
    t->sorted_ready = 0;
    for (int i = 0; i < vocab_size; i++) {
        int len;
        memcpy(&t->vocab_scores[i], p, 4);
        memcpy(&len, p + 4, 4);
        p += 8;
        t->vocab[i] = (char *)malloc((size_t)len + 1);
        memcpy(t->vocab[i], p, (size_t)len);
        t->vocab[i][len] = '\0';
        p += len;
    }
}

void pt_tokenizer_free(pt_tokenizer_t *t) {
    if (!t->vocab) return;
    for (int i = 0; i < t->vocab_size; i++) free(t->vocab[i]);
    free(t->vocab);
    free(t->vocab_scores);
    free(t->sorted_vocab);
    memset(t, 0, sizeof(*t));
}

/* The tokenizer follows the model weights in a combined file (pt_text.c:30-34). */
void pt_load_tokenizer(pt_tokenizer_t *t, const void *combined_file, int vocab_size) {
    pt_tokenizer_init(t, (const char *)combined_file + pt_file_size(combined_file), vocab_size);
}

static unsigned char g_byte_piece[2];

/* pt_text.c:74-98: BOS strips the leading space; <0xHH> pieces are raw bytes. */
const char *pt_decode(pt_tokenizer_t *t, int prev_token, int token) {
    const char *piece = t->vocab[token];
    if (prev_token == 1 && piece[0] == ' ') piece++;
    if (strlen(piece) == 6 && piece[0] == '<' && piece[1] == '0' && piece[2] == 'x' && piece[5] == '>') {
        unsigned v = 0;
        for (int i = 3; i < 5; i++) {
            char c = piece[i];
            v <<= 4;
            if (c >= '0' && c <= '9') v |= (unsigned)(c - '0');
            else if (c >= 'a' && c <= 'f') v |= (unsigned)(c - 'a' + 10);
            else if (c >= 'A' && c <= 'F') v |= (unsigned)(c - 'A' + 10);
        }
        g_byte_piece[0] = (unsigned char)v;
        g_byte_piece[1] = '\0';
        return (const char *)g_byte_piece;
    }
    return piece;
}

static int cmp_index(const void *a, const void *b) {
    return strcmp(((const pt_token_index_t *)a)->str, ((const pt_token_index_t *)b)->str);
}

static int lookup(pt_tokenizer_t *t, const char *str) {
    pt_token_index_t key = {(char *)str, 0};
    const pt_token_index_t *hit =
        (const pt_token_index_t *)bsearch(&key, t->sorted_vocab, (size_t)t->vocab_size, sizeof(key), cmp_index);
    return hit ? hit->id : -1;
}

/* pt_text.c:139-203: codepoints (byte fallback id = byte + 3), then merge the
 * adjacent pair whose concatenation has the highest score until none does. */
void pt_encode(pt_tokenizer_t *t, const char *text, int bos, int eos, int *tokens, int *n_tokens) {
    if (!t->sorted_ready) {
        for (int i = 0; i < t->vocab_size; i++) {
            t->sorted_vocab[i].str = t->vocab[i];
            t->sorted_vocab[i].id = i;
        }
        qsort(t->sorted_vocab, (size_t)t->vocab_size, sizeof(pt_token_index_t), cmp_index);
        t->sorted_ready = 1;
    }
    int n = 0;
    if (bos) tokens[n++] = 1;
    if (text[0]) {
        int sp = lookup(t, " ");
        if (sp != -1) tokens[n++] = sp;
    }
    for (const char *c = text; *c;) {
        int len = 1;
        unsigned char b = (unsigned char)*c;
        if ((b & 0x80) == 0) len = 1;
        else if ((b & 0xE0) == 0xC0) len = 2;
        else if ((b & 0xF0) == 0xE0) len = 3;
        else if ((b & 0xF8) == 0xF0) len = 4;
        char cp[8];
        memcpy(cp, c, (size_t)len);
        cp[len] = '\0';
        int id = lookup(t, cp);
        if (id != -1) tokens[n++] = id;
        else
            for (int i = 0; i < len; i++) tokens[n++] = (unsigned char)c[i] + 3;
        c += len;
    }
    char *buf = (char *)malloc((size_t)2 * t->max_token_length + 2);
    for (;;) {
        float best = -1e10f;
        int at = -1, best_id = -1;
        for (int i = 0; i + 1 < n; i++) {
            strcpy(buf, t->vocab[tokens[i]]);
            strcat(buf, t->vocab[tokens[i + 1]]);
            int id = lookup(t, buf);
            if (id != -1 && t->vocab_scores[id] > best) {
                best = t->vocab_scores[id];
                at = i;
                best_id = id;
            }
        }
        if (at < 0) break;
        tokens[at] = best_id;
        memmove(tokens + at + 1, tokens + at + 2, (size_t)(n - at - 2) * sizeof(int));
        n--;
    }
    free(buf);
    if (eos) tokens[n++] = 2;
    *n_tokens = n;
}

/* ---- sampler (pt_text.c:209-308) ------------------------------------------- */

/* pitorch's exp (pitorch/ops/core/pt_math.c:8-25), used by its softmax. */
static float host_expf(float x) {
    if (x > 88.7f) return 3.4028235e+38f;
    if (x < -87.3f) return 0.0f;
    float t = x * 1.4426950408889634f;
    int k = (int)(t + (t >= 0 ? 0.5f : -0.5f));
    float r = x - (float)k * 0.6931471805599453f;
    float p = 0.0083333333f;
    p = 0.0416666667f + r * p;
    p = 0.1666666667f + r * p;
    p = 0.5f + r * p;
    p = 1.0f + r * p;
    p = 1.0f + r * p;
    union { float f; unsigned u; } sc;
    sc.u = (unsigned)(k + 127) << 23;
    return p * sc.f;
}

static void host_softmax(float *x, int n) {
    float mx = x[0];
    for (int i = 1; i < n; i++) if (x[i] > mx) mx = x[i];
    float total = 0.0f;
    for (int i = 0; i < n; i++) { x[i] = host_expf(x[i] - mx); total += x[i]; }
    float r = 1.0f / total;
    for (int i = 0; i < n; i++) x[i] *= r;
}

static uint64_t xorshift(uint64_t *s) {
    uint64_t x = *s;
    x ^= x << 13;
    x ^= x >> 7;
    x ^= x << 17;
    *s = x;
    return x;
}

void pt_sampler_init(pt_sampler_t *s, int vocab_size, float temp, float topp, uint64_t seed) {
    s->vocab_size = vocab_size;
    s->temperature = temp;
    s->topp = topp;
    s->rng_state = seed ? seed : 42;
}

typedef struct { float prob; int index; } prob_index_t;

static void sift(prob_index_t *a, int n, int i) {
    for (;;) {
        int big = i, l = 2 * i + 1, r = 2 * i + 2;
        if (l < n && a[l].prob > a[big].prob) big = l;
        if (r < n && a[r].prob > a[big].prob) big = r;
        if (big == i) return;
        prob_index_t tmp = a[i]; a[i] = a[big]; a[big] = tmp;
        i = big;
    }
}

/* in-place heapsort, ascending by prob (same ordering of ties as the reference) */
static void heapsort_probs(prob_index_t *a, int n) {
    for (int i = n / 2 - 1; i >= 0; i--) sift(a, n, i);
    for (int i = n - 1; i > 0; i--) {
        prob_index_t tmp = a[0]; a[0] = a[i]; a[i] = tmp;
        sift(a, i, 0);
    }
}

int pt_sample(pt_sampler_t *s, float *logits) {
    const int n = s->vocab_size;
    if (s->temperature == 0.0f) return pt_argmax(logits, n);
    const float inv_t = 1.0f / s->temperature;
    for (int i = 0; i < n; i++) logits[i] *= inv_t;
    host_softmax(logits, n);
    const float coin = (float)(xorshift(&s->rng_state) >> 40) * 5.9604644775390625e-08f;
    if (s->topp > 0.0f && s->topp < 1.0f) {
        prob_index_t *pool = (prob_index_t *)malloc((size_t)n * sizeof(prob_index_t));
        const float cutoff = (1.0f - s->topp) / (float)(n - 1);
        int n0 = 0;
        for (int i = 0; i < n; i++)
            if (logits[i] >= cutoff) { pool[n0].index = i; pool[n0].prob = logits[i]; n0++; }
        if (n0 > 0) {
            heapsort_probs(pool, n0);
            float cum = 0.0f;
            int last = 0;
            for (int i = n0 - 1; i >= 0; i--) {
                cum += pool[i].prob;
                if (cum > s->topp) { last = i; break; }
            }
            const float r = coin * cum;
            float cdf = 0.0f;
            int pick = pool[last].index;
            for (int i = n0 - 1; i >= last; i--) {
                cdf += pool[i].prob;
                if (r < cdf) { pick = pool[i].index; break; }
            }
            free(pool);
            return pick;
        }
        free(pool);
    }
    float cdf = 0.0f;
    for (int i = 0; i < n; i++) {
        cdf += logits[i];
        if (coin < cdf) return i;
    }
    return n - 1;
}

/* ---- generation (pt_text.c:314-379) ---------------------------------------- */

static double now_s(void) {
    struct timespec t;
    clock_gettime(CLOCK_MONOTONIC, &t);
    return (double)t.tv_sec + 1e-9 * (double)t.tv_nsec;
}

void pt_generate(const pt_config_t *cfg, const pt_weights_t *w, pt_state_t *s, pt_tokenizer_t *tok,
                 pt_sampler_t *sampler, const char *prompt, int max_tokens, pt_matvec_fn matvec) {
    (void)matvec;
    struct pt_device *d = pt_state_device(cfg, w, s);
    int *ptoks = (int *)malloc((strlen(prompt) + 3) * sizeof(int));
    int n_prompt = 0;
    pt_encode(tok, prompt, 1, 0, ptoks, &n_prompt);
    if (max_tokens > cfg->seq_len) max_tokens = cfg->seq_len;
    ptc_decoder_reset(d->dec);
    int token = ptoks[0], n_decode = 0;
    double prefill = 0.0, decode = 0.0;
    const int greedy = sampler->temperature == 0.0f;
    for (int pos = 0; pos < max_tokens; pos++) {
        const double t0 = now_s();
        /* greedy sampling uses the GPU argmax; other modes need the logits */
        const int dev_next = ptc_decoder_step(d->dec, token, pos, greedy ? NULL : s->logits);
        const double dt = now_s() - t0;
        int next;
        if (pos < n_prompt - 1) {
            next = ptoks[pos + 1];
            prefill += dt;
        } else {
            next = greedy ? dev_next : pt_sample(sampler, s->logits);
            decode += dt;
            n_decode++;
            if (next == 1 || next == 2) break;
            printf("%s", pt_decode(tok, token, next));
            fflush(stdout);
        }
        token = next;
    }
    printf("\n[%d tokens | prefill %.1fs | decode %.1fs", n_prompt - 1 + n_decode, prefill, decode);
    if (n_decode > 0 && decode > 0.0) printf(" | %.1f tok/s", (double)n_decode / decode);
    printf("]\n");
    fflush(stdout);
    free(ptoks);
}
