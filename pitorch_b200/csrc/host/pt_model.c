/*
 * pt_model.c -- llama2.c .bin and SHRD shard parsing (host C).
 *
 * Same formats and pointer layout as pitorch/model/llama2.c:9-70 and
 * pitorch/model/pt_shard.c:15-130; shard cutting follows the layer
 * assignment of tools/shard_weights.py:49-66.
 */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "../../../include/llama2.h"
#include "../../../include/pt_shard.h"

/* llama2.c:9-19 -- negative vocab marks an untied classifier. */
void pt_load_config(pt_config_t *cfg, const void *data) {
    const int *h = (const int *)data;
    cfg->dim = h[0];
    cfg->hidden_dim = h[1];
    cfg->n_layers = h[2];
    cfg->n_heads = h[3];
    cfg->n_kv_heads = h[4];
    cfg->vocab_size = h[5] < 0 ? -h[5] : h[5];
    cfg->seq_len = h[6];
}

typedef struct {
    size_t emb, rms, attn_q, attn_kv, ffn, rms_final, freq;
} sizes_t;

static sizes_t tensor_sizes(const pt_config_t *c) {
    sizes_t s;
    size_t hd = (size_t)c->dim / c->n_heads;
    size_t kvd = (size_t)c->n_kv_heads * hd;
    s.emb = (size_t)c->vocab_size * c->dim;
    s.rms = (size_t)c->dim;
    s.attn_q = (size_t)c->dim * c->dim;
    s.attn_kv = kvd * c->dim;
    s.ffn = (size_t)c->hidden_dim * c->dim;
    s.rms_final = (size_t)c->dim;
    s.freq = (size_t)c->seq_len * hd / 2;
    return s;
}

/* Floats of one transformer layer in file order (rms_att, wq, wk, wv, wo,
 * rms_ffn, w1, w2, w3 per layer -- each stored for all layers at once). */
static size_t layer_floats(const sizes_t *s) {
    return 2 * s->rms + 2 * s->attn_q + 2 * s->attn_kv + 3 * s->ffn;
}

/* llama2.c:21-47 */
unsigned pt_file_size(const void *data) {
    pt_config_t c;
    pt_load_config(&c, data);
    int shared = ((const int *)data)[5] > 0;
    sizes_t s = tensor_sizes(&c);
    size_t n = s.emb + (size_t)c.n_layers * layer_floats(&s) + s.rms_final + 2 * s.freq;
    if (!shared) n += s.emb;
    return (unsigned)(28 + 4 * n);
}

/* llama2.c:49-70 */
void pt_load_weights(pt_weights_t *w, const pt_config_t *cfg, void *data) {
    int shared = ((const int *)data)[5] > 0;
    sizes_t s = tensor_sizes(cfg);
    size_t L = (size_t)cfg->n_layers;
    float *p = (float *)((char *)data + 28);
    w->token_embedding = p; p += s.emb;
    w->rms_att_weight = p;  p += L * s.rms;
    w->wq = p;              p += L * s.attn_q;
    w->wk = p;              p += L * s.attn_kv;
    w->wv = p;              p += L * s.attn_kv;
    w->wo = p;              p += L * s.attn_q;
    w->rms_ffn_weight = p;  p += L * s.rms;
    w->w1 = p;              p += L * s.ffn;
    w->w2 = p;              p += L * s.ffn;
    w->w3 = p;              p += L * s.ffn;
    w->rms_final_weight = p; p += s.rms_final;
    p += 2 * s.freq;
    w->wcls = shared ? w->token_embedding : p;
}

/* ---- shards --------------------------------------------------------------- */

static void shard_die(const char *msg, unsigned v) {
    fprintf(stderr, "pitorch_b200: %s (0x%x)\n", msg, v);
    abort();
}

/* pt_shard.c:15-39 */
void pt_load_shard_header(pt_config_t *global_cfg, pt_shard_info_t *shard, const void *data) {
    pt_load_config(global_cfg, data);
    const int *ext = (const int *)((const char *)data + 28);
    if ((unsigned)ext[0] != PT_SHARD_MAGIC) shard_die("not a shard file: bad magic", (unsigned)ext[0]);
    shard->rank = ext[1];
    shard->world_size = ext[2];
    shard->l_start = ext[3];
    shard->l_end = ext[4];
    shard->has_embed = ext[5];
    shard->has_head = ext[6];
    shard->n_local = shard->l_end - shard->l_start;
    shard->n_layers_global = global_cfg->n_layers;
}

/* pt_shard.c:41-92: pointers for the owned parts only; absent parts NULL.
 * Per-layer tensors hold n_local layers. */
void pt_load_shard_weights(pt_weights_t *w, const pt_config_t *global_cfg,
                           const pt_shard_info_t *shard, void *data) {
    int shared = ((const int *)data)[5] > 0;
    sizes_t s = tensor_sizes(global_cfg);
    size_t n = (size_t)shard->n_local;
    float *p = (float *)((char *)data + 56);
    memset(w, 0, sizeof(*w));
    if (shard->has_embed) { w->token_embedding = p; p += s.emb; }
    if (n > 0) {
        w->rms_att_weight = p; p += n * s.rms;
        w->wq = p;             p += n * s.attn_q;
        w->wk = p;             p += n * s.attn_kv;
        w->wv = p;             p += n * s.attn_kv;
        w->wo = p;             p += n * s.attn_q;
        w->rms_ffn_weight = p; p += n * s.rms;
        w->w1 = p;             p += n * s.ffn;
        w->w2 = p;             p += n * s.ffn;
        w->w3 = p;             p += n * s.ffn;
    }
    if (shard->has_head) { w->rms_final_weight = p; p += s.rms_final; }
    p += 2 * s.freq;
    if (shard->has_head) w->wcls = shared ? w->token_embedding : p;
}

/* pt_shard.c:94-130 */
unsigned pt_shard_file_size(const void *data) {
    pt_config_t c;
    pt_shard_info_t sh;
    pt_load_shard_header(&c, &sh, data);
    int shared = ((const int *)data)[5] > 0;
    sizes_t s = tensor_sizes(&c);
    size_t n = 0;
    if (sh.has_embed) n += s.emb;
    if (sh.n_local > 0) n += (size_t)sh.n_local * layer_floats(&s);
    if (sh.has_head) n += s.rms_final;
    n += 2 * s.freq;
    if (sh.has_head && !shared) n += s.emb;
    return (unsigned)(56 + 4 * n);
}

/* tools/shard_weights.py:49-66 */
static void assign_layers(int n_layers, int rank, int world, int *l0, int *l1, int *emb, int *head) {
    if (world == 1) { *l0 = 0; *l1 = n_layers; *emb = 1; *head = 1; return; }
    if (rank == world - 1) { *l0 = *l1 = n_layers; *emb = 1; *head = 1; return; }
    int compute = world - 1, base = n_layers / compute, extra = n_layers % compute;
    int off = 0;
    for (int r = 0; r < rank; r++) off += base + (r < extra ? 1 : 0);
    *l0 = off;
    *l1 = off + base + (rank < extra ? 1 : 0);
    *emb = 0;
    *head = 0;
}

/* Copies `count` floats per layer for layers [l0, l1) out of a tensor that
 * stores all `L` layers contiguously. */
static char *put_layers(char *dst, const float *src, size_t per_layer, int l0, int l1) {
    size_t bytes = per_layer * (size_t)(l1 - l0) * 4;
    memcpy(dst, src + per_layer * (size_t)l0, bytes);
    return dst + bytes;
}

unsigned long pt_make_shard(const void *full_bin, int rank, int world_size, void *out,
                            unsigned long out_cap) {
    pt_config_t c;
    pt_weights_t w;
    pt_load_config(&c, full_bin);
    pt_load_weights(&w, &c, (void *)full_bin);
    int shared = ((const int *)full_bin)[5] > 0;
    if (world_size < 1 || rank < 0 || rank >= world_size) return 0;
    int l0, l1, emb, head;
    assign_layers(c.n_layers, rank, world_size, &l0, &l1, &emb, &head);
    sizes_t s = tensor_sizes(&c);
    size_t n = 0;
    if (emb) n += s.emb;
    if (l1 > l0) n += (size_t)(l1 - l0) * layer_floats(&s);
    if (head) n += s.rms_final;
    n += 2 * s.freq;
    if (head && !shared) n += s.emb;
    unsigned long total = 56 + 4 * n;
    if (total > out_cap) return 0;
    char *o = (char *)out;
    memcpy(o, full_bin, 28);
    int ext[7] = {(int)PT_SHARD_MAGIC, rank, world_size, l0, l1, emb, head};
    memcpy(o + 28, ext, 28);
    char *p = o + 56;
    if (emb) { memcpy(p, w.token_embedding, s.emb * 4); p += s.emb * 4; }
    if (l1 > l0) {
        p = put_layers(p, w.rms_att_weight, s.rms, l0, l1);
        p = put_layers(p, w.wq, s.attn_q, l0, l1);
        p = put_layers(p, w.wk, s.attn_kv, l0, l1);
        p = put_layers(p, w.wv, s.attn_kv, l0, l1);
        p = put_layers(p, w.wo, s.attn_q, l0, l1);
        p = put_layers(p, w.rms_ffn_weight, s.rms, l0, l1);
        p = put_layers(p, w.w1, s.ffn, l0, l1);
        p = put_layers(p, w.w2, s.ffn, l0, l1);
        p = put_layers(p, w.w3, s.ffn, l0, l1);
    }
    if (head) { memcpy(p, w.rms_final_weight, s.rms_final * 4); p += s.rms_final * 4; }
    memcpy(p, w.rms_final_weight + s.rms_final, 2 * s.freq * 4);
    p += 2 * s.freq * 4;
    if (head && !shared) { memcpy(p, w.wcls, s.emb * 4); p += s.emb * 4; }
    return (unsigned long)(p - o);
}

/* pt_ops.c:65-70 */
int pt_argmax(const float *x, int n) {
    int best = 0;
    for (int i = 1; i < n; i++)
        if (x[i] > x[best]) best = i;
    return best;
}
