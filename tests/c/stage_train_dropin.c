/*
 * A C caller of pitorch's low-level training API that owns its structs, as
 * the reference's own host programs do (they allocate pt_activations_t,
 * pt_grads_t and pt_backward_buf_t with the pt_alloc_* calls and drive the
 * staged forward, backward and SGD themselves: pitorch/train/pt_train.h,
 * used by dev/host/test_stage_train.c). Compiled against include/ and linked
 * to libpitorch_b200.so by tests/test_train_dropin_gpu.py.
 *
 *   stage_train_dropin <model.bin> <tokens.i32> <T> <steps> <lr> <split>
 *
 * Three copies of the same weights train side by side, each step:
 *   mono    pt_forward_train -> pt_backward -> pt_sgd_update
 *   staged  the same through the staged calls, layers split at `split`
 *   pp      a two-stage pipeline with its own weight copy per stage: stage 0
 *           holds the embedding, layers [0, split) and the head, stage 1
 *           layers [split, L); the [T, dim] residual rows and d_res are
 *           handed over by memcpy between the stages' host arrays
 * and the program checks that staged and pp give mono's loss bit for bit
 * and that staged leaves mono's weight image byte for byte. One line per
 * step: "step <k> <loss>"; then "OK" or "FAIL <why>" (exit status 1).
 */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "llama2.h"
#include "pt_train.h"

static void *read_all(const char *path, long *n) {
    FILE *f = fopen(path, "rb");
    if (!f) { perror(path); exit(2); }
    fseek(f, 0, SEEK_END);
    *n = ftell(f);
    fseek(f, 0, SEEK_SET);
    void *p = malloc((size_t)*n);
    if (fread(p, 1, (size_t)*n, f) != (size_t)*n) { perror(path); exit(2); }
    fclose(f);
    return p;
}

typedef struct {
    void *image;
    pt_weights_t w;
    pt_activations_t a;
    pt_grads_t g;
    pt_backward_buf_t b;
} replica_t;

static void replica_open(replica_t *r, const void *image, long bytes, const pt_config_t *cfg, int T) {
    r->image = malloc((size_t)bytes);
    memcpy(r->image, image, (size_t)bytes);
    pt_load_weights(&r->w, cfg, r->image);
    pt_alloc_activations(&r->a, cfg, T);
    pt_alloc_grads(&r->g, cfg, ((const int *)image)[5] > 0);
    pt_alloc_backward_buf(&r->b, cfg, T);
}

static void replica_close(replica_t *r) {
    pt_free_activations(&r->a);
    pt_free_grads(&r->g);
    pt_free_backward_buf(&r->b);
    free(r->image);
}

int main(int argc, char **argv) {
    if (argc != 7) {
        fprintf(stderr, "usage: %s <model.bin> <tokens.i32> <T> <steps> <lr> <split>\n", argv[0]);
        return 2;
    }
    long bytes = 0, tbytes = 0;
    void *image = read_all(argv[1], &bytes);
    int *tokens = (int *)read_all(argv[2], &tbytes);
    const int T = atoi(argv[3]), steps = atoi(argv[4]), split = atoi(argv[6]);
    const float lr = (float)atof(argv[5]);
    if ((long)T * 4 > tbytes) { fprintf(stderr, "tokens file holds fewer than T tokens\n"); return 2; }
    pt_config_t cfg;
    pt_load_config(&cfg, image);
    const int L = cfg.n_layers, dim = cfg.dim;
    const size_t rows = (size_t)T * dim * sizeof(float);

    replica_t mono, stg, s0, s1;
    replica_open(&mono, image, bytes, &cfg, T);
    replica_open(&stg, image, bytes, &cfg, T);
    replica_open(&s0, image, bytes, &cfg, T);
    replica_open(&s1, image, bytes, &cfg, T);

    int ok = 1;
    for (int k = 0; k < steps && ok; k++) {
        pt_zero_grads(&mono.g);
        const float loss = pt_forward_train(&cfg, &mono.w, &mono.a, tokens, T, NULL, NULL);
        pt_backward(&cfg, &mono.w, &mono.g, &mono.a, &mono.b, tokens, T, NULL, NULL);
        pt_sgd_update(&mono.w, &mono.g, lr, &cfg);

        pt_zero_grads(&stg.g);
        pt_forward_train_embed(&stg.w, &stg.a, tokens, T, dim);
        pt_forward_train_layers_range(&cfg, &stg.w, &stg.a, T, 0, split, NULL, NULL);
        pt_forward_train_layers_range(&cfg, &stg.w, &stg.a, T, split, L, NULL, NULL);
        const float loss_stg = pt_forward_train_head(&cfg, &stg.w, &stg.a, tokens, T, NULL, NULL);
        pt_backward_head(&cfg, &stg.w, &stg.g, &stg.a, &stg.b, tokens, T, NULL, NULL);
        pt_backward_layers_range(&cfg, &stg.w, &stg.g, &stg.a, &stg.b, T, split, L, NULL, NULL);
        pt_backward_layers_range(&cfg, &stg.w, &stg.g, &stg.a, &stg.b, T, 0, split, NULL, NULL);
        pt_backward_embed(&stg.g, &stg.b, tokens, T, dim);
        pt_sgd_update_head(&stg.w, &stg.g, lr, &cfg);
        pt_sgd_update_layers(&stg.w, &stg.g, lr, &cfg, 0, split);
        pt_sgd_update_layers(&stg.w, &stg.g, lr, &cfg, split, L);

        pt_zero_grads(&s0.g);
        pt_zero_grads(&s1.g);
        pt_forward_train_embed(&s0.w, &s0.a, tokens, T, dim);
        pt_forward_train_layers_range(&cfg, &s0.w, &s0.a, T, 0, split, NULL, NULL);
        memcpy(s1.a.residuals + (size_t)split * T * dim, s0.a.residuals + (size_t)split * T * dim, rows);
        pt_forward_train_layers_range(&cfg, &s1.w, &s1.a, T, split, L, NULL, NULL);
        memcpy(s0.a.residuals + (size_t)L * T * dim, s1.a.residuals + (size_t)L * T * dim, rows);
        const float loss_pp = pt_forward_train_head(&cfg, &s0.w, &s0.a, tokens, T, NULL, NULL);
        pt_backward_head(&cfg, &s0.w, &s0.g, &s0.a, &s0.b, tokens, T, NULL, NULL);
        memcpy(s1.b.d_res, s0.b.d_res, rows);
        pt_backward_layers_range(&cfg, &s1.w, &s1.g, &s1.a, &s1.b, T, split, L, NULL, NULL);
        memcpy(s0.b.d_res, s1.b.d_res, rows);
        pt_backward_layers_range(&cfg, &s0.w, &s0.g, &s0.a, &s0.b, T, 0, split, NULL, NULL);
        pt_backward_embed(&s0.g, &s0.b, tokens, T, dim);
        pt_sgd_update_head(&s0.w, &s0.g, lr, &cfg);
        pt_sgd_update_layers(&s0.w, &s0.g, lr, &cfg, 0, split);
        pt_sgd_update_layers(&s1.w, &s1.g, lr, &cfg, split, L);

        printf("step %d %.9g\n", k, (double)loss);
        if (loss_stg != loss) { printf("FAIL staged loss %.9g != %.9g at step %d\n", loss_stg, loss, k); ok = 0; }
        else if (loss_pp != loss) { printf("FAIL pipeline loss %.9g != %.9g at step %d\n", loss_pp, loss, k); ok = 0; }
        else if (memcmp(mono.image, stg.image, (size_t)bytes) != 0) { printf("FAIL staged image differs at step %d\n", k); ok = 0; }
    }
    /* the gradients a caller reads after a backward sequence */
    if (ok) {
        for (int i = 0; i < mono.g._n_params && ok; i++)
            if (mono.g._mem[i] != stg.g._mem[i]) { printf("FAIL gradient %d differs\n", i); ok = 0; }
    }
    replica_close(&mono);
    replica_close(&stg);
    replica_close(&s0);
    replica_close(&s1);
    free(image);
    free(tokens);
    if (ok) printf("OK\n");
    return ok ? 0 : 1;
}
