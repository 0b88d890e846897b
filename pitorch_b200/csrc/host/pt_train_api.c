/*
 * pt_train_api.c -- training entry points (pitorch/pt.c:339-364,
 * pitorch/train/pt_train.h). The device trainer is not part of this build
 * yet: contexts created with max_T > 0 abort with a message rather than
 * computing anything on the host.
 */
#include <stdlib.h>
#include <string.h>

#include "pt_device.h"

void pt_train_init(pt_context_t *ctx, int max_T) {
    (void)ctx;
    (void)max_T;
    pt_fatal("training (max_T > 0) is not available in this build");
}

void pt_train_free(pt_context_t *ctx) { (void)ctx; }

float pt_train_step(pt_context_t *ctx, const int *tokens, int T, float lr) {
    (void)ctx; (void)tokens; (void)T; (void)lr;
    pt_fatal("pt_train_step: training is not available in this build");
    return 0.0f;
}

void pt_sync_weights(pt_context_t *ctx) { (void)ctx; }
void pt_sync_grads(pt_context_t *ctx) { (void)ctx; }
