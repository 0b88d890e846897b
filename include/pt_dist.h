#ifndef PT_DIST_H
#define PT_DIST_H

/*
 * Distributed context for the layer pipeline -- drop-in for
 * pitorch/dist/pt_dist.h. The reference wires Pi Zeros into a ring with two
 * GPIO links per board (pt_dist.h:15-22); here each rank is one process
 * driving one GPU, and the links are an NCCL communicator over NVLink /
 * NVSwitch (send/recv to the next and previous rank of the same ring).
 *
 * Ring order is the reference's: the last rank holds embedding + classifier
 * (tools/shard_weights.py:49-66); rank 0..world-2 hold consecutive layer
 * ranges; activations flow embed(W-1) -> 0 -> 1 -> ... -> W-2 -> head(W-1).
 */

typedef struct {
    int rank, world_size;
    int l_start, l_end;     /* layer range [l_start, l_end), local indices */
    int has_embed;
    int has_head;
    /* replaces the two pt_link_gpio_t links: the rank's communicator */
    void *comm;             /* opaque (NCCL), created by pt_dist_setup */
    int timeout_ms;         /* bound on every wait (0 = 300 s, the GPIO first-byte timeout) */
} pt_dist_t;

#endif
