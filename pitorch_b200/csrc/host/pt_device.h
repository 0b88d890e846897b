/* pt_device.h -- private host-side view of a context's device resources. */
#ifndef PT_DEVICE_H
#define PT_DEVICE_H

#include <stddef.h>

#include "../../../include/pt.h"
#include "../../../include/ptc.h"

struct ptc_trainer;

struct pt_device {
    ptc_ctx *ctx;
    const char *host_image;  /* caller's blob (byte 0 of the header) */
    char *dev_image;         /* device copy of byte 0 */
    size_t image_bytes;
    ptc_config cfg;          /* local config (n_layers = owned layers) */
    ptc_weights dw;          /* device weight pointers */
    ptc_decoder *dec;
    int has_embed, has_head;
    int is_shard;
    pt_shard_info_t shard;
    struct ptc_trainer *trainer;
    int owns_ctx;
};

/* Translate a host pointer inside the uploaded image to its device copy. */
const float *pt_dev_ptr(const struct pt_device *d, const float *host);

/* Create the device side for a (global or shard) image. */
struct pt_device *pt_device_open(const void *image, size_t image_bytes, size_t header_bytes,
                                 const pt_config_t *local_cfg, const pt_weights_t *host_w,
                                 int has_embed, int has_head, int device, size_t arena_bytes,
                                 int max_T);
void pt_device_close(struct pt_device *d);

/* Device selection: num_qpus if it names a visible device, else $PT_DEVICE, else 0. */
int pt_pick_device(int requested);

void pt_fatal(const char *fmt, ...);

/* The device twin of a host decode state (created on first use). */
struct pt_device *pt_state_device(const pt_config_t *cfg, const pt_weights_t *w, pt_state_t *s);

#endif
