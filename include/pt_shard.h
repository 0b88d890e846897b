#ifndef PT_SHARD_H
#define PT_SHARD_H

/*
 * Weight shard files for the layer pipeline -- drop-in for
 * pitorch/model/pt_shard.h. Format (pitorch/model/pt_shard.c:15-130,
 * tools/shard_weights.py:1-23): the 28-byte llama2.c header with the GLOBAL
 * config, a 28-byte extension {magic "SHRD", rank, world_size, l_start,
 * l_end, has_embed, has_head}, then [embedding] [local layers] [rms_final]
 * freq_cis [wcls if untied and has_head].
 */

#include "llama2.h"

#define PT_SHARD_MAGIC  0x53485244  /* "SHRD" */

/* pitorch/model/pt_shard.h:21-30 */
typedef struct {
    int rank;
    int world_size;
    int l_start;
    int l_end;
    int n_local;
    int has_embed;
    int has_head;
    int n_layers_global;
} pt_shard_info_t;

/* pitorch/model/pt_shard.h:38-57. pt_load_shard_header aborts with a message
 * when the magic is missing (the reference panics). */
void pt_load_shard_header(pt_config_t *global_cfg, pt_shard_info_t *shard, const void *data);
void pt_load_shard_weights(pt_weights_t *w, const pt_config_t *global_cfg,
                           const pt_shard_info_t *shard, void *data);
unsigned pt_shard_file_size(const void *data);

/* Write the shard of `rank` (of world_size) cut from a full .bin image into
 * `out` (capacity out_cap bytes); returns the shard size, or 0 if out_cap is
 * too small. Layer assignment of tools/shard_weights.py:49-66: the last rank
 * holds embedding + head and no layers, the others split the layers evenly,
 * earlier ranks taking the remainder. world_size == 1 gives one shard with
 * everything. */
unsigned long pt_make_shard(const void *full_bin, int rank, int world_size,
                            void *out, unsigned long out_cap);

#endif
