// ptc_persist.h -- internal interface of the persistent decode kernel.
#pragma once

#include <cuda_runtime.h>

#include "ptc_decode.cuh"

namespace ptc {

constexpr int PS_STAGES = 6;          // shared-memory weight stages of MV_STAGE_BYTES
constexpr int PS_MAX_DIM = 2048;      // model dim
constexpr int PS_MAX_HBLOCK = 64;     // hidden units per CTA
constexpr int PS_MAX_ITEM_POS = 128;  // positions per attention item
constexpr int PS_STAT_FLOATS = 320;   // attention merge scratch in shared memory
constexpr int PS_PART_FLOATS = 9984;  // staged attention partials (items x (hd + 2))
constexpr int PS_MAX_WO_ROWS = 32;    // wo rows per CTA (residual prefetch)

struct PersistArgs {
    DecodeModel m;
    const float *w2t;   // [L][hidden][dim] transposed w2
    float *x1;          // [dim] post-attention residual (FFN input)
    float *att_part;    // [nh][max_chunks][hd + 2] attention partials
    int max_chunks;     // attention chunks per head capacity (= G / nh)
    unsigned *bar;      // grid barrier counter, zeroed before each launch
    int n_steps;        // positions decoded by this launch
    int has_embed, has_head;
    // Optional phase timeline (block 0): trace[2k] = %globaltimer when the
    // CTA finished phase k's work, trace[2k+1] = when barrier k released.
    unsigned long long *trace;
    int trace_cap;      // entries available (2 per barrier)
};

bool persist_supported(const DecodeModel &m, int n_sm);
size_t persist_smem_bytes(const DecodeModel &m);
void persist_transpose_w2(const DecodeModel &m, float *w2t, cudaStream_t s);
void persist_launch(const PersistArgs &a, int n_sm, cudaStream_t s);

}  // namespace ptc
