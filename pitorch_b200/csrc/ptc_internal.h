// ptc_internal.h -- declarations shared between the CUDA translation units
// of libpitorch_b200 (not part of the C ABI).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>

#include "../../include/ptc.h"

struct ptc_chunk {
    void *base;
    size_t size;
    size_t used;
};

bool ptc_lookup_range(const void *host, size_t bytes, const void **dev, ptc_ctx **owner);
cudaStream_t ptc_ctx_stream(ptc_ctx *c);
int ptc_ctx_device(ptc_ctx *c);

namespace ptc {
// Grants `kernel` at least `smem` bytes of dynamic shared memory and the
// maximal shared-memory carveout on the current device. cudaFuncSetAttribute
// acts on one device, so what each (kernel, device) pair was granted is
// remembered per pair; thread-safe.
void ensure_kernel_smem(const void *kernel, size_t smem);
struct DecodeModel;
// Layers [l0, l1) of one decode position; the range reads and leaves x in m.x.
void launch_layers(const DecodeModel &m, int l0, int l1, bool from_embedding, int n_sm, cudaStream_t s);
int decode_ffn_rows(int dim, int hidden, int n_sm);
void launch_block(const DecodeModel &m, int kind, int l, int n_sm, cudaStream_t s);
int decode_attn_stage(int dim, int nh, int nkv, int seq);
void build_rope_table(float2 *t, int seq, int hd, cudaStream_t s);
void transpose_w2(const DecodeModel &m, float *w2t, cudaStream_t s);
// host_next: pinned host word that also receives the argmax (or null).
void launch_head(const DecodeModel &m, int n_sm, cudaStream_t s, int *host_next = nullptr);
void launch_embed(const DecodeModel &m, cudaStream_t s);
// A pipeline layer rank's output x into the next stage's mailbox.
void launch_stage_send(const DecodeModel &m, cudaStream_t s);
int decode_attn_limits_ok(int hd, int chunk, int n_chunks);
void launch_matvec(const float *W, const float *x, float *y, int rows, int cols, cudaStream_t s);
}  // namespace ptc
