// ptc_gemm.h -- internal interface of the fp32 training GEMM.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>

namespace ptc {

enum GemmEpilogue {
    EPI_STORE = 0,  // C = A.B
    EPI_ACCUM = 1,  // C += A.B          (weight gradients accumulate)
    EPI_RESID = 2,  // C = R + A.B       (residual adds of the forward pass)
    EPI_ROPE = 3,   // C = RoPE_row(A.B) (q/k projections; row index = position)
};

struct GemmArgs {
    int M, N, K;
    const float *A;
    int lda;
    bool a_kcontig;   // A(m,k) = A[m*lda+k] if true, else A[k*lda+m]
    const float *B;
    int ldb;
    bool b_kcontig;   // B(k,n) = B[n*ldb+k] if true, else B[k*ldb+n]
    float *C;
    int ldc;
    const float *R;   // residual input (EPI_RESID)
    int ldr;
    int epi;
    int rope_hd;      // head_dim for EPI_ROPE
    float *partial;   // split-K workspace (may be null: no split)
    size_t partial_cap;  // floats available in `partial`
    int splits;       // set by gemm()
    int no_alloc;     // 1: no allocation may happen (keeps the product off the
                      // tensor-core kernel, whose workspace is allocated on demand)
    int cluster_red;  // set by gemm(): the splits of a tile form a thread-block
                      // cluster and sum their partials through distributed
                      // shared memory (no workspace, no reduction kernel)
};

void gemm(GemmArgs g, int n_sm, cudaStream_t s);

// Per-process launch counters of the GEMM paths (ptc_gemm_counters):
// tensor-core kernels, SIMT tile kernels, split-K reduction kernels, and
// SIMT launches whose splits were summed inside a cluster.
enum GemmCounter { GC_TENSOR_CORE = 0, GC_SIMT = 1, GC_SPLITK_REDUCE = 2, GC_CLUSTER_REDUCED = 3, GC_N = 4 };
void gemm_count(int which);

// Fixed-order sum of g.splits partials from g.partial into C with g's epilogue.
void launch_splitk_reduce(const GemmArgs &g, int n_sm, cudaStream_t s);

// Tensor-core fp32 GEMM (ptc_gemm_tc.cu), used by gemm() for the large
// products unless PTC_GEMM_TC=0; returns false when it does not take g.
bool gemm_tc_enabled();
// PTC_GEMM_TC=1: every product that qualifies must run on the tensor cores
// (a CUTLASS refusal is then fatal instead of falling back).
bool gemm_tc_required();
bool gemm_tc(const GemmArgs &g, int n_sm, cudaStream_t s);

}  // namespace ptc
