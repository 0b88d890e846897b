// ptc_gemm.cu -- shared-memory-tiled fp32 GEMM for the training step.
//
// Replaces, for the batched training passes, the per-position matvecs of
// pitorch/train/pt_train.c (forward: 7 matvecs per layer per position,
// :204-303; input grads: transposed matvecs, :442-453) and its CPU weight
// gradient matmul_backward_weight_batched (:475-492), whose QPU counterpart
// sgemm_rect_tmu (pitorch/ops/gemm/gemm_rect.c:28-104) ships compiled out.
//
// C[m][n] = sum_k A(m,k) B(k,n) in fp32 with fp32 accumulation, for the three
// layouts a linear layer needs (W is [out, in] row-major):
//   forward   Y[T,out]  = X[T,in] . W^T     A k-contiguous, B k-contiguous
//   input gr. dX[T,in]  = dY[T,out] . W     A k-contiguous, B n-contiguous
//   weight gr dW[out,in] += dY^T . X        A m-contiguous, B n-contiguous
// Tiles of A and B are staged k-major in shared memory (double-buffered,
// 128-bit global loads where the layout allows), each thread accumulates a
// TMxTN register block. Long-K products (the classifier input gradient,
// K = vocab) are split over K into a partial buffer and reduced in a fixed
// order, so results are deterministic.
#include "ptc_common.cuh"
#include "ptc_gemm.h"

#include <cooperative_groups.h>
#include <string.h>

#include <atomic>

#include "../../include/ptc.h"

namespace ptc {

static std::atomic<long long> g_gemm_counts[GC_N];

void gemm_count(int which) { g_gemm_counts[which].fetch_add(1, std::memory_order_relaxed); }

namespace cg = cooperative_groups;

// One reduced element pair (m, n), (m, n + 1) through the product's epilogue
// (n even; N is even for RoPE products, so pairs never straddle rows).
__device__ __forceinline__ void store_pair(const GemmArgs &g, int m, int n, float v0, float v1) {
    if (g.epi == EPI_ROPE) {
        if (n + 1 >= g.N) return;
        const float th = rope_theta(n, g.rope_hd, m);
        const float cs = pt_cosf(th), sn = pt_sinf(th);
        float *c = g.C + (size_t)m * g.ldc + n;
        c[0] = __fsub_rn(__fmul_rn(v0, cs), __fmul_rn(v1, sn));
        c[1] = __fadd_rn(__fmul_rn(v0, sn), __fmul_rn(v1, cs));
        return;
    }
    const float v[2] = {v0, v1};
#pragma unroll
    for (int j = 0; j < 2; j++) {
        if (n + j >= g.N) continue;
        float *c = g.C + (size_t)m * g.ldc + n + j;
        switch (g.epi) {
            case EPI_STORE: *c = v[j]; break;
            case EPI_ACCUM: *c = *c + v[j]; break;
            case EPI_RESID: *c = __fadd_rn(g.R[(size_t)m * g.ldr + n + j], v[j]); break;
            default: *c = v[j]; break;
        }
    }
}

// Split-K inside a thread-block cluster: the cluster's CTAs are the splits of
// one BM x BN tile. Each parks its partial tile in its own (free) staging
// buffer; after a cluster barrier CTA r sums rows [r*BM/cs, (r+1)*BM/cs) of
// all partials in split order -- the order of k_splitk_reduce, so results
// are the same bit for bit -- and stores them through the epilogue.
template <int BM, int BN, int TM, int TN, int NT>
__device__ __forceinline__ void cluster_reduce(const GemmArgs &g, const float (&acc)[TM][TN], float *tile, int m0,
                                               int n0, int tx, int ty) {
#pragma unroll
    for (int i = 0; i < TM; i++)
#pragma unroll
        for (int j = 0; j < TN; j += 4)
            *reinterpret_cast<float4 *>(&tile[(ty * TM + i) * BN + tx * TN + j]) =
                make_float4(acc[i][j], acc[i][j + 1], acc[i][j + 2], acc[i][j + 3]);
    cg::cluster_group cl = cg::this_cluster();
    cl.sync();
    const int cs = (int)cl.num_blocks(), rank = (int)cl.block_rank();
    const int rows = BM / cs, r0 = rank * rows;
    for (int e = 2 * (int)threadIdx.x; e < rows * BN; e += 2 * NT) {
        const int rr = r0 + e / BN, cc = e % BN;
        const int m = m0 + rr, n = n0 + cc;
        float v0 = 0.f, v1 = 0.f;
        for (int s = 0; s < cs; s++) {
            const float *p = cl.map_shared_rank(tile, s) + rr * BN + cc;
            v0 += p[0];
            v1 += p[1];
        }
        if (m < g.M && n < g.N) store_pair(g, m, n, v0, v1);
    }
    cl.sync();   // no CTA leaves while another still reads its tile
}

// Store a thread's TM x TN block (rows mb.., columns nb..) with the
// product's epilogue, or into the split-K partial buffer.
template <int TM, int TN>
__device__ __forceinline__ void gemm_epilogue(const GemmArgs &g, const float (&acc)[TM][TN], int mb, int nb,
                                              int split) {
#pragma unroll
    for (int i = 0; i < TM; i++) {
        const int m = mb + i;
        if (m >= g.M) continue;
#pragma unroll
        for (int j = 0; j < TN; j++) {
            const int n = nb + j;
            if (n >= g.N) continue;
            const float v = acc[i][j];
            if (g.splits > 1) {
                g.partial[((size_t)split * g.M + m) * g.N + n] = v;
                continue;
            }
            float *c = g.C + (size_t)m * g.ldc + n;
            switch (g.epi) {
                case EPI_STORE: *c = v; break;
                case EPI_ACCUM: *c = *c + v; break;
                case EPI_RESID: *c = __fadd_rn(g.R[(size_t)m * g.ldr + n], v); break;
            }
        }
    }
    // RoPE epilogue (q/k projections): pairs (n, n+1) are held by the same
    // thread since TN is even and tiles start at even n.
    if (g.epi == EPI_ROPE && g.splits == 1) {
#pragma unroll
        for (int i = 0; i < TM; i++) {
            const int m = mb + i;
            if (m >= g.M) continue;
#pragma unroll
            for (int j = 0; j < TN; j += 2) {
                const int n = nb + j;
                if (n + 1 >= g.N) continue;
                const float th = rope_theta(n, g.rope_hd, m);
                const float cs = pt_cosf(th), sn = pt_sinf(th);
                const float a0 = acc[i][j], a1 = acc[i][j + 1];
                float *c = g.C + (size_t)m * g.ldc + n;
                c[0] = __fsub_rn(__fmul_rn(a0, cs), __fmul_rn(a1, sn));
                c[1] = __fadd_rn(__fmul_rn(a0, sn), __fmul_rn(a1, cs));
            }
        }
    }
}

template <int BM, int BN, int BK, int TM, int TN, bool A_KC, bool B_KC>
__global__ void __launch_bounds__((BM / TM) * (BN / TN))
    k_gemm(GemmArgs g) {
    constexpr int NT = (BM / TM) * (BN / TN);
    __shared__ __align__(16) float As[2][BK][BM + 4];
    __shared__ __align__(16) float Bs[2][BK][BN + 4];

    const int tid = threadIdx.x;
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    const int split = blockIdx.z;
    const int kper = (g.K + g.splits - 1) / g.splits;
    const int kbeg = split * kper;
    const int kend = min(g.K, kbeg + kper);

    const int tx = tid % (BN / TN), ty = tid / (BN / TN);
    float acc[TM][TN];
#pragma unroll
    for (int i = 0; i < TM; i++)
#pragma unroll
        for (int j = 0; j < TN; j++) acc[i][j] = 0.f;

    auto loadA = [&](int buf, int k0) {
        if (A_KC) {
            // A(m,k) = A[m*lda + k]: BM rows x BK cols, read along k.
            for (int e = tid; e < BM * BK; e += NT) {
                const int r = e / BK, c = e % BK;
                const int m = m0 + r, k = k0 + c;
                As[buf][c][r] = (m < g.M && k < kend) ? __ldg(g.A + (size_t)m * g.lda + k) : 0.f;
            }
        } else {
            // A(m,k) = A[k*lda + m]: BK rows x BM cols, read along m.
            for (int e = tid; e < BM * BK; e += NT) {
                const int r = e / BM, c = e % BM;
                const int m = m0 + c, k = k0 + r;
                As[buf][r][c] = (m < g.M && k < kend) ? __ldg(g.A + (size_t)k * g.lda + m) : 0.f;
            }
        }
    };
    auto loadB = [&](int buf, int k0) {
        if (B_KC) {
            // B(k,n) = B[n*ldb + k]
            for (int e = tid; e < BN * BK; e += NT) {
                const int r = e / BK, c = e % BK;
                const int n = n0 + r, k = k0 + c;
                Bs[buf][c][r] = (n < g.N && k < kend) ? __ldg(g.B + (size_t)n * g.ldb + k) : 0.f;
            }
        } else {
            // B(k,n) = B[k*ldb + n]
            for (int e = tid; e < BN * BK; e += NT) {
                const int r = e / BN, c = e % BN;
                const int n = n0 + c, k = k0 + r;
                Bs[buf][r][c] = (n < g.N && k < kend) ? __ldg(g.B + (size_t)k * g.ldb + n) : 0.f;
            }
        }
    };

    int buf = 0;
    if (kbeg < kend) {
        loadA(0, kbeg);
        loadB(0, kbeg);
    }
    __syncthreads();
    for (int k0 = kbeg; k0 < kend; k0 += BK) {
        if (k0 + BK < kend) {
            loadA(buf ^ 1, k0 + BK);
            loadB(buf ^ 1, k0 + BK);
        }
#pragma unroll
        for (int kk = 0; kk < BK; kk++) {
            float a[TM], b[TN];
#pragma unroll
            for (int i = 0; i < TM; i++) a[i] = As[buf][kk][ty * TM + i];
#pragma unroll
            for (int j = 0; j < TN; j++) b[j] = Bs[buf][kk][tx * TN + j];
#pragma unroll
            for (int i = 0; i < TM; i++)
#pragma unroll
                for (int j = 0; j < TN; j++) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        __syncthreads();
        buf ^= 1;
    }

    gemm_epilogue<TM, TN>(g, acc, m0 + ty * TM, n0 + tx * TN, split);
}

// Vectorised variant for operands whose contiguous dimension and leading
// dimensions are multiples of 4 floats (every product of the training step):
// 128-bit global loads along the contiguous dimension, staged through
// registers into the next shared-memory buffer while the current one is
// used; 128-bit shared reads of the TM x TN operand fragments. K is split
// into chunks of kper (a multiple of BK) by blockIdx.z.
template <int BM, int BN, int BK, int TM, int TN, bool A_KC, bool B_KC>
__global__ void __launch_bounds__((BM / TM) * (BN / TN)) k_gemm_v(GemmArgs g, int kper) {
    constexpr int NT = (BM / TM) * (BN / TN);
    constexpr int A4 = BM * BK / 4 / NT, B4 = BN * BK / 4 / NT;
    static_assert(A4 >= 1 && B4 >= 1 && A4 * 4 * NT == BM * BK && B4 * 4 * NT == BN * BK, "tile / threads");
    constexpr int SA = 2 * BK * (BM + 4), SB = 2 * BK * (BN + 4);
    __shared__ __align__(16) float sbuf[SA + SB];
    auto As = reinterpret_cast<float (*)[BK][BM + 4]>(sbuf);
    auto Bs = reinterpret_cast<float (*)[BK][BN + 4]>(sbuf + SA);
    const int tid = threadIdx.x;
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    const int split = blockIdx.z;
    const int kbeg = split * kper, kend = min(g.K, kbeg + kper);
    const int tx = tid % (BN / TN), ty = tid / (BN / TN);
    float4 ra[A4], rb[B4];
    const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);

    auto gload = [&](int k0) {
#pragma unroll
        for (int i = 0; i < A4; i++) {
            const int e = tid + i * NT;
            if (A_KC) {   // BM rows of BK/4 float4 along k
                const int r = e / (BK / 4), c = e % (BK / 4), m = m0 + r, k = k0 + 4 * c;
                ra[i] = (m < g.M && k < kend) ? __ldg(reinterpret_cast<const float4 *>(g.A + (size_t)m * g.lda + k))
                                              : zero;
            } else {      // BK rows (k) of BM/4 float4 along m
                const int r = e / (BM / 4), c = e % (BM / 4), k = k0 + r, m = m0 + 4 * c;
                ra[i] = (k < kend && m < g.M) ? __ldg(reinterpret_cast<const float4 *>(g.A + (size_t)k * g.lda + m))
                                              : zero;
            }
        }
#pragma unroll
        for (int i = 0; i < B4; i++) {
            const int e = tid + i * NT;
            if (B_KC) {
                const int r = e / (BK / 4), c = e % (BK / 4), n = n0 + r, k = k0 + 4 * c;
                rb[i] = (n < g.N && k < kend) ? __ldg(reinterpret_cast<const float4 *>(g.B + (size_t)n * g.ldb + k))
                                              : zero;
            } else {
                const int r = e / (BN / 4), c = e % (BN / 4), k = k0 + r, n = n0 + 4 * c;
                rb[i] = (k < kend && n < g.N) ? __ldg(reinterpret_cast<const float4 *>(g.B + (size_t)k * g.ldb + n))
                                              : zero;
            }
        }
    };
    auto sstore = [&](int buf) {
#pragma unroll
        for (int i = 0; i < A4; i++) {
            const int e = tid + i * NT;
            if (A_KC) {
                const int r = e / (BK / 4), c = e % (BK / 4);
                As[buf][4 * c + 0][r] = ra[i].x;
                As[buf][4 * c + 1][r] = ra[i].y;
                As[buf][4 * c + 2][r] = ra[i].z;
                As[buf][4 * c + 3][r] = ra[i].w;
            } else {
                const int r = e / (BM / 4), c = e % (BM / 4);
                *reinterpret_cast<float4 *>(&As[buf][r][4 * c]) = ra[i];
            }
        }
#pragma unroll
        for (int i = 0; i < B4; i++) {
            const int e = tid + i * NT;
            if (B_KC) {
                const int r = e / (BK / 4), c = e % (BK / 4);
                Bs[buf][4 * c + 0][r] = rb[i].x;
                Bs[buf][4 * c + 1][r] = rb[i].y;
                Bs[buf][4 * c + 2][r] = rb[i].z;
                Bs[buf][4 * c + 3][r] = rb[i].w;
            } else {
                const int r = e / (BN / 4), c = e % (BN / 4);
                *reinterpret_cast<float4 *>(&Bs[buf][r][4 * c]) = rb[i];
            }
        }
    };

    float acc[TM][TN];
#pragma unroll
    for (int i = 0; i < TM; i++)
#pragma unroll
        for (int j = 0; j < TN; j++) acc[i][j] = 0.f;
    if (kbeg < kend) {
        gload(kbeg);
        sstore(0);
    }
    __syncthreads();
    int buf = 0;
    for (int k0 = kbeg; k0 < kend; k0 += BK) {
        const bool more = k0 + BK < kend;
        if (more) gload(k0 + BK);
#pragma unroll
        for (int kk = 0; kk < BK; kk++) {
            float a[TM], b[TN];
#pragma unroll
            for (int q = 0; q < TM / 4; q++) {
                const float4 v = *reinterpret_cast<const float4 *>(&As[buf][kk][ty * TM + 4 * q]);
                a[4 * q] = v.x; a[4 * q + 1] = v.y; a[4 * q + 2] = v.z; a[4 * q + 3] = v.w;
            }
#pragma unroll
            for (int q = 0; q < TN / 4; q++) {
                const float4 v = *reinterpret_cast<const float4 *>(&Bs[buf][kk][tx * TN + 4 * q]);
                b[4 * q] = v.x; b[4 * q + 1] = v.y; b[4 * q + 2] = v.z; b[4 * q + 3] = v.w;
            }
#pragma unroll
            for (int i = 0; i < TM; i++)
#pragma unroll
                for (int j = 0; j < TN; j++) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        if (more) sstore(buf ^ 1);
        __syncthreads();
        buf ^= 1;
    }
    if constexpr (BM * BN <= SA + SB) {
        if (g.cluster_red) {   // the loop ended with a barrier: sbuf is free
            cluster_reduce<BM, BN, TM, TN, NT>(g, acc, sbuf, m0, n0, tx, ty);
            return;
        }
    }
    gemm_epilogue<TM, TN>(g, acc, m0 + ty * TM, n0 + tx * TN, split);
}

// Fixed-order reduction of split-K partials into C with the epilogue
// (RoPE rows rotate pairs (n, n+1), so that case walks pairs).
__global__ void k_splitk_reduce(GemmArgs g) {
    const size_t total = (size_t)g.M * g.N;
    if (g.epi == EPI_ROPE) {
        // N is even (a head dimension multiple), so pairs never straddle rows
        for (size_t e = 2 * (blockIdx.x * (size_t)blockDim.x + threadIdx.x); e < total;
             e += 2 * (size_t)gridDim.x * blockDim.x) {
            float v0 = 0.f, v1 = 0.f;
            for (int s = 0; s < g.splits; s++) {
                v0 += g.partial[(size_t)s * total + e];
                v1 += g.partial[(size_t)s * total + e + 1];
            }
            const int m = (int)(e / g.N), n = (int)(e % g.N);
            const float th = rope_theta(n, g.rope_hd, m);
            const float cs = pt_cosf(th), sn = pt_sinf(th);
            float *c = g.C + (size_t)m * g.ldc + n;
            c[0] = __fsub_rn(__fmul_rn(v0, cs), __fmul_rn(v1, sn));
            c[1] = __fadd_rn(__fmul_rn(v0, sn), __fmul_rn(v1, cs));
        }
        return;
    }
    for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < total;
         e += (size_t)gridDim.x * blockDim.x) {
        float v = 0.f;
        for (int s = 0; s < g.splits; s++) v += g.partial[(size_t)s * total + e];
        const int m = (int)(e / g.N), n = (int)(e % g.N);
        float *c = g.C + (size_t)m * g.ldc + n;
        switch (g.epi) {
            case EPI_STORE: *c = v; break;
            case EPI_ACCUM: *c = *c + v; break;
            case EPI_RESID: *c = __fadd_rn(g.R[(size_t)m * g.ldr + n], v); break;
            default: *c = v; break;
        }
    }
}

template <int BM, int BN, int BK, int TM, int TN>
static void launch_tile(const GemmArgs &g, cudaStream_t s) {
    dim3 grid((g.N + BN - 1) / BN, (g.M + BM - 1) / BM, g.splits);
    dim3 block((BM / TM) * (BN / TN));
    if (g.a_kcontig && g.b_kcontig) k_gemm<BM, BN, BK, TM, TN, true, true><<<grid, block, 0, s>>>(g);
    else if (g.a_kcontig) k_gemm<BM, BN, BK, TM, TN, true, false><<<grid, block, 0, s>>>(g);
    else if (g.b_kcontig) k_gemm<BM, BN, BK, TM, TN, false, true><<<grid, block, 0, s>>>(g);
    else k_gemm<BM, BN, BK, TM, TN, false, false><<<grid, block, 0, s>>>(g);
    PTC_CHECK(cudaGetLastError());
    gemm_count(GC_SIMT);
}

template <int BM, int BN, int BK, int TM, int TN, bool A_KC, bool B_KC>
static void launch_v(const GemmArgs &g, int kper, cudaStream_t s) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((g.N + BN - 1) / BN, (g.M + BM - 1) / BM, g.splits);
    cfg.blockDim = dim3((BM / TM) * (BN / TN));
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    if (g.cluster_red) {   // one cluster = the splits of one tile
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 1;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = g.splits;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    PTC_CHECK(cudaLaunchKernelEx(&cfg, k_gemm_v<BM, BN, BK, TM, TN, A_KC, B_KC>, g, kper));
    gemm_count(GC_SIMT);
    if (g.cluster_red) gemm_count(GC_CLUSTER_REDUCED);
}

template <int BM, int BN, int BK, int TM, int TN>
static void launch_tile_v(const GemmArgs &g, int kper, cudaStream_t s) {
    if (g.a_kcontig && g.b_kcontig) launch_v<BM, BN, BK, TM, TN, true, true>(g, kper, s);
    else if (g.a_kcontig) launch_v<BM, BN, BK, TM, TN, true, false>(g, kper, s);
    else if (g.b_kcontig) launch_v<BM, BN, BK, TM, TN, false, true>(g, kper, s);
    else launch_v<BM, BN, BK, TM, TN, false, false>(g, kper, s);
}

static bool aligned16(const void *p) { return ((uintptr_t)p & 15) == 0; }

void launch_splitk_reduce(const GemmArgs &g, int n_sm, cudaStream_t s) {
    int blocks = (int)(((size_t)g.M * g.N + 255) / 256);
    if (blocks > 8 * n_sm) blocks = 8 * n_sm;
    k_splitk_reduce<<<blocks, 256, 0, s>>>(g);
    PTC_CHECK(cudaGetLastError());
    gemm_count(GC_SPLITK_REDUCE);
}

// The vectorised kernel reads float4s along each operand's contiguous
// dimension: that dimension (K for a k-contiguous operand, else M or N) and
// the leading dimensions must be multiples of 4, the bases 16-byte aligned.
static bool vec_ok(const GemmArgs &g) {
    if (g.lda % 4 || g.ldb % 4) return false;
    if (g.a_kcontig ? g.K % 4 : g.M % 4) return false;
    if (g.b_kcontig ? g.K % 4 : g.N % 4) return false;
    return aligned16(g.A) && aligned16(g.B);
}

void gemm(GemmArgs g, int n_sm, cudaStream_t s) {
    if (g.M <= 0 || g.N <= 0) return;
    if (g.K <= 0) {
        if (g.epi == EPI_STORE) {
            for (int m = 0; m < g.M; m++)
                PTC_CHECK(cudaMemsetAsync(g.C + (size_t)m * g.ldc, 0, (size_t)g.N * 4, s));
        }
        return;
    }
    if (vec_ok(g)) {
        // The classifier's products (about 2.4 GFLOP each at 15M) on the
        // tensor cores; the layer products are too small to gain.
        if (gemm_tc_enabled() && !g.no_alloc && (double)g.M * g.N * g.K >= 1e9 && aligned16(g.C) &&
            (g.epi != EPI_RESID || aligned16(g.R)) && g.ldc % 4 == 0 && (g.epi != EPI_RESID || g.ldr % 4 == 0)) {
            if (gemm_tc(g, n_sm, s)) return;
            if (gemm_tc_required() && g.epi != EPI_ROPE)
                PTC_FATAL("PTC_GEMM_TC=1: the tensor-core GEMM refused %d x %d x %d (a_kcontig %d, b_kcontig %d)",
                          g.M, g.N, g.K, (int)g.a_kcontig, (int)g.b_kcontig);
        }
        // Tile: 128x128 when the product alone fills the GPU, else 64x64;
        // then split K (chunks of at least 64, a multiple of the k-tile)
        // until about one wave of CTAs covers the SMs.
        const bool big = (long)((g.M + 127) / 128) * ((g.N + 127) / 128) >= n_sm;
        const int BK = big ? 8 : 16;
        const long tiles = big ? (long)((g.M + 127) / 128) * ((g.N + 127) / 128)
                               : (long)((g.M + 63) / 64) * ((g.N + 63) / 64);
        int splits = 1;
        if (g.partial)
            while (tiles * splits * 2 <= 2L * n_sm && g.K / (splits * 2) >= 64 &&
                   (size_t)(splits * 2) * g.M * g.N <= g.partial_cap)
                splits *= 2;
        int kper = (g.K + splits - 1) / splits;
        kper = (kper + BK - 1) / BK * BK;
        g.splits = (g.K + kper - 1) / kper;
        // 64x64 tiles split 2, 4 or 8 ways reduce inside a cluster (at most
        // 8 CTAs, whole rows per CTA); anything else through the workspace
        g.cluster_red = !big && g.splits > 1 && g.splits <= 8 && 64 % g.splits == 0;
        if (big) launch_tile_v<128, 128, 8, 8, 8>(g, kper, s);
        else launch_tile_v<64, 64, 16, 4, 4>(g, kper, s);
        if (g.splits > 1 && !g.cluster_red) launch_splitk_reduce(g, n_sm, s);
        return;
    }
    const bool big = (long)g.M * g.N >= (long)128 * 128 * n_sm;
    const long tiles = big ? (long)((g.M + 127) / 128) * ((g.N + 127) / 128)
                           : (long)((g.M + 63) / 64) * ((g.N + 63) / 64);
    // Split K when the tile grid cannot fill the GPU and K is long.
    int splits = 1;
    if (g.partial && g.epi != EPI_ROPE) {
        while (tiles * splits * 2 <= 2L * n_sm && g.K / (splits * 2) >= 256 &&
               (size_t)(splits * 2) * g.M * g.N <= g.partial_cap)
            splits *= 2;
    }
    g.splits = splits;
    if (big) launch_tile<128, 128, 8, 8, 8>(g, s);
    else launch_tile<64, 64, 16, 4, 4>(g, s);
    if (splits > 1) launch_splitk_reduce(g, n_sm, s);
}

}  // namespace ptc

extern "C" void ptc_sgemm(int M, int N, int K, const float *A, int lda, int a_kcontig, const float *B, int ldb,
                          int b_kcontig, float *C, int ldc, int accumulate, float *workspace,
                          size_t workspace_floats, void *stream) {
    int dev = 0, n_sm = 148;
    PTC_CHECK(cudaGetDevice(&dev));
    PTC_CHECK(cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev));
    ptc::GemmArgs g;
    memset(&g, 0, sizeof(g));
    g.M = M; g.N = N; g.K = K;
    g.A = A; g.lda = lda; g.a_kcontig = a_kcontig != 0;
    g.B = B; g.ldb = ldb; g.b_kcontig = b_kcontig != 0;
    g.C = C; g.ldc = ldc;
    g.epi = accumulate ? ptc::EPI_ACCUM : ptc::EPI_STORE;
    g.partial = workspace;
    g.partial_cap = workspace ? workspace_floats : 0;
    ptc::gemm(g, n_sm, (cudaStream_t)stream);
}

extern "C" void ptc_gemm_counters(long long *out) {
    for (int i = 0; i < ptc::GC_N; i++) out[i] = ptc::g_gemm_counts[i].load(std::memory_order_relaxed);
}
