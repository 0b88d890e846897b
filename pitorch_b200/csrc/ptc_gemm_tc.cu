// ptc_gemm_tc.cu -- fp32 GEMM on the sm_100a tensor cores for the large
// training products (the classifier's forward, input-gradient and
// weight-gradient GEMMs of pitorch/train/pt_train.c:296-303, :442-453,
// :475-492).
//
// CUTLASS's sm100 "FastFP32" collective (header templates, instantiated here)
// loads fp32 tiles by TMA, each CTA its own (cluster 1x1x1, this GPU's own
// memory), splits each operand element into three bf16 parts in
// shared memory and sums all nine partial products with tcgen05.mma into
// fp32 accumulators in tensor memory, which keeps fp32 accuracy. The epilogue is D = A.B (+ C): store, accumulate or
// residual add; RoPE products stay on the SIMT kernel.
//
// Products whose tile grid cannot fill the GPU (the classifier input
// gradient: 2x3 tiles over K = 32000) are split over K as a batch of
// K-slices into the split-K workspace and summed by k_splitk_reduce.
#include <pthread.h>
#include <stdlib.h>

#include <map>
#include <type_traits>
#include <utility>

#include "cute/tensor.hpp"
#include "cutlass/cutlass.h"
#include "cutlass/epilogue/collective/collective_builder.hpp"
#include "cutlass/gemm/collective/collective_builder.hpp"
#include "cutlass/gemm/device/gemm_universal_adapter.h"
#include "cutlass/gemm/kernel/gemm_universal.hpp"

#include "ptc_common.cuh"
#include "ptc_gemm.h"

namespace ptc {

namespace {

using TcTile = cute::Shape<cute::_128, cute::_128, cute::_32>;
using TcCluster = cute::Shape<cute::_1, cute::_1, cute::_1>;

template <class LayoutA, class LayoutB>
struct TcGemm {
    using LayoutC = cutlass::layout::RowMajor;
    using Epilogue = typename cutlass::epilogue::collective::CollectiveBuilder<
        cutlass::arch::Sm100, cutlass::arch::OpClassTensorOp, TcTile, TcCluster,
        cutlass::epilogue::collective::EpilogueTileAuto, float, float, float, LayoutC, 4, float, LayoutC, 4,
        cutlass::epilogue::collective::EpilogueScheduleAuto>::CollectiveOp;
    using Mainloop = typename cutlass::gemm::collective::CollectiveBuilder<
        cutlass::arch::Sm100, cutlass::arch::OpClassTensorOp, float, LayoutA, 4, float, LayoutB, 4, float, TcTile,
        TcCluster,
        cutlass::gemm::collective::StageCountAutoCarveout<static_cast<int>(sizeof(typename Epilogue::SharedStorage))>,
        cutlass::gemm::KernelTmaWarpSpecialized1SmFastFP32Sm100>::CollectiveOp;
    using Kernel = cutlass::gemm::kernel::GemmUniversal<cute::Shape<int, int, int, int>, Mainloop, Epilogue>;
    using Gemm = cutlass::gemm::device::GemmUniversalAdapter<Kernel>;
};

// A cute stride with its dynamic modes set to (s0, s1, s2); static modes
// (the unit stride of the contiguous dimension) keep their value.
template <class Stride>
Stride make_strides(int64_t s0, int64_t s1, int64_t s2) {
    Stride st{};
    auto set = [](auto &&e, int64_t v) {
        if constexpr (!cute::is_static<std::decay_t<decltype(e)>>::value) e = v;
    };
    set(cute::get<0>(st), s0);
    set(cute::get<1>(st), s1);
    set(cute::get<2>(st), s2);
    return st;
}

// Workspace of the CUTLASS kernels, one per device and stream (grown on
// demand, never freed): products on different streams of a device may run
// at the same time.
void *tc_workspace(size_t bytes, cudaStream_t s) {
    static pthread_mutex_t mu = PTHREAD_MUTEX_INITIALIZER;
    static std::map<std::pair<int, cudaStream_t>, std::pair<void *, size_t>> ws;
    if (bytes == 0) return nullptr;
    int dev = 0;
    PTC_CHECK(cudaGetDevice(&dev));
    pthread_mutex_lock(&mu);
    auto &w = ws[{dev, s}];
    if (w.second < bytes) {
        if (w.first) PTC_CHECK(cudaFree(w.first));
        PTC_CHECK(cudaMalloc(&w.first, bytes));
        w.second = bytes;
    }
    void *p = w.first;
    pthread_mutex_unlock(&mu);
    return p;
}

// D[l] = alpha A[l].B[l] + beta C[l] over L batches; the strides of A, B, C,
// D are (leading, batch) pairs in elements. Returns false if CUTLASS cannot
// run this problem (the caller then uses the SIMT kernel).
template <class LayoutA, class LayoutB>
bool run_tc(int M, int N, int K, int L, const float *A, int64_t lda, int64_t bsa, const float *B, int64_t ldb,
            int64_t bsb, const float *C, int64_t ldc, int64_t bsc, float *D, int64_t ldd, int64_t bsd, float beta,
            cudaStream_t s) {
    using G = TcGemm<LayoutA, LayoutB>;
    using K_ = typename G::Kernel;
    constexpr bool a_rowmajor = std::is_same_v<LayoutA, cutlass::layout::RowMajor>;
    constexpr bool b_rowmajor = std::is_same_v<LayoutB, cutlass::layout::RowMajor>;
    // A modes (M, K, L); B modes (N, K, L); C/D modes (M, N, L)
    auto sA = make_strides<typename K_::StrideA>(a_rowmajor ? lda : 1, a_rowmajor ? 1 : lda, bsa);
    auto sB = make_strides<typename K_::StrideB>(b_rowmajor ? 1 : ldb, b_rowmajor ? ldb : 1, bsb);
    auto sC = make_strides<typename K_::StrideC>(ldc, 1, bsc);
    auto sD = make_strides<typename K_::StrideD>(ldd, 1, bsd);
    typename G::Gemm::Arguments args{cutlass::gemm::GemmUniversalMode::kGemm,
                                     {M, N, K, L},
                                     {A, sA, B, sB},
                                     {{1.0f, beta}, C, sC, D, sD}};
    typename G::Gemm gemm;
    if (gemm.can_implement(args) != cutlass::Status::kSuccess) return false;
    void *ws = tc_workspace(G::Gemm::get_workspace_size(args), s);
    if (gemm.initialize(args, ws, s) != cutlass::Status::kSuccess) return false;
    if (gemm.run(s) != cutlass::Status::kSuccess) PTC_FATAL("tensor-core GEMM launch failed (%d x %d x %d)", M, N, K);
    PTC_CHECK(cudaGetLastError());
    gemm_count(GC_TENSOR_CORE);
    return true;
}

template <class LayoutA, class LayoutB>
bool dispatch(const GemmArgs &g, int n_sm, cudaStream_t s) {
    const long tiles = (long)((g.M + 127) / 128) * ((g.N + 127) / 128);
    // Split K into a batch of slices when the tile grid leaves most SMs idle
    // and the split-K workspace holds the partials (slices of whole float4s).
    int S = 1;
    if (g.partial)
        while (tiles * S * 2 <= n_sm && g.K % (S * 2) == 0 && (g.K / (S * 2)) % 4 == 0 && g.K / (S * 2) >= 512 &&
               (size_t)(S * 2) * g.M * g.N <= g.partial_cap)
            S *= 2;
    constexpr bool a_rowmajor = std::is_same_v<LayoutA, cutlass::layout::RowMajor>;
    constexpr bool b_rowmajor = std::is_same_v<LayoutB, cutlass::layout::RowMajor>;
    if (S > 1) {
        const int kper = g.K / S;
        // slice l starts kper columns (k-contiguous) or kper rows further on
        const int64_t bsa = a_rowmajor ? kper : (int64_t)kper * g.lda;
        const int64_t bsb = b_rowmajor ? (int64_t)kper * g.ldb : kper;
        const int64_t slice = (int64_t)g.M * g.N;
        if (!run_tc<LayoutA, LayoutB>(g.M, g.N, kper, S, g.A, g.lda, bsa, g.B, g.ldb, bsb, g.partial, g.N, slice,
                                      g.partial, g.N, slice, 0.0f, s))
            return false;
        GemmArgs r = g;
        r.splits = S;
        launch_splitk_reduce(r, n_sm, s);
        return true;
    }
    const float *C = g.epi == EPI_RESID ? g.R : g.C;
    const int64_t ldc = g.epi == EPI_RESID ? g.ldr : g.ldc;
    const float beta = (g.epi == EPI_ACCUM || g.epi == EPI_RESID) ? 1.0f : 0.0f;
    return run_tc<LayoutA, LayoutB>(g.M, g.N, g.K, 1, g.A, g.lda, 0, g.B, g.ldb, 0, C, ldc, 0, g.C, g.ldc, 0, beta, s);
}

}  // namespace

// On unless PTC_GEMM_TC=0 (which keeps every product on the SIMT kernel).
bool gemm_tc_enabled() {
    static const bool on = [] {
        const char *e = getenv("PTC_GEMM_TC");
        return !(e && e[0] == '0');
    }();
    return on;
}

bool gemm_tc_required() {
    static const bool req = [] {
        const char *e = getenv("PTC_GEMM_TC");
        return e && e[0] == '1';
    }();
    return req;
}

bool gemm_tc(const GemmArgs &g, int n_sm, cudaStream_t s) {
    if (g.epi == EPI_ROPE) return false;
    if (g.a_kcontig && g.b_kcontig) return dispatch<cutlass::layout::RowMajor, cutlass::layout::ColumnMajor>(g, n_sm, s);
    if (g.a_kcontig) return dispatch<cutlass::layout::RowMajor, cutlass::layout::RowMajor>(g, n_sm, s);
    if (!g.b_kcontig) return dispatch<cutlass::layout::ColumnMajor, cutlass::layout::RowMajor>(g, n_sm, s);
    return false;   // A m-contiguous with B k-contiguous: no product of the training step
}

}  // namespace ptc
