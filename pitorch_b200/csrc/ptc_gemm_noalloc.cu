// ptc_gemm_noalloc.cu -- ptc_sgemm for callers that cannot allocate device
// memory.
//
// Some callers of this library cannot call cudaMalloc at all: code running
// while a CUDA stream is being captured into a graph (allocation is not a
// capturable operation), inside an allocator or memory-pool callback, or
// under a host framework that owns every device allocation and forbids
// others. They cannot hand ptc_sgemm a workspace either. This variant keeps
// its split-K partial sums in a fixed static device array instead, so a call
// needs nothing but the caller's own inputs and output.
//
// The array is a file-scope __device__ variable: every GPU that loads the
// library holds its PTC_SGEMM_NOALLOC_MAX_MN floats until the process exits.
// Host code cannot use the array's name as a device address; the device
// address is looked up once per device with cudaGetSymbolAddress.
#include <pthread.h>
#include <stdio.h>
#include <string.h>

#include "../../include/ptc.h"
#include "ptc_common.cuh"
#include "ptc_gemm.h"

static __device__ __align__(256) float g_sgemm_noalloc_scratch[PTC_SGEMM_NOALLOC_MAX_MN];

namespace {
constexpr int kMaxDevices = 64;
// Per device: the array's device address and the SM count. A set-up stores
// the SM count first and then publishes the pointer with a release store;
// readers load the pointer with acquire, so a non-null pointer comes with a
// valid SM count.
float *g_scratch_dev[kMaxDevices];
int g_sm_count[kMaxDevices];
pthread_mutex_t g_setup_mu = PTHREAD_MUTEX_INITIALIZER;

float *scratch_of(int dev) { return __atomic_load_n(&g_scratch_dev[dev], __ATOMIC_ACQUIRE); }

// One-time set-up for the current device: resolve the array's device address.
bool setup_device(int dev) {
    bool ok = true;
    pthread_mutex_lock(&g_setup_mu);
    if (!scratch_of(dev)) {
        float *p = nullptr;
        cudaError_t e = cudaGetSymbolAddress((void **)&p, g_sgemm_noalloc_scratch);
        int n_sm = 0;
        cudaError_t e2 = cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess || e2 != cudaSuccess || !p) {
            fprintf(stderr, "pitorch_b200: ptc_sgemm_noalloc: scratch set-up failed on device %d: %s\n", dev,
                    cudaGetErrorString(e != cudaSuccess ? e : e2));
            ok = false;
        } else {
            g_sm_count[dev] = n_sm;
            __atomic_store_n(&g_scratch_dev[dev], p, __ATOMIC_RELEASE);
        }
    }
    pthread_mutex_unlock(&g_setup_mu);
    return ok;
}
}  // namespace

extern "C" int ptc_sgemm_noalloc(int M, int N, int K, const float *A, int lda, int a_kcontig, const float *B,
                                 int ldb, int b_kcontig, float *C, int ldc, int accumulate, void *stream) {
    if (M < 0 || N < 0 || K < 0) {
        fprintf(stderr, "pitorch_b200: ptc_sgemm_noalloc: negative size (M=%d N=%d K=%d)\n", M, N, K);
        return -1;
    }
    if ((unsigned long long)M * (unsigned long long)N > (unsigned long long)PTC_SGEMM_NOALLOC_MAX_MN) {
        fprintf(stderr,
                "pitorch_b200: ptc_sgemm_noalloc: M*N = %llu exceeds the static scratch of %u floats; "
                "use ptc_sgemm with a workspace for this shape\n",
                (unsigned long long)M * (unsigned long long)N, (unsigned)PTC_SGEMM_NOALLOC_MAX_MN);
        return -1;
    }
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        fprintf(stderr, "pitorch_b200: ptc_sgemm_noalloc: no usable current device\n");
        return -1;
    }
    float *scratch = scratch_of(dev);
    if (!scratch) {
        if (!setup_device(dev)) return -1;
        scratch = scratch_of(dev);
    }

    ptc::GemmArgs g;
    memset(&g, 0, sizeof(g));
    g.M = M; g.N = N; g.K = K;
    g.A = A; g.lda = lda; g.a_kcontig = a_kcontig != 0;
    g.B = B; g.ldb = ldb; g.b_kcontig = b_kcontig != 0;
    g.C = C; g.ldc = ldc;
    g.epi = accumulate ? ptc::EPI_ACCUM : ptc::EPI_STORE;
    // Every split writes all of its M*N partials before the reduction reads
    // them, so whatever an earlier call left in the array is never read.
    g.partial = scratch;
    g.partial_cap = PTC_SGEMM_NOALLOC_MAX_MN;
    g.no_alloc = 1;
    ptc::gemm(g, g_sm_count[dev], (cudaStream_t)stream);
    return 0;
}
