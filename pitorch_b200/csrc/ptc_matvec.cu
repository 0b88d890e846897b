// ptc_matvec.cu -- standalone fp32 y = W . x for sm_100a.
//
// Replaces smatvec_tmu (pitorch/ops/matvec/matvec.c:13-86) and its QPU
// kernel (pitorch/kernels/matvec/matvec_tmu.qasm), where each of 16 lanes
// per QPU owned one row and walked its columns sequentially. Here a warp
// owns a row (or a pair of rows): its 32 lanes stream consecutive 16-byte
// chunks of the row (fully coalesced 512-byte warp requests, L1 bypassed),
// multiply by the lane's slice of x held in registers, and reduce with a
// shuffle tree -- the row's K dimension split over the 32 lanes. Matrices
// of many narrow rows stage x in shared memory once per CTA and keep two
// passes of rows in flight per warp (k_matvec_pf). Rows wider than 2048
// floats, or unaligned operands, use a scalar-load variant with x staged in
// shared memory.
//
// The kernel is HBM-bound at 0.5 flop/byte: algorithmic bytes per call are
// 4 * (rows*cols + rows + cols).
#include <pthread.h>
#include <string.h>

#include <map>

#include "../../include/ptc.h"
#include "ptc_common.cuh"
#include "ptc_internal.h"

namespace ptc {

template <int NV, int R>
__global__ void __launch_bounds__(256) k_matvec(const float *__restrict__ W, const float *__restrict__ x,
                                                float *__restrict__ y, int rows, int cols) {
    // Programmatic dependent launch: W never comes from the previous kernel
    // of the stream, so the first rows are requested before
    // griddepcontrol.wait and consecutive matvecs overlap; x (possibly the
    // previous kernel's output) is read after it.
    pdl_trigger();
    const int lane = threadIdx.x & 31;
    const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int nw = (gridDim.x * blockDim.x) >> 5;
    const int c4 = cols >> 2;
    float4 w[R][NV];
    auto load_rows = [&](int r0) {
#pragma unroll
        for (int k = 0; k < R; k++) {
            const float4 *row = reinterpret_cast<const float4 *>(W + (size_t)(r0 + k) * cols);
#pragma unroll
            for (int v = 0; v < NV; v++) {
                int c = lane + 32 * v;
                w[k][v] = (r0 + k < rows && c < c4) ? ldg_stream(row + c) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
    };
    int r0 = gw * R;
    if (r0 < rows) load_rows(r0);
    pdl_wait();
    float4 xr[NV];
    const float4 *x4 = reinterpret_cast<const float4 *>(x);
#pragma unroll
    for (int v = 0; v < NV; v++) {
        int c = lane + 32 * v;
        xr[v] = (c < c4) ? __ldcg(x4 + c) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    for (; r0 < rows; r0 += nw * R) {
        if (r0 != gw * R) load_rows(r0);
#pragma unroll
        for (int k = 0; k < R; k++) {
            float acc = 0.f;
#pragma unroll
            for (int v = 0; v < NV; v++) acc = dot4(w[k][v], xr[v], acc);
            acc = warp_sum(acc);
            if (lane == 0 && r0 + k < rows) y[r0 + k] = acc;
        }
    }
}

// Many rows of up to 768 floats (1376 x 512, 2048 x 768, 32000 x 288): x
// staged in shared memory once per CTA (the per-warp reads of x otherwise
// queue at the few L2 lines that hold it), and each warp requests its next
// R rows before it reduces the current ones (a register double buffer), so
// two passes of rows are in flight per warp. The two-row form is held to 64
// registers so that 4 CTAs fit per SM (at 71 registers, 3: 8.2 instead of
// 7.6 us at 32000 x 288). Measured against the one-warp-per-row kernel above
// on the same B200: 32000 x 288 9.97 -> 7.6 us, 1376 x 512 2.30-2.40 ->
// 2.19 us, 2048 x 768 2.62 -> 2.60 us per call; for fewer rows, and for the
// 32000 x 768 classifier, the kernel above is as fast or faster (there the
// staging's block barrier costs more than it saves).
template <int NV, int R>
__global__ void __launch_bounds__(256, R == 2 ? 4 : 1) k_matvec_pf(const float *__restrict__ W, const float *__restrict__ x,
                                                   float *__restrict__ y, int rows, int cols) {
    pdl_trigger();
    __shared__ __align__(16) float4 s_x[512];   // x, once per CTA (cols <= 2048)
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int c4 = cols >> 2;
    const int ng = gridDim.x * 8;               // warps (row groups) in the grid
    float4 w[R][NV];
    auto load_rows = [&](float4 (&dst)[R][NV], int r0) {
#pragma unroll
        for (int k = 0; k < R; k++) {
            const float4 *row = reinterpret_cast<const float4 *>(W + (size_t)(r0 + k) * cols);
#pragma unroll
            for (int v = 0; v < NV; v++) {
                const int c = lane + 32 * v;
                dst[k][v] = (r0 + k < rows && c < c4) ? ldg_stream(row + c) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
    };
    int r0 = (blockIdx.x * 8 + warp) * R;
    load_rows(w, r0);
    pdl_wait();
    const float4 *x4 = reinterpret_cast<const float4 *>(x);
    float4 xr[NV];
    for (int i = tid; i < c4; i += 256) cp_async16(&s_x[i], x4 + i);
    cp_async_commit();
    cp_async_wait_all();
    __syncthreads();
#pragma unroll
    for (int v = 0; v < NV; v++) {
        const int c = lane + 32 * v;
        xr[v] = (c < c4) ? s_x[c] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    // passes counted by the CTA's first row; the next pass's rows are
    // requested before the current ones are reduced (rows past the end read
    // as zeros)
    for (int rb = blockIdx.x * 8 * R; rb < rows; rb += ng * R, r0 += ng * R) {
        float4 wn[R][NV];
        if (rb + ng * R < rows) load_rows(reinterpret_cast<float4 (&)[R][NV]>(wn), r0 + ng * R);
        float acc[R];
#pragma unroll
        for (int k = 0; k < R; k++) {
            float a = 0.f;
#pragma unroll
            for (int v = 0; v < NV; v++) a = dot4(w[k][v], xr[v], a);
            acc[k] = warp_sum(a);
        }
        if (lane == 0)
#pragma unroll
            for (int k = 0; k < R; k++)
                if (r0 + k < rows) y[r0 + k] = acc[k];
#pragma unroll
        for (int k = 0; k < R; k++)
#pragma unroll
            for (int v = 0; v < NV; v++) w[k][v] = reinterpret_cast<float4 (&)[R][NV]>(wn)[k][v];
    }
}

// Any shape / alignment: x staged in shared memory in tiles, one warp per
// row, scalar coalesced loads.
__global__ void __launch_bounds__(256) k_matvec_any(const float *__restrict__ W, const float *__restrict__ x,
                                                    float *__restrict__ y, int rows, int cols) {
    __shared__ float sx[4096];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int row_base = blockIdx.x * (blockDim.x >> 5);
    const int r = row_base + warp;
    float acc = 0.f;
    for (int k0 = 0; k0 < cols; k0 += 4096) {
        const int kn = min(4096, cols - k0);
        __syncthreads();
        for (int i = threadIdx.x; i < kn; i += blockDim.x) sx[i] = x[k0 + i];
        __syncthreads();
        if (r < rows) {
            const float *row = W + (size_t)r * cols + k0;
            for (int i = lane; i < kn; i += 32) acc = fmaf(row[i], sx[i], acc);
        }
    }
    acc = warp_sum(acc);
    if (r < rows && lane == 0) y[r] = acc;
}

template <int NV, int R, bool PF>
static void launch_k_matvec(int grid, const float *W, const float *x, float *y, int rows, int cols,
                            cudaStream_t s) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(256);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if constexpr (PF) PTC_CHECK(cudaLaunchKernelEx(&cfg, k_matvec_pf<NV, R>, W, x, y, rows, cols));
    else PTC_CHECK(cudaLaunchKernelEx(&cfg, k_matvec<NV, R>, W, x, y, rows, cols));
}

// One warp per row (pair), the row's float4s spread over the lanes: for
// every shape of the sweep this measured as fast as or faster than splitting
// a row over 2, 4 or 8 warps with the slice sums added in shared memory
// (288 x 768: 1.48 us one warp per row, 1.73 us over 4 warps; 288 x 288,
// 512 x 512, 768 x 288 and 32000 x 288 slower split as well): at these
// sizes a call is bound by its launch and one memory round trip, which a
// split does not shorten, and the split adds two block barriers.
#define MV_CASE(NVV)                                                                        \
    case NVV:                                                                               \
        if constexpr (NVV <= 3) {                                                           \
            if (rows >= 4096) launch_k_matvec<NVV, 2, true>(grid2, W, x, y, rows, cols, s);  \
            else if (rows >= 1024) launch_k_matvec<NVV, 1, true>(grid1, W, x, y, rows, cols, s); \
            else launch_k_matvec<NVV, 1, false>(grid1, W, x, y, rows, cols, s);             \
        } else if constexpr (NVV <= 6) {                                                    \
            if (rows >= 4096) launch_k_matvec<NVV, 2, false>(grid2, W, x, y, rows, cols, s); \
            else if (rows >= 1024) launch_k_matvec<NVV, 1, true>(grid1, W, x, y, rows, cols, s); \
            else launch_k_matvec<NVV, 1, false>(grid1, W, x, y, rows, cols, s);             \
        } else {                                                                            \
            if (rows >= 4096) launch_k_matvec<NVV, 2, false>(grid2, W, x, y, rows, cols, s); \
            else launch_k_matvec<NVV, 1, false>(grid1, W, x, y, rows, cols, s);             \
        }                                                                                   \
        break;

void launch_matvec(const float *W, const float *x, float *y, int rows, int cols, cudaStream_t s) {
    if (rows <= 0) return;
    if (cols <= 0) {
        PTC_CHECK(cudaMemsetAsync(y, 0, (size_t)rows * 4, s));
        return;
    }
    const bool vec_ok = (cols % 4 == 0) && (((uintptr_t)W | (uintptr_t)x) % 16 == 0) && cols <= 2048;
    if (!vec_ok) {
        k_matvec_any<<<(rows + 7) / 8, 256, 0, s>>>(W, x, y, rows, cols);
        PTC_CHECK(cudaGetLastError());
        return;
    }
    int dev = 0, n_sm = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev);
    // One warp per row (pair): enough warps to cover all rows in one pass
    // when possible, capped at 4 resident 8-warp blocks per SM.
    const int cap = 4 * n_sm;
    int grid1 = (rows + 7) / 8;
    if (grid1 > cap) grid1 = cap;
    int grid2 = (rows / 2 + 7) / 8;
    if (grid2 > cap) grid2 = cap;
    if (grid2 < 1) grid2 = 1;
    const int nv = (cols / 4 + 31) / 32;
    switch (nv) {
        MV_CASE(1) MV_CASE(2) MV_CASE(3) MV_CASE(4) MV_CASE(5) MV_CASE(6) MV_CASE(7) MV_CASE(8)
        MV_CASE(9) MV_CASE(10) MV_CASE(11) MV_CASE(12) MV_CASE(13) MV_CASE(14) MV_CASE(15) MV_CASE(16)
        default: PTC_FATAL("unreachable matvec width");
    }
    PTC_CHECK(cudaGetLastError());
}

// Read bandwidth probe: every thread streams float4s of buf (grid-stride,
// L2-only loads) and folds them into one value, written so the loads are
// not removed. Over a buffer that fits in L2 and was just read, this is the
// L2 read bandwidth; over one larger than L2, HBM.
__global__ void __launch_bounds__(256) k_read_probe(const float4 *__restrict__ buf, size_t n4, float *sink) {
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += 4 * stride) {
        float4 v[4];
#pragma unroll
        for (int k = 0; k < 4; k++) v[k] = (i + k * stride < n4) ? __ldcg(buf + i + k * stride) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int k = 0; k < 4; k++) { a.x += v[k].x; a.y += v[k].y; a.z += v[k].z; a.w += v[k].w; }
    }
    const float t = a.x + a.y + a.z + a.w;
    if (t == 123456.789f) *sink = t;   // practically never: keeps the loads live
}

}  // namespace ptc

extern "C" void ptc_matvec(const float *W, const float *x, float *y, int rows, int cols, void *stream) {
    ptc::launch_matvec(W, x, y, rows, cols, (cudaStream_t)stream);
}

extern "C" void ptc_read_probe(const void *buf, size_t bytes, float *sink, void *stream) {
    int dev = 0, n_sm = 148;
    PTC_CHECK(cudaGetDevice(&dev));
    PTC_CHECK(cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev));
    ptc::k_read_probe<<<4 * n_sm, 256, 0, (cudaStream_t)stream>>>((const float4 *)buf, bytes / 16, sink);
    PTC_CHECK(cudaGetLastError());
}

// ---------------------------------------------------------------------------
// Host-pointer path (pt_matvec_fn contract). Per device: a context for the
// staging stream plus grow-only device/pinned scratch.
// ---------------------------------------------------------------------------
struct HostMatvecScratch {
    ptc_ctx *ctx;
    float *dW, *dx, *dy;
    size_t capW, capx, capy;
    float *hx, *hy;
    size_t caphx, caphy;
};
static std::map<int, HostMatvecScratch> g_scratch;
static pthread_mutex_t g_mv_mu = PTHREAD_MUTEX_INITIALIZER;

static float *grow_dev(float *p, size_t *cap, size_t need) {
    if (need <= *cap) return p;
    if (p) cudaFree(p);
    size_t n = need + need / 2;
    PTC_CHECK(cudaMalloc(&p, n));
    *cap = n;
    return p;
}

static float *grow_host(float *p, size_t *cap, size_t need) {
    if (need <= *cap) return p;
    if (p) cudaFreeHost(p);
    size_t n = need + need / 2;
    PTC_CHECK(cudaMallocHost(&p, n));
    *cap = n;
    return p;
}

extern "C" void ptc_matvec_host(const float *W, const float *x, float *y, int rows, int cols) {
    if (rows <= 0) return;
    const size_t wbytes = (size_t)rows * cols * 4;
    const void *dW = nullptr;
    ptc_ctx *owner = nullptr;
    const bool resident = ptc_lookup_range(W, wbytes, &dW, &owner);
    int dev = 0;
    if (resident) dev = ptc_device(owner);
    else PTC_CHECK(cudaGetDevice(&dev));
    PTC_CHECK(cudaSetDevice(dev));

    pthread_mutex_lock(&g_mv_mu);
    HostMatvecScratch &sc = g_scratch[dev];
    if (!sc.ctx) sc.ctx = ptc_create(dev, 0);
    cudaStream_t s = ptc_ctx_stream(sc.ctx);
    if (!resident) {
        sc.dW = grow_dev(sc.dW, &sc.capW, wbytes);
        PTC_CHECK(cudaMemcpyAsync(sc.dW, W, wbytes, cudaMemcpyHostToDevice, s));
        dW = sc.dW;
    }
    sc.dx = grow_dev(sc.dx, &sc.capx, (size_t)cols * 4 + 16);
    sc.dy = grow_dev(sc.dy, &sc.capy, (size_t)rows * 4 + 16);
    sc.hx = grow_host(sc.hx, &sc.caphx, (size_t)cols * 4 + 16);
    sc.hy = grow_host(sc.hy, &sc.caphy, (size_t)rows * 4 + 16);
    memcpy(sc.hx, x, (size_t)cols * 4);
    PTC_CHECK(cudaMemcpyAsync(sc.dx, sc.hx, (size_t)cols * 4, cudaMemcpyHostToDevice, s));
    ptc::launch_matvec((const float *)dW, sc.dx, sc.dy, rows, cols, s);
    PTC_CHECK(cudaMemcpyAsync(sc.hy, sc.dy, (size_t)rows * 4, cudaMemcpyDeviceToHost, s));
    PTC_CHECK(cudaStreamSynchronize(s));
    memcpy(y, sc.hy, (size_t)rows * 4);
    pthread_mutex_unlock(&g_mv_mu);
}
