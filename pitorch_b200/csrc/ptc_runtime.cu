// ptc_runtime.cu -- contexts, the device arena, image upload, the
// host-to-device range registry and CUDA-event timers.
//
// Replaces pitorch/runtime/ (gpu.c: qpu_enable/gpu_alloc/qpu_launch;
// arena.c: the one-shot bump arena). On the Pi the arena exists because the
// firmware allocator breaks after two allocations (arena.h:6-8); here it
// exists so that a context does all its device allocation up front and the
// decode/train steps allocate nothing.
#include <pthread.h>
#include <string.h>
#include <time.h>

#include <map>
#include <utility>
#include <vector>

#include "../../include/ptc.h"
#include "ptc_common.cuh"
#include "ptc_internal.h"

struct ptc_ctx {
    int device;
    int n_sm;
    cudaStream_t stream;
    std::vector<ptc_chunk> chunks;   // arena chunks; the last one is active
    size_t used_total;               // bytes handed out (incl. alignment)
};

static const size_t kGrowChunk = 256ull << 20;

namespace ptc {
void ensure_kernel_smem(const void *kernel, size_t smem) {
    static pthread_mutex_t mu = PTHREAD_MUTEX_INITIALIZER;
    static std::map<std::pair<const void *, int>, size_t> granted;
    int dev = 0;
    PTC_CHECK(cudaGetDevice(&dev));
    pthread_mutex_lock(&mu);
    const auto key = std::make_pair(kernel, dev);
    auto it = granted.find(key);
    if (it == granted.end() || it->second < smem) {
        if (it == granted.end())
            PTC_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100));
        PTC_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        granted[key] = smem;
    }
    pthread_mutex_unlock(&mu);
}
}  // namespace ptc

extern "C" int ptc_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n;
}

extern "C" ptc_ctx *ptc_create(int device, size_t arena_bytes) {
    int n = ptc_device_count();
    if (n <= 0) PTC_FATAL("no CUDA device available (pitorch_b200 has no CPU path)");
    if (device < 0 || device >= n) PTC_FATAL("device %d out of range (%d visible)", device, n);
    PTC_CHECK(cudaSetDevice(device));
    ptc_ctx *c = new ptc_ctx();
    c->device = device;
    PTC_CHECK(cudaDeviceGetAttribute(&c->n_sm, cudaDevAttrMultiProcessorCount, device));
    PTC_CHECK(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking));
    c->used_total = 0;
    if (arena_bytes) {
        ptc_chunk ch;
        PTC_CHECK(cudaMalloc(&ch.base, arena_bytes));
        ch.size = arena_bytes;
        ch.used = 0;
        c->chunks.push_back(ch);
    }
    return c;
}

extern "C" void ptc_destroy(ptc_ctx *c) {
    if (!c) return;
    cudaSetDevice(c->device);
    cudaStreamSynchronize(c->stream);
    ptc_unregister_ctx(c);
    for (auto &ch : c->chunks) cudaFree(ch.base);
    cudaStreamDestroy(c->stream);
    delete c;
}

extern "C" void *ptc_alloc(ptc_ctx *c, size_t bytes) {
    const size_t align = 256;
    if (bytes == 0) bytes = align;
    if (c->chunks.empty() || c->chunks.back().used + align + bytes > c->chunks.back().size) {
        ptc_chunk ch;
        ch.size = bytes + align > kGrowChunk ? bytes + align : kGrowChunk;
        PTC_CHECK(cudaSetDevice(c->device));
        PTC_CHECK(cudaMalloc(&ch.base, ch.size));
        ch.used = 0;
        c->chunks.push_back(ch);
    }
    ptc_chunk &ch = c->chunks.back();
    uintptr_t p = (uintptr_t)ch.base + ch.used;
    uintptr_t a = (p + align - 1) & ~(uintptr_t)(align - 1);
    ch.used = (a - (uintptr_t)ch.base) + bytes;
    c->used_total += (a - p) + bytes;
    return (void *)a;
}

extern "C" size_t ptc_arena_used(const ptc_ctx *c) { return c->used_total; }

extern "C" void ptc_arena_reset(ptc_ctx *c, size_t mark) {
    // Rewind within the active chunk only (the reference's reset rewinds to
    // the arena base, arena.c:28-31; callers here reset to their own mark).
    if (c->chunks.empty()) return;
    ptc_chunk &ch = c->chunks.back();
    size_t drop = c->used_total > mark ? c->used_total - mark : 0;
    if (drop <= ch.used) {
        ch.used -= drop;
        c->used_total = mark;
    }
}

extern "C" void *ptc_stream(ptc_ctx *c) { return (void *)c->stream; }
extern "C" int ptc_device(const ptc_ctx *c) { return c->device; }
extern "C" int ptc_sm_count(const ptc_ctx *c) { return c->n_sm; }

extern "C" void ptc_sync(ptc_ctx *c) { PTC_CHECK(cudaStreamSynchronize(c->stream)); }

extern "C" void ptc_h2d(ptc_ctx *c, void *dst, const void *src, size_t bytes) {
    if (!bytes) return;
    PTC_CHECK(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, c->stream));
    PTC_CHECK(cudaStreamSynchronize(c->stream));
}

extern "C" void ptc_d2h(ptc_ctx *c, void *dst, const void *src, size_t bytes) {
    if (!bytes) return;
    PTC_CHECK(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, c->stream));
    PTC_CHECK(cudaStreamSynchronize(c->stream));
}

extern "C" void ptc_d2d(ptc_ctx *c, void *dst, const void *src, size_t bytes) {
    if (!bytes) return;
    PTC_CHECK(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, c->stream));
}

extern "C" void ptc_memset(ptc_ctx *c, void *dst, int value, size_t bytes) {
    if (!bytes) return;
    PTC_CHECK(cudaMemsetAsync(dst, value, bytes, c->stream));
}

extern "C" void *ptc_host_alloc(size_t bytes) {
    void *p = nullptr;
    PTC_CHECK(cudaMallocHost(&p, bytes ? bytes : 1));
    return p;
}

extern "C" void ptc_host_free(void *p) {
    if (p) cudaFreeHost(p);
}

extern "C" void *ptc_upload_image(ptc_ctx *c, const void *image, size_t bytes, size_t header_bytes) {
    // Place byte `header_bytes` of the image on a 256-byte boundary so that
    // every tensor (all multiples of 16 bytes for the supported shapes) is
    // aligned for 128-bit loads.
    char *base = (char *)ptc_alloc(c, bytes + 256);
    size_t pad = (256 - (header_bytes % 256)) % 256;
    char *dev = base + pad;
    PTC_CHECK(cudaSetDevice(c->device));
    PTC_CHECK(cudaMemcpyAsync(dev, image, bytes, cudaMemcpyHostToDevice, c->stream));
    PTC_CHECK(cudaStreamSynchronize(c->stream));
    ptc_register_range(image, dev, bytes, c);
    return dev;
}

// ---------------------------------------------------------------------------
// Host range -> device copy registry (used by the host-pointer matvec).
// ---------------------------------------------------------------------------
struct RangeEntry {
    uintptr_t host;
    uintptr_t dev;
    size_t bytes;
    ptc_ctx *owner;
};
static std::vector<RangeEntry> g_ranges;
static pthread_mutex_t g_ranges_mu = PTHREAD_MUTEX_INITIALIZER;

extern "C" void ptc_register_range(const void *host, const void *dev, size_t bytes, ptc_ctx *owner) {
    pthread_mutex_lock(&g_ranges_mu);
    g_ranges.push_back({(uintptr_t)host, (uintptr_t)dev, bytes, owner});
    pthread_mutex_unlock(&g_ranges_mu);
}

extern "C" void ptc_unregister_ctx(ptc_ctx *owner) {
    pthread_mutex_lock(&g_ranges_mu);
    std::vector<RangeEntry> keep;
    for (auto &e : g_ranges)
        if (e.owner != owner) keep.push_back(e);
    g_ranges.swap(keep);
    pthread_mutex_unlock(&g_ranges_mu);
}

bool ptc_lookup_range(const void *host, size_t bytes, const void **dev, ptc_ctx **owner) {
    uintptr_t h = (uintptr_t)host;
    bool found = false;
    pthread_mutex_lock(&g_ranges_mu);
    // Most recent registration wins (a context re-registering a range).
    for (size_t i = g_ranges.size(); i-- > 0;) {
        const RangeEntry &e = g_ranges[i];
        if (h >= e.host && h + bytes <= e.host + e.bytes) {
            *dev = (const void *)(e.dev + (h - e.host));
            *owner = e.owner;
            found = true;
            break;
        }
    }
    pthread_mutex_unlock(&g_ranges_mu);
    return found;
}

// ---------------------------------------------------------------------------
// Timers
// ---------------------------------------------------------------------------
struct ptc_timer {
    ptc_ctx *c;
    cudaEvent_t a, b;
};

extern "C" ptc_timer *ptc_timer_create(ptc_ctx *c) {
    ptc_timer *t = new ptc_timer();
    t->c = c;
    PTC_CHECK(cudaSetDevice(c->device));
    PTC_CHECK(cudaEventCreate(&t->a));
    PTC_CHECK(cudaEventCreate(&t->b));
    return t;
}
extern "C" void ptc_timer_start(ptc_timer *t) { PTC_CHECK(cudaEventRecord(t->a, t->c->stream)); }
extern "C" void ptc_timer_stop(ptc_timer *t) { PTC_CHECK(cudaEventRecord(t->b, t->c->stream)); }
extern "C" float ptc_timer_ms(ptc_timer *t) {
    float ms = 0.f;
    PTC_CHECK(cudaEventSynchronize(t->b));
    PTC_CHECK(cudaEventElapsedTime(&ms, t->a, t->b));
    return ms;
}
extern "C" void ptc_timer_destroy(ptc_timer *t) {
    if (!t) return;
    cudaEventDestroy(t->a);
    cudaEventDestroy(t->b);
    delete t;
}

// ---------------------------------------------------------------------------
// Graphs of stream work
// ---------------------------------------------------------------------------
struct ptc_graph {
    ptc_ctx *c;
    cudaGraphExec_t exec;
};

extern "C" void ptc_capture_begin(ptc_ctx *c) {
    PTC_CHECK(cudaSetDevice(c->device));
    PTC_CHECK(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
}
extern "C" ptc_graph *ptc_capture_end(ptc_ctx *c) {
    cudaGraph_t g;
    PTC_CHECK(cudaStreamEndCapture(c->stream, &g));
    ptc_graph *pg = new ptc_graph();
    pg->c = c;
    PTC_CHECK(cudaGraphInstantiate(&pg->exec, g, 0));
    PTC_CHECK(cudaGraphDestroy(g));
    return pg;
}
extern "C" void ptc_graph_launch(ptc_graph *g) { PTC_CHECK(cudaGraphLaunch(g->exec, g->c->stream)); }
extern "C" void ptc_graph_destroy(ptc_graph *g) {
    if (!g) return;
    cudaGraphExecDestroy(g->exec);
    delete g;
}

cudaStream_t ptc_ctx_stream(ptc_ctx *c) { return c->stream; }
int ptc_ctx_device(ptc_ctx *c) { return c->device; }

extern "C" int ptc_wait_deadline(ptc_ctx *c, int timeout_ms) {
    struct timespec t0, t;
    clock_gettime(CLOCK_MONOTONIC, &t0);
    for (;;) {
        cudaError_t e = cudaStreamQuery(c->stream);
        if (e == cudaSuccess) return 0;
        if (e != cudaErrorNotReady) PTC_CHECK(e);
        clock_gettime(CLOCK_MONOTONIC, &t);
        const long ms = (t.tv_sec - t0.tv_sec) * 1000L + (t.tv_nsec - t0.tv_nsec) / 1000000L;
        if (ms > timeout_ms) return 1;
    }
}
