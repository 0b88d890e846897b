// ptc_p2p.cu -- the decode pipeline's activation hop as stores into the next
// rank's memory over NVLink.
//
// pitorch moves a decode hop's [pos | x] message between boards with a
// blocking GPIO send/recv (pitorch/dist/pt_dist_pipeline.c:287-333,
// pitorch/dist/transport/pt_transport.h:15-18). Here every rank owns a
// mailbox in its own device memory, exported to its predecessor with CUDA
// IPC. The sender's kernel writes pos and x straight into the successor's
// mailbox (peer stores over NVLink), makes them visible system-wide, and
// then publishes a sequence number. The receiver's kernel waits for that
// number -- bounded by a deadline on %globaltimer, after which it records an
// error and returns -- and copies the message into the decoder's own
// buffers. A link carries one message at a time (the next one is only sent
// after the ring came round), so one slot per mailbox suffices.
#include "../../include/ptc.h"
#include "ptc_common.cuh"
#include "ptc_internal.h"

namespace ptc {

static size_t mailbox_bytes(int dim) { return sizeof(MailboxHeader) + (size_t)dim * 4; }

__global__ void k_hop_send(const float *__restrict__ x, const int *__restrict__ pos, unsigned char *peer,
                           unsigned *sent, int dim) {
    MailboxHeader *h = reinterpret_cast<MailboxHeader *>(peer);
    float *px = reinterpret_cast<float *>(peer + sizeof(MailboxHeader));
    const float4 *x4 = reinterpret_cast<const float4 *>(x);
    float4 *p4 = reinterpret_cast<float4 *>(px);
    for (int i = threadIdx.x; i < dim / 4; i += blockDim.x) p4[i] = __ldcg(x4 + i);
    for (int i = (dim / 4) * 4 + threadIdx.x; i < dim; i += blockDim.x) px[i] = __ldcg(x + i);
    if (threadIdx.x == 0) h->pos = __ldcg(pos);
    __threadfence_system();   // this thread's stores reach the peer before the flag
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned s = *sent + 1;
        *sent = s;
        st_release_sys(&h->seq, s);
    }
}

// The kernel after a receive may start at once (programmatic dependent
// launch): it streams its weights while this one waits, and reads x only
// after its griddepcontrol.wait, i.e. after this kernel has completed.
__global__ void k_hop_recv(const unsigned char *box, float *__restrict__ x, int *pos, unsigned *recvd, int dim,
                           int *err, unsigned long long timeout_ns) {
    pdl_trigger();
    const MailboxHeader *h = reinterpret_cast<const MailboxHeader *>(box);
    const float *bx = reinterpret_cast<const float *>(box + sizeof(MailboxHeader));
    __shared__ int s_ok;
    if (threadIdx.x == 0) {
        const unsigned want = *recvd + 1;
        const unsigned long long t0 = globaltimer_ns();
        // after one expired wait the link is broken: the hops queued behind
        // it return at once instead of each waiting out its own deadline
        int ok = 0;
        for (int broken = *(volatile int *)err; !broken;) {
            if ((int)(ld_acquire_sys(&h->seq) - want) >= 0) {
                ok = 1;
                break;
            }
            if (globaltimer_ns() - t0 > timeout_ns) break;
            __nanosleep(128);
        }
        if (ok) *recvd = want;
        else atomicExch(err, 1);
        s_ok = ok;
    }
    __syncthreads();
    if (!s_ok) return;
    const float4 *b4 = reinterpret_cast<const float4 *>(bx);
    float4 *x4 = reinterpret_cast<float4 *>(x);
    for (int i = threadIdx.x; i < dim / 4; i += blockDim.x) x4[i] = __ldcv(b4 + i);
    for (int i = (dim / 4) * 4 + threadIdx.x; i < dim; i += blockDim.x) x[i] = __ldcv(bx + i);
    if (pos && threadIdx.x == 0) *pos = __ldcv(&h->pos);
}

}  // namespace ptc

extern "C" void *ptc_mailbox_alloc(ptc_ctx *c, int dim) {
    PTC_CHECK(cudaSetDevice(ptc_device(c)));
    void *p = nullptr;
    if (cudaMalloc(&p, ptc::mailbox_bytes(dim)) != cudaSuccess) return nullptr;
    PTC_CHECK(cudaMemset(p, 0, ptc::mailbox_bytes(dim)));
    return p;
}

extern "C" void ptc_mailbox_free(void *box) {
    if (box) cudaFree(box);
}

extern "C" int ptc_mailbox_handle(void *box, void *handle_out) {
    cudaIpcMemHandle_t h;
    if (cudaIpcGetMemHandle(&h, box) != cudaSuccess) return -1;
    memcpy(handle_out, &h, sizeof(h) < PTC_MAILBOX_HANDLE_BYTES ? sizeof(h) : PTC_MAILBOX_HANDLE_BYTES);
    return 0;
}

extern "C" void *ptc_mailbox_open(ptc_ctx *c, const void *handle) {
    PTC_CHECK(cudaSetDevice(ptc_device(c)));
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    void *p = nullptr;
    if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    return p;
}

extern "C" void ptc_mailbox_close(void *peer) {
    if (peer) cudaIpcCloseMemHandle(peer);
}

extern "C" void ptc_hop_send(ptc_ctx *c, const float *x, const int *pos, void *peer_box, unsigned *sent, int dim) {
    ptc::k_hop_send<<<1, 256, 0, ptc_ctx_stream(c)>>>(x, pos, (unsigned char *)peer_box, sent, dim);
    PTC_CHECK(cudaGetLastError());
}

extern "C" void ptc_hop_recv(ptc_ctx *c, const void *box, float *x, int *pos, unsigned *recvd, int dim, int *err,
                             long long timeout_ns) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(256);
    cfg.stream = ptc_ctx_stream(c);
    PTC_CHECK(cudaLaunchKernelEx(&cfg, ptc::k_hop_recv, (const unsigned char *)box, x, pos, recvd, dim, err,
                                 (unsigned long long)timeout_ns));
}
