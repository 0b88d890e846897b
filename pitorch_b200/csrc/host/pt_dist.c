/*
 * pt_dist.c -- the layer pipeline over NVLink (pitorch/dist/pt_dist_pipeline.c
 * on GPUs instead of a GPIO ring of Pi Zeros).
 *
 * One process per GPU. Links are an NCCL communicator: the reference's
 * blocking send_raw/recv_raw over the GPIO bus (pitorch/dist/transport/
 * pt_transport.h:15-18) become ncclSend/ncclRecv of device buffers on the
 * context's stream, so activations never touch the host. The message of a
 * decode hop keeps the reference's [int32 pos | float x[dim]] layout
 * (pt_dist_pipeline.c:287, 298-302); training hops carry the [T, dim]
 * residual stream forward and d_res backward (pt_dist_pipeline.c:134).
 *
 * Every wait is bounded by dist->timeout_ms: on expiry the rank prints a
 * FAIL line, aborts its communicator and returns an error code -- the
 * reference's recv_raw returns -1 after its 300 s first-byte timeout
 * (pt_link_gpio.c:134-136) and its callers reboot the board.
 */
#include <arpa/inet.h>
#include <errno.h>
#include <fcntl.h>
#include <netdb.h>
#include <netinet/in.h>
#include <netinet/tcp.h>
#include <poll.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/socket.h>
#include <sys/time.h>
#include <time.h>
#include <unistd.h>

#include <cuda_runtime.h>
#include <nccl.h>

#include "../../../include/pt_dist_pipeline.h"
#include "pt_device.h"

typedef struct {
    ncclComm_t comm;
    int device;
    float *sbuf, *rbuf;   /* [1 + dim] device message buffers: pos bits, x */
    float *scal;          /* device scratch scalar */
    int dim;
    int verbose;
    int step;
    /* decode hops over NVLink peer memory (ptc_hop_*), when every rank could
     * map its successor's mailbox; otherwise NCCL send/recv */
    int p2p;
    void *box;            /* this rank's mailbox (the predecessor writes it) */
    void *peer_box;       /* the successor's mailbox, mapped */
    unsigned *ctr;        /* device [0] messages sent, [1] messages received */
    int *hop_err;         /* device: a hop wait ran out */
    int *hop_err_host;    /* pinned copy of it, fetched with each host-driven step */
    /* vocab-parallel classifier (pt_dist_vocab_parallel) */
    int vp;
    void *vp_box;                      /* this rank's classifier mailbox */
    void *vp_peer[PTC_VP_MAX_RANKS];   /* other ranks' classifier mailboxes, mapped where needed */
    unsigned *vp_sent;                 /* device [0] residuals sent, [1] keys sent */
    int *tokmsg;                       /* device: the head's input token of a host-driven step */
} dist_comm_t;

static long now_ms(void) {
    struct timespec t;
    clock_gettime(CLOCK_MONOTONIC, &t);
    return t.tv_sec * 1000L + t.tv_nsec / 1000000L;
}

static int timeout_of(const pt_dist_t *d) { return d->timeout_ms > 0 ? d->timeout_ms : 300000; }

/* ---- TCP rendezvous for the NCCL unique id -------------------------------- */

static int set_nonblock(int fd, int on) {
    int fl = fcntl(fd, F_GETFL, 0);
    return fcntl(fd, F_SETFL, on ? (fl | O_NONBLOCK) : (fl & ~O_NONBLOCK));
}

static int io_full(int fd, unsigned char *buf, int n, int sending, long deadline) {
    int done = 0;
    while (done < n) {
        long left = deadline - now_ms();
        if (left <= 0) return -1;
        struct pollfd p = {fd, (short)(sending ? POLLOUT : POLLIN), 0};
        int r = poll(&p, 1, (int)(left > 1000 ? 1000 : left));
        if (r < 0 && errno != EINTR) return -1;
        if (r <= 0) continue;
        ssize_t k = sending ? send(fd, buf + done, n - done, MSG_NOSIGNAL) : recv(fd, buf + done, n - done, 0);
        if (k <= 0) {
            if (k < 0 && (errno == EAGAIN || errno == EINTR)) continue;
            return -1;
        }
        done += (int)k;
    }
    return 0;
}

int pt_dist_rendezvous(int rank, int world_size, const char *addr, int port, int timeout_ms,
                       unsigned char blob[128]) {
    const long deadline = now_ms() + timeout_ms;
    if (world_size <= 1) return 0;
    if (rank == 0) {
        int ls = socket(AF_INET, SOCK_STREAM, 0);
        if (ls < 0) return -1;
        int one = 1;
        setsockopt(ls, SOL_SOCKET, SO_REUSEADDR, &one, sizeof(one));
        struct sockaddr_in sa;
        memset(&sa, 0, sizeof(sa));
        sa.sin_family = AF_INET;
        sa.sin_port = htons((unsigned short)port);
        sa.sin_addr.s_addr = htonl(INADDR_ANY);
        if (bind(ls, (struct sockaddr *)&sa, sizeof(sa)) < 0 || listen(ls, world_size) < 0) {
            close(ls);
            return -1;
        }
        set_nonblock(ls, 1);
        int served = 0, rc = 0;
        while (served < world_size - 1) {
            long left = deadline - now_ms();
            if (left <= 0) { rc = -1; break; }
            struct pollfd p = {ls, POLLIN, 0};
            int r = poll(&p, 1, (int)(left > 1000 ? 1000 : left));
            if (r <= 0) continue;
            int fd = accept(ls, NULL, NULL);
            if (fd < 0) continue;
            set_nonblock(fd, 1);
            if (io_full(fd, blob, 128, 1, deadline) < 0) rc = -1;
            close(fd);
            if (rc < 0) break;
            served++;
        }
        close(ls);
        return rc;
    }
    for (;;) {
        if (now_ms() > deadline) return -1;
        int fd = socket(AF_INET, SOCK_STREAM, 0);
        if (fd < 0) return -1;
        struct sockaddr_in sa;
        memset(&sa, 0, sizeof(sa));
        sa.sin_family = AF_INET;
        sa.sin_port = htons((unsigned short)port);
        if (inet_pton(AF_INET, addr, &sa.sin_addr) != 1) {
            struct hostent *he = gethostbyname(addr);
            if (!he) { close(fd); return -1; }
            memcpy(&sa.sin_addr, he->h_addr_list[0], sizeof(sa.sin_addr));
        }
        if (connect(fd, (struct sockaddr *)&sa, sizeof(sa)) == 0) {
            set_nonblock(fd, 1);
            int rc = io_full(fd, blob, 128, 0, deadline);
            close(fd);
            return rc;
        }
        close(fd);
        usleep(50000);
    }
}

static int rendezvous_port(void) {
    const char *p = getenv("PT_DIST_PORT");
    if (p) return atoi(p);
    const char *m = getenv("MASTER_PORT");
    return m ? atoi(m) + 17 : 29517;
}

static const char *rendezvous_addr(void) {
    const char *a = getenv("MASTER_ADDR");
    return a ? a : "127.0.0.1";
}

/* ---- setup ------------------------------------------------------------------ */

static void fail(const pt_dist_t *d, const char *what) {
    fprintf(stderr, "FAIL: rank %d: %s\n", d->rank, what);
}

static dist_comm_t *comm_of(pt_dist_t *d) { return (dist_comm_t *)d->comm; }
static int finish(pt_dist_t *dist, pt_context_t *ctx, const char *what);
static long long hop_timeout_ns(const pt_dist_t *dist);
static int next_rank(const pt_dist_t *d) { return (d->rank + 1) % d->world_size; }
static int prev_rank(const pt_dist_t *d) { return (d->rank + d->world_size - 1) % d->world_size; }

/* All-gather the IPC handle of this rank's mailbox `box` (NULL: none) into
 * hh[world][PTC_MAILBOX_HANDLE_BYTES]. Returns 0, or -1 on a timeout. */
static int gather_handles(pt_dist_t *dist, pt_context_t *ctx, void *box, unsigned char *hh) {
    dist_comm_t *c = comm_of(dist);
    ptc_ctx *pc = ctx->dev->ctx;
    cudaStream_t s = (cudaStream_t)ptc_stream(pc);
    const int W = dist->world_size, H = PTC_MAILBOX_HANDLE_BYTES;
    unsigned char *dh = (unsigned char *)ptc_alloc(pc, (size_t)W * H);
    memset(hh, 0, (size_t)W * H);
    if (box) ptc_mailbox_handle(box, hh + (size_t)dist->rank * H);
    cudaMemcpyAsync(dh + (size_t)dist->rank * H, hh + (size_t)dist->rank * H, H, cudaMemcpyHostToDevice, s);
    ncclAllGather(dh + (size_t)dist->rank * H, dh, H, ncclUint8, c->comm, s);
    cudaMemcpyAsync(hh, dh, (size_t)W * H, cudaMemcpyDeviceToHost, s);
    return finish(dist, ctx, "mailbox exchange timeout");
}

/* 1 when every rank's `ok` is non-zero (a min all-reduce), -1 on a timeout. */
static int agree(pt_dist_t *dist, pt_context_t *ctx, int ok, const char *what) {
    dist_comm_t *c = comm_of(dist);
    cudaStream_t s = (cudaStream_t)ptc_stream(ctx->dev->ctx);
    float v = ok ? 1.f : 0.f;
    cudaMemcpyAsync(c->scal, &v, 4, cudaMemcpyHostToDevice, s);
    ncclAllReduce(c->scal, c->scal, 1, ncclFloat, ncclMin, c->comm, s);
    cudaMemcpyAsync(&v, c->scal, 4, cudaMemcpyDeviceToHost, s);
    if (finish(dist, ctx, what) < 0) return -1;
    return v < 1.f ? 0 : 1;
}

/* Decode hops over NVLink: allocate this rank's mailbox, all-gather the IPC
 * handles, map the successor's mailbox, and agree on the transport (every
 * rank must use the same one). PT_DIST_P2P=0 keeps NCCL send/recv. Returns
 * -1 only when a collective of the agreement times out. */
static int setup_p2p(pt_dist_t *dist, pt_context_t *ctx) {
    dist_comm_t *c = comm_of(dist);
    const char *e = getenv("PT_DIST_P2P");
    if (e && e[0] == '0') return 0;
    ptc_ctx *pc = ctx->dev->ctx;
    cudaStream_t s = (cudaStream_t)ptc_stream(pc);
    const int W = dist->world_size, H = PTC_MAILBOX_HANDLE_BYTES;
    unsigned char *hh = (unsigned char *)calloc((size_t)W, H);
    c->box = ptc_mailbox_alloc(pc, c->dim);
    unsigned char probe[PTC_MAILBOX_HANDLE_BYTES];
    int ok = c->box && ptc_mailbox_handle(c->box, probe) == 0;
    if (gather_handles(dist, ctx, ok ? c->box : NULL, hh) < 0) {
        free(hh);
        return -1;
    }
    if (ok) c->peer_box = ptc_mailbox_open(pc, hh + (size_t)next_rank(dist) * H);
    free(hh);
    ok = ok && c->peer_box;
    const int all = agree(dist, ctx, ok, "mailbox agreement timeout");
    if (all < 0) return -1;
    if (!all) {   /* somebody could not map its successor: NCCL hops everywhere */
        ptc_mailbox_close(c->peer_box);
        ptc_mailbox_free(c->box);
        c->peer_box = c->box = NULL;
        return 0;
    }
    c->ctr = (unsigned *)ptc_alloc(pc, 2 * sizeof(unsigned));
    c->hop_err = (int *)ptc_alloc(pc, sizeof(int));
    c->hop_err_host = (int *)ptc_host_alloc(sizeof(int));
    *c->hop_err_host = 0;
    cudaMemsetAsync(c->ctr, 0, 2 * sizeof(unsigned), s);
    cudaMemsetAsync(c->hop_err, 0, sizeof(int), s);
    c->p2p = 1;
    if (finish(dist, ctx, "mailbox setup timeout") < 0) return -1;
    /* the decoder takes its input from the mailbox and sends its output
     * itself: no receive kernels, and on the head rank no embedding or send
     * kernel per position */
    ptc_decoder_set_links(ctx->dev->dec, c->box, c->peer_box, c->ctr, c->hop_err, hop_timeout_ns(dist));
    return 0;
}

/* A decode hop wait that ran out on the GPU (after the stream finished). */
static long long hop_timeout_ns(const pt_dist_t *dist) {
    /* the GPU-side bound of one wait: the dist timeout, at most 60 s (the
     * host's deadline still bounds the whole call) */
    const int ms = timeout_of(dist) < 60000 ? timeout_of(dist) : 60000;
    return (long long)ms * 1000000LL;
}

/* The hop error word of a host-driven step: its copy into pinned memory is
 * enqueued with the step, so the step's one wait for the stream covers it. */
static void hop_err_enqueue(pt_dist_t *dist, pt_context_t *ctx) {
    dist_comm_t *c = comm_of(dist);
    if (c->p2p)
        cudaMemcpyAsync(c->hop_err_host, c->hop_err, sizeof(int), cudaMemcpyDeviceToHost,
                        (cudaStream_t)ptc_stream(ctx->dev->ctx));
}
static int hop_err_seen(const pt_dist_t *dist) {
    const dist_comm_t *c = (const dist_comm_t *)dist->comm;
    const int e = c->p2p ? *(volatile int *)c->hop_err_host : 0;
    if (e) fprintf(stderr, "R%d FAIL: decode hop wait expired\n", dist->rank);
    return e;
}

static int hop_failed(pt_dist_t *dist, pt_context_t *ctx) {
    dist_comm_t *c = comm_of(dist);
    if (!c->p2p) return 0;
    int e = 0;
    cudaMemcpyAsync(&e, c->hop_err, sizeof(int), cudaMemcpyDeviceToHost, (cudaStream_t)ptc_stream(ctx->dev->ctx));
    cudaStreamSynchronize((cudaStream_t)ptc_stream(ctx->dev->ctx));
    if (e) fprintf(stderr, "R%d FAIL: decode hop wait expired\n", dist->rank);
    return e;
}

static int join(pt_dist_t *dist, pt_context_t *ctx) {
    if (dist->comm) return 0;
    if (!ctx || !ctx->dev) pt_fatal("pipeline call without an initialised context");
    unsigned char id[128];
    memset(id, 0, sizeof(id));
    ncclUniqueId uid;
    if (dist->rank == 0) {
        if (ncclGetUniqueId(&uid) != ncclSuccess) pt_fatal("ncclGetUniqueId failed");
        memcpy(id, &uid, sizeof(uid) < 128 ? sizeof(uid) : 128);
    }
    if (pt_dist_rendezvous(dist->rank, dist->world_size, rendezvous_addr(), rendezvous_port(),
                           timeout_of(dist), id) < 0) {
        fail(dist, "ring rendezvous timeout");
        return -1;
    }
    memcpy(&uid, id, sizeof(uid));
    dist_comm_t *c = (dist_comm_t *)calloc(1, sizeof(dist_comm_t));
    c->device = ptc_device(ctx->dev->ctx);
    c->dim = ctx->cfg.dim;
    if (cudaSetDevice(c->device) != cudaSuccess) pt_fatal("cudaSetDevice(%d) failed", c->device);
    if (ncclCommInitRank(&c->comm, dist->world_size, uid, dist->rank) != ncclSuccess) {
        free(c);
        fail(dist, "ncclCommInitRank failed");
        return -1;
    }
    c->sbuf = (float *)ptc_alloc(ctx->dev->ctx, (size_t)(1 + c->dim) * 4);
    c->rbuf = (float *)ptc_alloc(ctx->dev->ctx, (size_t)(1 + c->dim) * 4);
    c->scal = (float *)ptc_alloc(ctx->dev->ctx, 256);
    dist->comm = c;
    if (setup_p2p(dist, ctx) < 0) return -1;
    return 0;
}

/* pt_dist_pipeline.c:26-33 */
void pt_dist_setup(pt_dist_t *dist, const pt_shard_info_t *shard, int rank, int world_size) {
    memset(dist, 0, sizeof(*dist));
    dist->rank = rank;
    dist->world_size = world_size;
    dist->l_start = 0;
    dist->l_end = shard->n_local;
    dist->has_embed = shard->has_embed;
    dist->has_head = shard->has_head;
    const char *t = getenv("PT_DIST_TIMEOUT_MS");
    dist->timeout_ms = t ? atoi(t) : 0;
}

int pt_dist_setup_ctx(pt_dist_t *dist, pt_context_t *ctx, const pt_shard_info_t *shard, int rank,
                      int world_size) {
    pt_dist_setup(dist, shard, rank, world_size);
    return join(dist, ctx);
}

void pt_dist_free(pt_dist_t *dist) {
    dist_comm_t *c = comm_of(dist);
    if (!c) return;
    if (c->hop_err_host) ptc_host_free(c->hop_err_host);
    for (int q = 0; q < PTC_VP_MAX_RANKS; q++) ptc_mailbox_close(c->vp_peer[q]);
    ptc_mailbox_free(c->vp_box);
    ptc_mailbox_close(c->peer_box);
    ptc_mailbox_free(c->box);
    if (c->comm) ncclCommDestroy(c->comm);
    free(c);
    dist->comm = NULL;
}

void pt_dist_set_verbose(pt_dist_t *dist, int verbose) {
    if (comm_of(dist)) comm_of(dist)->verbose = verbose;
}

void pt_dist_reset_links(pt_dist_t *dist) { (void)dist; }

int pt_dist_comm_size(const pt_dist_t *dist) {
    const dist_comm_t *c = (const dist_comm_t *)dist->comm;
    int n = -1;
    if (!c || !c->comm || ncclCommCount(c->comm, &n) != ncclSuccess) return -1;
    return n;
}

int pt_dist_transport(const pt_dist_t *dist) {
    const dist_comm_t *c = (const dist_comm_t *)dist->comm;
    return c ? c->p2p : -1;
}

/* Wait for the stream with the dist deadline; abort the communicator on expiry. */
static int finish(pt_dist_t *dist, pt_context_t *ctx, const char *what) {
    dist_comm_t *c = comm_of(dist);
    if (ptc_wait_deadline(ctx->dev->ctx, timeout_of(dist)) == 0) {
        ncclResult_t ae = ncclSuccess;
        ncclCommGetAsyncError(c->comm, &ae);
        if (ae == ncclSuccess) return 0;
    }
    fail(dist, what);
    ncclCommAbort(c->comm);
    c->comm = NULL;
    return -1;
}

static cudaStream_t stream_of(pt_context_t *ctx) { return (cudaStream_t)ptc_stream(ctx->dev->ctx); }

int pt_dist_ring_sync(pt_dist_t *dist) {
    (void)dist;
    return 0;
}

static int ring_sync_ctx(pt_dist_t *dist, pt_context_t *ctx) {
    dist_comm_t *c = comm_of(dist);
    if (!c || !c->comm) return -1;
    ncclAllReduce(c->scal, c->scal, 1, ncclFloat, ncclSum, c->comm, stream_of(ctx));
    return finish(dist, ctx, "ring handshake timeout");
}

float pt_dist_max_float(pt_context_t *ctx, pt_dist_t *dist, float v) {
    if (join(dist, ctx) < 0) return v;
    dist_comm_t *c = comm_of(dist);
    cudaStream_t s = stream_of(ctx);
    cudaMemcpyAsync(c->scal, &v, 4, cudaMemcpyHostToDevice, s);
    ncclAllReduce(c->scal, c->scal, 1, ncclFloat, ncclMax, c->comm, s);
    float out = v;
    cudaMemcpyAsync(&out, c->scal, 4, cudaMemcpyDeviceToHost, s);
    if (finish(dist, ctx, "max-over-ranks timeout") < 0) return v;
    return out;
}

int pt_dist_allreduce_grads_avg(pt_context_t *ctx, pt_dist_t *dist) {
    if (join(dist, ctx) < 0) return -1;
    dist_comm_t *c = comm_of(dist);
    if (!ctx->dev->trainer) pt_fatal("pt_dist_allreduce_grads_avg needs a training context");
    float *g = ptc_trainer_grads(ctx->dev->trainer);
    size_t n = ptc_trainer_n_params(ctx->dev->trainer);
    ncclAllReduce(g, g, n, ncclFloat, ncclAvg, c->comm, stream_of(ctx));
    return finish(dist, ctx, "gradient allreduce timeout");
}

/* ---- decode ------------------------------------------------------------------ */

/* Enqueue one position's hop sequence for this rank (no host sync). For the
 * head rank in device-loop mode the embedding reads the token from the
 * device and the head advances position/token on the device. */
static void enqueue_position(pt_dist_t *dist, pt_context_t *ctx, int host_token, int host_pos, int devloop) {
    dist_comm_t *c = comm_of(dist);
    ptc_decoder *dec = ctx->dev->dec;
    cudaStream_t s = stream_of(ctx);
    const size_t msg = (size_t)(1 + c->dim);
    float *x = ptc_decoder_x_dev(dec);
    int *pos_dev = ptc_decoder_pos_dev(dec);
    if (c->p2p) {
        /* link form: the decoder's stage graph of one position (its first
         * kernel waits for this rank's mailbox; a layer rank's last one
         * sends on). The head rank first sends the position's embedding row
         * itself: in host-driven steps the token is the caller's. */
        (void)devloop;
        if (dist->has_embed && dist->has_head) {
            ptc_decoder_enqueue_embed_at(dec, host_token, host_pos);
            ptc_hop_send(ctx->dev->ctx, x, pos_dev, c->peer_box, c->ctr, c->dim);
        }
        ptc_decoder_enqueue_stage(dec, 1);
        return;
    }
    if (dist->has_embed && dist->has_head) {
        if (devloop) {
            ptc_decoder_enqueue_embed_dev(dec);
        } else {
            ptc_decoder_enqueue_embed_at(dec, host_token, host_pos);
        }
        cudaMemcpyAsync(c->sbuf, pos_dev, 4, cudaMemcpyDeviceToDevice, s);
        cudaMemcpyAsync(c->sbuf + 1, x, (size_t)c->dim * 4, cudaMemcpyDeviceToDevice, s);
        ncclSend(c->sbuf, msg, ncclFloat, next_rank(dist), c->comm, s);
        ncclRecv(c->rbuf, msg, ncclFloat, prev_rank(dist), c->comm, s);
        cudaMemcpyAsync(x, c->rbuf + 1, (size_t)c->dim * 4, cudaMemcpyDeviceToDevice, s);
        ptc_decoder_enqueue_head(dec);
    } else {
        ncclRecv(c->rbuf, msg, ncclFloat, prev_rank(dist), c->comm, s);
        cudaMemcpyAsync(pos_dev, c->rbuf, 4, cudaMemcpyDeviceToDevice, s);
        cudaMemcpyAsync(x, c->rbuf + 1, (size_t)c->dim * 4, cudaMemcpyDeviceToDevice, s);
        ptc_decoder_enqueue_layers_devpos(dec, dist->l_start, dist->l_end);
        cudaMemcpyAsync(c->sbuf, c->rbuf, 4, cudaMemcpyDeviceToDevice, s);
        cudaMemcpyAsync(c->sbuf + 1, x, (size_t)c->dim * 4, cudaMemcpyDeviceToDevice, s);
        ncclSend(c->sbuf, msg, ncclFloat, next_rank(dist), c->comm, s);
    }
}

/* ---- vocab-parallel classifier --------------------------------------------- */

/* First classifier row of rank q's share: rank q computes rows
 * [vp_row(q), vp_row(q + 1)). */
static long vp_row(const pt_context_t *ctx, const pt_dist_t *d, int q) {
    return (long)ctx->dev->cfg.vocab_size * q / d->world_size;
}

static int is_head(const pt_dist_t *d) { return d->has_embed && d->has_head; }

/* Every rank computes the logits of its share of the classifier rows (the
 * reference's head rank computes them all, pitorch/model/llama2.c:194-198);
 * the last layer rank sends the final residual to every rank, and each rank
 * sends its argmax key to rank 0 (which embeds the next token itself) and to
 * the head rank (which keeps the token stream). The head sends every rank
 * its rows and the final rmsnorm gain once, and rank 0 the embedding table,
 * over NCCL; the decode hops stay peer stores over NVLink. */
int pt_dist_vocab_parallel(pt_context_t *ctx, pt_dist_t *dist) {
    if (join(dist, ctx) < 0) return -1;
    dist_comm_t *c = comm_of(dist);
    if (!c->comm) return -1;
    if (c->vp) return 0;
    const int W = dist->world_size, r = dist->rank, head = W - 1, last = W - 2;
    const struct pt_device *dv = ctx->dev;
    const int dim = dv->cfg.dim, V = dv->cfg.vocab_size, n_local = dv->cfg.n_layers;
    /* the reference's layout: layers on ranks 0..W-2, embedding + classifier on the last */
    int ok = c->p2p && W >= 2 && W <= PTC_VP_MAX_RANKS && V >= W && (r == head) == (is_head(dist) != 0) &&
             (r == head ? n_local == 0 : n_local > 0);
    int all = agree(dist, ctx, ok, "vocab-parallel agreement timeout");
    if (all <= 0) {
        if (all == 0 && r == 0)
            fprintf(stderr, "R%d: vocab-parallel classifier needs the NVLink hop transport, 2..%d ranks and the "
                            "layers-then-head layout\n", r, PTC_VP_MAX_RANKS);
        return -1;
    }
    ptc_ctx *pc = dv->ctx;
    cudaStream_t s = stream_of(ctx);
    const long r0 = vp_row(ctx, dist, r), nr = vp_row(ctx, dist, r + 1) - r0;
    const float *rows, *gain, *table = NULL;
    ncclGroupStart();
    if (r == head) {
        rows = dv->dw.wcls + (size_t)r0 * dim;
        gain = dv->dw.rms_final_weight;
        for (int q = 0; q < head; q++) {
            const long q0 = vp_row(ctx, dist, q), qn = vp_row(ctx, dist, q + 1) - q0;
            ncclSend(gain, (size_t)dim, ncclFloat, q, c->comm, s);
            ncclSend(dv->dw.wcls + (size_t)q0 * dim, (size_t)qn * dim, ncclFloat, q, c->comm, s);
            if (q == 0) ncclSend(dv->dw.token_embedding, (size_t)V * dim, ncclFloat, 0, c->comm, s);
        }
    } else {
        float *g = (float *)ptc_alloc(pc, (size_t)dim * 4);
        float *w = (float *)ptc_alloc(pc, (size_t)nr * dim * 4);
        ncclRecv(g, (size_t)dim, ncclFloat, head, c->comm, s);
        ncclRecv(w, (size_t)nr * dim, ncclFloat, head, c->comm, s);
        if (r == 0) {
            float *t = (float *)ptc_alloc(pc, (size_t)V * dim * 4);
            ncclRecv(t, (size_t)V * dim, ncclFloat, head, c->comm, s);
            table = t;
        }
        rows = w;
        gain = g;
    }
    ncclGroupEnd();
    if (finish(dist, ctx, "vocab-parallel weights timeout") < 0) return -1;

    /* mailboxes: every rank's, mapped by the ranks that write it */
    const int H = PTC_MAILBOX_HANDLE_BYTES;
    unsigned char *hh = (unsigned char *)calloc((size_t)W, H);
    c->vp_box = ptc_mailbox_alloc(pc, dim + 4 * W);
    if (gather_handles(dist, ctx, c->vp_box, hh) < 0) {
        free(hh);
        return -1;
    }
    ok = c->vp_box != NULL;
    for (int q = 0; q < W && ok; q++) {
        const int need = q != r && (q == 0 || q == head || r == last);
        if (need) ok = (c->vp_peer[q] = ptc_mailbox_open(pc, hh + (size_t)q * H)) != NULL;
    }
    free(hh);
    all = agree(dist, ctx, ok, "vocab-parallel mailbox timeout");
    if (all <= 0) {
        for (int q = 0; q < W; q++) {
            ptc_mailbox_close(c->vp_peer[q]);
            c->vp_peer[q] = NULL;
        }
        ptc_mailbox_free(c->vp_box);
        c->vp_box = NULL;
        return -1;
    }
    c->vp_sent = (unsigned *)ptc_alloc(pc, 2 * sizeof(unsigned));
    c->tokmsg = (int *)ptc_alloc(pc, 16);
    cudaMemsetAsync(c->vp_sent, 0, 2 * sizeof(unsigned), s);
    if (finish(dist, ctx, "vocab-parallel setup timeout") < 0) return -1;

    ptc_vocab_split vp;
    memset(&vp, 0, sizeof(vp));
    vp.row0 = (int)r0;
    vp.rows = (int)nr;
    vp.ranks = W;
    vp.rank = r;
    vp.combine = r == 0 || r == head;
    vp.x_local = r == last;
    vp.embed_local = r == 0;
    vp.cls_rows = rows;
    vp.rms_final = gain;
    vp.embedding = table;
    vp.box = c->vp_box;
    if (r == last)
        for (int q = 0; q < W; q++)
            if (q != r) vp.x_out[vp.n_x_out++] = c->vp_peer[q];
    if (r != 0) vp.key_out[vp.n_key_out++] = c->vp_peer[0];
    if (r != head) vp.key_out[vp.n_key_out++] = c->vp_peer[head];
    vp.sent = c->vp_sent;
    ptc_decoder_set_vocab_parallel(dv->dec, &vp);
    c->vp = 1;
    return 0;
}

int pt_dist_is_vocab_parallel(const pt_dist_t *dist) {
    const dist_comm_t *c = (const dist_comm_t *)dist->comm;
    return c && c->vp;
}

/* The head rank's logits of a host-driven step: every rank's share of the
 * rows, gathered over NCCL (each rank wrote its rows at their global index). */
static void vp_gather_logits(pt_dist_t *dist, pt_context_t *ctx) {
    dist_comm_t *c = comm_of(dist);
    cudaStream_t s = stream_of(ctx);
    float *lg = ptc_decoder_logits_dev(ctx->dev->dec);
    const int head = dist->world_size - 1;
    ncclGroupStart();
    if (dist->rank == head) {
        for (int q = 0; q < head; q++) {
            const long q0 = vp_row(ctx, dist, q), qn = vp_row(ctx, dist, q + 1) - q0;
            ncclRecv(lg + q0, (size_t)qn, ncclFloat, q, c->comm, s);
        }
    } else {
        const long r0 = vp_row(ctx, dist, dist->rank), nr = vp_row(ctx, dist, dist->rank + 1) - r0;
        ncclSend(lg + r0, (size_t)nr, ncclFloat, head, c->comm, s);
    }
    ncclGroupEnd();
}

/* One host-driven position with the vocab-parallel classifier: the head's
 * token goes to every rank (an NCCL broadcast; rank 0 embeds it), every rank
 * replays its one-position stage graph, and the head gathers the logits when
 * the caller keeps host logits. */
static int vp_forward_step(pt_context_t *ctx, pt_dist_t *dist, int token) {
    dist_comm_t *c = comm_of(dist);
    ptc_decoder *dec = ctx->dev->dec;
    cudaStream_t s = stream_of(ctx);
    const int head = dist->world_size - 1;
    if (dist->rank == head) cudaMemcpyAsync(c->tokmsg, &token, sizeof(int), cudaMemcpyHostToDevice, s);
    ncclBroadcast(c->tokmsg, c->tokmsg, 1, ncclInt, head, c->comm, s);
    if (dist->rank == 0) ptc_decoder_set_input(dec, ctx->pos, c->tokmsg);
    else if (dist->rank == head) ptc_decoder_set_input(dec, ctx->pos, NULL);
    ptc_decoder_enqueue_stage(dec, 1);
    if (ctx->sync_logits) vp_gather_logits(dist, ctx);
    hop_err_enqueue(dist, ctx);
    if (dist->rank == head) ptc_decoder_enqueue_fetch(dec, ctx->sync_logits);
    if (finish(dist, ctx, "dist forward timeout") < 0) return -1;
    if (hop_err_seen(dist)) return -1;
    int next = 0;
    if (dist->rank == head) next = ptc_decoder_take_next(dec, ctx->sync_logits ? ctx->state.logits : NULL);
    ctx->pos++;
    return next;
}

/* pt_dist_pipeline.c:284-372 */
int pt_dist_forward_step(pt_context_t *ctx, pt_dist_t *dist, int token) {
    if (join(dist, ctx) < 0) return -1;
    dist_comm_t *c = comm_of(dist);
    if (!c->comm) return -1;
    if (dist->world_size < 2) pt_fatal("pt_dist_forward_step needs world_size >= 2");
    if (dist->has_embed && dist->has_head && (token < 0 || token >= ctx->cfg.vocab_size))
        pt_fatal("token %d outside [0, %d)", token, ctx->cfg.vocab_size);
    long t0 = now_ms();
    int next = 0;
    if (c->vp) {
        if ((next = vp_forward_step(ctx, dist, token)) < 0) return -1;
    } else {
        /* one wait per step: the hop error word, the argmax, the kernels'
         * error word and the logits are copied back by work enqueued with it */
        enqueue_position(dist, ctx, token, ctx->pos, 0);
        hop_err_enqueue(dist, ctx);
        const int head = dist->has_embed && dist->has_head;
        if (head) ptc_decoder_enqueue_fetch(ctx->dev->dec, ctx->sync_logits);
        if (finish(dist, ctx, "dist forward recv timeout") < 0) return -1;
        if (hop_err_seen(dist)) return -1;
        if (head) {
            next = ptc_decoder_take_next(ctx->dev->dec, ctx->sync_logits ? ctx->state.logits : NULL);
            ctx->pos++;
        }
    }
    if (c->verbose)
        printf("R%d pos %d -> %d | %ldms\n", dist->rank, c->step, next, now_ms() - t0);
    c->step++;
    return next;
}

int pt_dist_generate_greedy(pt_context_t *ctx, pt_dist_t *dist, const int *prompt, int n_prompt, int n_pos,
                            int *out_tokens) {
    if (join(dist, ctx) < 0) return -1;
    dist_comm_t *c = comm_of(dist);
    if (!c->comm) return -1;
    ptc_decoder *dec = ctx->dev->dec;
    if (n_pos > ctx->cfg.seq_len) n_pos = ctx->cfg.seq_len;
    ptc_decoder_reset(dec);   /* also position 0 */
    if (dist->has_embed && dist->has_head) ptc_decoder_generate_begin(dec, prompt, n_prompt);
    if (c->vp) {
        /* vocab-parallel: rank 0 selects tokens too (it embeds them) */
        if (dist->rank == 0) ptc_decoder_generate_begin(dec, prompt, n_prompt);
        ptc_decoder_enqueue_stage(dec, n_pos);
    } else if (c->p2p) {
        /* Link form: the head rank sends position 0's embedding row; from
         * then on every position's input travels inside the decode kernels
         * (the classifier sends the next embedding row, the layer ranks
         * send their outputs), replayed from the decoders' stage graphs. */
        if (dist->has_embed && dist->has_head) {
            ptc_decoder_set_stop(dec, n_pos);
            const float *row = ctx->dev->dw.token_embedding + (size_t)prompt[0] * ctx->cfg.dim;
            ptc_hop_send(ctx->dev->ctx, row, ptc_decoder_pos_dev(dec), c->peer_box, c->ctr, c->dim);
        }
        ptc_decoder_enqueue_stage(dec, n_pos);
    } else {
        for (int p = 0; p < n_pos; p++) enqueue_position(dist, ctx, 0, 0, 1);
    }
    if (finish(dist, ctx, "dist generate timeout") < 0) return -1;
    if (hop_failed(dist, ctx)) return -1;
    if (dist->has_embed && dist->has_head) {
        ptc_decoder_read_tokens(dec, out_tokens, n_pos);
        ctx->pos = n_pos;
    }
    if (c->vp) ctx->pos = n_pos;
    return 0;
}

/* ---- training (pt_dist_pipeline.c:128-278) ----------------------------------- */

pt_dist_result_t pt_dist_train_step(pt_context_t *ctx, pt_dist_t *dist, const int *tokens, int T, float lr) {
    pt_dist_result_t res = {0.0f, 0};
    if (join(dist, ctx) < 0) return res;
    dist_comm_t *c = comm_of(dist);
    if (!c->comm) return res;
    ptc_trainer *tr = ctx->dev->trainer;
    if (!tr) pt_fatal("pt_dist_train_step needs a context initialised with max_T > 0");
    cudaStream_t s = stream_of(ctx);
    const long t0 = now_ms();
    const int n_local = dist->l_end - dist->l_start;
    const size_t act = (size_t)T * ctx->cfg.dim;
    ptc_trainer_set_tokens(tr, tokens, T);
    ptc_trainer_zero_grads(tr);
    if (dist->has_embed && dist->has_head) {
        ptc_trainer_fwd_embed(tr);
        ncclSend(ptc_trainer_residual(tr, 0), act, ncclFloat, next_rank(dist), c->comm, s);
        ncclRecv(ptc_trainer_residual(tr, n_local), act, ncclFloat, prev_rank(dist), c->comm, s);
        if (finish(dist, ctx, "recv fwd act") < 0) return res;
        const float loss = ptc_trainer_fwd_head(tr);
        ptc_trainer_bwd_head(tr);
        ncclSend(ptc_trainer_dres(tr), act, ncclFloat, prev_rank(dist), c->comm, s);
        ncclRecv(ptc_trainer_dres(tr), act, ncclFloat, next_rank(dist), c->comm, s);
        ptc_trainer_bwd_embed(tr);
        ptc_trainer_sgd_head(tr, lr);
        if (finish(dist, ctx, "recv bwd d_res") < 0) return res;
        res.loss = loss;
    } else {
        ncclRecv(ptc_trainer_residual(tr, 0), act, ncclFloat, prev_rank(dist), c->comm, s);
        ptc_trainer_fwd_layers(tr, 0, n_local);
        ncclSend(ptc_trainer_residual(tr, n_local), act, ncclFloat, next_rank(dist), c->comm, s);
        ncclRecv(ptc_trainer_dres(tr), act, ncclFloat, next_rank(dist), c->comm, s);
        ptc_trainer_bwd_layers(tr, 0, n_local);
        ncclSend(ptc_trainer_dres(tr), act, ncclFloat, prev_rank(dist), c->comm, s);
        ptc_trainer_sgd_layers(tr, lr, 0, n_local);
        if (finish(dist, ctx, "recv bwd d_res") < 0) return res;
    }
    ptc_decoder_weights_updated(ctx->dev->dec);
    long dt = now_ms() - t0;
    res.total_ms = (unsigned)(dt > 0 ? dt : 1);
    if (c->verbose) printf("R%d STEP %d | loss %.4f | %ums\n", dist->rank, c->step, res.loss, res.total_ms);
    c->step++;
    (void)ring_sync_ctx;
    return res;
}

/* ---- GPipe microbatched training (dev/tests/dist/train_pp/test_train_pp_mb_rank0.c,
 *      _rank1.c: the same fill/drain order, on NCCL instead of GPIO) ---------- */

/* Select microbatch set m and return its buffer of layer l's residual input. */
static float *set_res(ptc_trainer *tr, int m, int l) {
    ptc_trainer_select(tr, m);
    return ptc_trainer_residual(tr, l);
}
static float *set_dres(ptc_trainer *tr, int m) {
    ptc_trainer_select(tr, m);
    return ptc_trainer_dres_save(tr);
}

pt_dist_result_t pt_dist_train_step_mb(pt_context_t *ctx, pt_dist_t *dist, const int *tokens, int T, int n_mb,
                                       float lr) {
    pt_dist_result_t res = {0.0f, 0};
    if (join(dist, ctx) < 0) return res;
    dist_comm_t *c = comm_of(dist);
    if (!c->comm) return res;
    ptc_trainer *tr = ctx->dev->trainer;
    if (!tr) pt_fatal("pt_dist_train_step_mb needs a context initialised with max_T > 0");
    if (n_mb < 1 || n_mb > 16) pt_fatal("pt_dist_train_step_mb: n_mb=%d outside [1, 16]", n_mb);
    cudaStream_t s = stream_of(ctx);
    const long t0 = now_ms();
    const int M = n_mb, n_local = dist->l_end - dist->l_start;
    const int nxt = next_rank(dist), prv = prev_rank(dist);
    const size_t act = (size_t)T * ctx->cfg.dim, act_bytes = act * sizeof(float);
    const int head = dist->has_embed && dist->has_head;
    ptc_trainer_set_microbatches(tr, M);
    ptc_trainer_zero_grads(tr);

    /* forward: the head embeds microbatch m and sends it round the ring while
     * the layer ranks work on earlier ones; each send of one microbatch is
     * grouped with the receive of the next, so neighbours never wait on each
     * other in opposite orders */
    float loss_sum = 0.0f;
    if (head) {
        for (int m = 0; m < M; m++) {
            ptc_trainer_select(tr, m);
            ptc_trainer_set_tokens(tr, tokens + (size_t)m * T, T);
            ptc_trainer_fwd_embed(tr);
            float *out = ptc_trainer_residual(tr, 0);
            if (m == 0) {
                ncclSend(out, act, ncclFloat, nxt, c->comm, s);
            } else {
                float *in_prev = set_res(tr, m - 1, 0);   /* x after the last layer, microbatch m - 1 */
                ncclGroupStart();
                ncclSend(out, act, ncclFloat, nxt, c->comm, s);
                ncclRecv(in_prev, act, ncclFloat, prv, c->comm, s);
                ncclGroupEnd();
            }
        }
        ncclRecv(set_res(tr, M - 1, 0), act, ncclFloat, prv, c->comm, s);
        if (finish(dist, ctx, "recv fwd act") < 0) return res;
        for (int m = 0; m < M; m++) {
            ptc_trainer_select(tr, m);
            loss_sum += ptc_trainer_fwd_head(tr);
        }
    } else {
        for (int m = 0; m < M; m++) {
            ptc_trainer_select(tr, m);
            ptc_trainer_set_T(tr, T);   /* a layer rank gets rows, not tokens */
            float *in = ptc_trainer_residual(tr, 0);
            if (m == 0) {
                ncclRecv(in, act, ncclFloat, prv, c->comm, s);
            } else {
                float *out_prev = set_res(tr, m - 1, n_local);
                ptc_trainer_select(tr, m);
                ncclGroupStart();
                ncclSend(out_prev, act, ncclFloat, nxt, c->comm, s);
                ncclRecv(in, act, ncclFloat, prv, c->comm, s);
                ncclGroupEnd();
            }
            ptc_trainer_fwd_layers(tr, 0, n_local);
        }
        ncclSend(set_res(tr, M - 1, n_local), act, ncclFloat, nxt, c->comm, s);
    }

    /* backward, microbatches M-1 .. 0: d_res goes the other way round; every
     * microbatch keeps its own d_res buffer while it is in flight */
    if (head) {
        for (int i = 0; i < M; i++) {
            const int m = M - 1 - i;
            ptc_trainer_select(tr, m);
            ptc_trainer_bwd_head(tr);
            float *d_out = ptc_trainer_dres_save(tr);
            cudaMemcpyAsync(d_out, ptc_trainer_dres(tr), act_bytes, cudaMemcpyDeviceToDevice, s);
            if (i == 0) {
                ncclSend(d_out, act, ncclFloat, prv, c->comm, s);
            } else {
                float *d_back = set_dres(tr, m + 1);   /* microbatch m + 1 back from rank 0 */
                ncclGroupStart();
                ncclSend(d_out, act, ncclFloat, prv, c->comm, s);
                ncclRecv(d_back, act, ncclFloat, nxt, c->comm, s);
                ncclGroupEnd();
                cudaMemcpyAsync(ptc_trainer_dres(tr), d_back, act_bytes, cudaMemcpyDeviceToDevice, s);
                ptc_trainer_bwd_embed(tr);
            }
        }
        float *d_back = set_dres(tr, 0);
        ncclRecv(d_back, act, ncclFloat, nxt, c->comm, s);
        cudaMemcpyAsync(ptc_trainer_dres(tr), d_back, act_bytes, cudaMemcpyDeviceToDevice, s);
        ptc_trainer_bwd_embed(tr);
        ptc_trainer_sgd_head(tr, lr);
    } else {
        for (int i = 0; i < M; i++) {
            const int m = M - 1 - i;
            float *d_in = set_dres(tr, m);
            if (i == 0) {
                ncclRecv(d_in, act, ncclFloat, nxt, c->comm, s);
            } else {
                float *d_prev = set_dres(tr, m + 1);
                ptc_trainer_select(tr, m);
                ncclGroupStart();
                ncclSend(d_prev, act, ncclFloat, prv, c->comm, s);
                ncclRecv(d_in, act, ncclFloat, nxt, c->comm, s);
                ncclGroupEnd();
            }
            cudaMemcpyAsync(ptc_trainer_dres(tr), d_in, act_bytes, cudaMemcpyDeviceToDevice, s);
            ptc_trainer_bwd_layers(tr, 0, n_local);
            cudaMemcpyAsync(d_in, ptc_trainer_dres(tr), act_bytes, cudaMemcpyDeviceToDevice, s);
        }
        ncclSend(set_dres(tr, 0), act, ncclFloat, prv, c->comm, s);
        ptc_trainer_sgd_layers(tr, lr, 0, n_local);
    }
    ptc_trainer_select(tr, 0);
    if (finish(dist, ctx, "microbatch pipeline step") < 0) return res;
    ptc_decoder_weights_updated(ctx->dev->dec);
    long dt = now_ms() - t0;
    res.total_ms = (unsigned)(dt > 0 ? dt : 1);
    res.loss = head ? loss_sum / (float)M : 0.0f;
    if (c->verbose)
        printf("R%d STEP %d | %d microbatches | loss %.4f | %ums\n", dist->rank, c->step, M, res.loss, res.total_ms);
    c->step++;
    return res;
}
