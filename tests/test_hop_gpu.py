"""The pipeline hop's bounded wait on one GPU (ptc_hop_recv, ptc_p2p.cu).

The reference's link receive gives up after its timeout and returns -1
(pitorch/dist/transport/pt_link_gpio.c:134-136); here the receiving kernel
polls its mailbox against a %globaltimer deadline, and on expiry records an
error word and returns without copying anything. These checks make that
deadline run out on purpose, with a mailbox in this GPU's own memory that
nobody sends to: a bounded wait that ends by itself, so no GPU is hung. A
matching send then shows the same link still delivers once the error word is
cleared.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

DIM = 64


class Dev:
    def __init__(self, L):
        self.L = L
        self.c = L.ptc_create(0, 0)

    def put(self, a):
        a = np.ascontiguousarray(a)
        p = self.L.ptc_alloc(self.c, a.nbytes)
        self.L.ptc_h2d(self.c, p, a.ctypes.data, a.nbytes)
        return p

    def get(self, p, like):
        out = np.zeros_like(like)
        self.L.ptc_d2h(self.c, out.ctypes.data, p, out.nbytes)
        return out


def timed_recv(L, dev, box, x, pos, recvd, err, timeout_ns):
    t = L.ptc_timer_create(dev.c)
    L.ptc_timer_start(t)
    L.ptc_hop_recv(dev.c, box, x, pos, recvd, DIM, err, timeout_ns)
    L.ptc_timer_stop(t)
    ms = L.ptc_timer_ms(t)
    L.ptc_timer_destroy(t)
    return ms


def test_hop_wait_expires_and_reports(ptlib):
    L = ptlib
    dev = Dev(L)
    box = L.ptc_mailbox_alloc(dev.c, DIM)
    assert box
    try:
        sentinel = np.full(DIM, 7.5, np.float32)
        x = dev.put(sentinel)
        pos = dev.put(np.array([-3], np.int32))
        recvd = dev.put(np.zeros(1, np.uint32))
        err = dev.put(np.zeros(1, np.int32))
        # nobody sends: the 1 ms deadline runs out
        ms = timed_recv(L, dev, box, x, pos, recvd, err, 1_000_000)
        assert ms >= 0.9, ms
        assert dev.get(err, np.zeros(1, np.int32))[0] == 1
        assert dev.get(recvd, np.zeros(1, np.uint32))[0] == 0
        assert np.array_equal(dev.get(x, sentinel), sentinel)
        assert dev.get(pos, np.zeros(1, np.int32))[0] == -3
        # the link is marked broken: the next receive returns at once
        # instead of waiting out a second (here 10 s) deadline
        ms2 = timed_recv(L, dev, box, x, pos, recvd, err, 10_000_000_000)
        assert ms2 < 100.0, ms2
        assert dev.get(recvd, np.zeros(1, np.uint32))[0] == 0
        assert np.array_equal(dev.get(x, sentinel), sentinel)

        # a message that does arrive is delivered once the error is cleared:
        # send into this GPU's own mailbox, then receive it
        msg = np.arange(DIM, dtype=np.float32)
        src = dev.put(msg)
        spos = dev.put(np.array([41], np.int32))
        sent = dev.put(np.zeros(1, np.uint32))
        L.ptc_memset(dev.c, err, 0, 4)
        L.ptc_hop_send(dev.c, src, spos, box, sent, DIM)
        ms3 = timed_recv(L, dev, box, x, pos, recvd, err, 1_000_000_000)
        assert dev.get(err, np.zeros(1, np.int32))[0] == 0
        assert dev.get(recvd, np.zeros(1, np.uint32))[0] == 1
        assert np.array_equal(dev.get(x, msg), msg)
        assert dev.get(pos, np.zeros(1, np.int32))[0] == 41
        assert ms3 < 100.0, ms3
    finally:
        L.ptc_mailbox_free(box)
        L.ptc_destroy(dev.c)
