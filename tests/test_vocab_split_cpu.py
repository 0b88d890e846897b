"""The argmax combination rule of the vocab-parallel classifier, on the CPU.

Each rank of a vocab-parallel decode reduces its rows [V*r/W, V*(r+1)/W) to
one packed key -- the logit's order-preserving bits in the high word and the
inverted global row index in the low word (ptc_common.cuh argmax_key) -- and
the combining ranks take the max over all ranks' keys. That must pick the
token of the reference's single scan with a strict '>' (pitorch/ops/core/
pt_ops.c:65-70, the oracle's or_argmax): the largest logit, and among equal
ones the lowest index, wherever the slice boundaries fall. The device kernels
run the same rule (test_pipeline_gpu checks their streams); this pins the rule
itself, with ties planted across slice boundaries.
"""
import ctypes

import numpy as np

import oracle


def float_key(v):
    u = int(np.float32(v).view(np.uint32))
    return (~u) & 0xFFFFFFFF if u & 0x80000000 else u | 0x80000000


def argmax_key(v, i):
    return (float_key(v) << 32) | (0xFFFFFFFF - i)


def key_index(k):
    return 0xFFFFFFFF - (k & 0xFFFFFFFF)


def split_argmax(logits, world):
    V = len(logits)
    keys = []
    for r in range(world):
        lo, hi = V * r // world, V * (r + 1) // world
        keys.append(max(argmax_key(logits[i], i) for i in range(lo, hi)))
    return key_index(max(keys))


def reference_argmax(logits):
    L = oracle.lib()
    L.or_argmax.restype = ctypes.c_int
    L.or_argmax.argtypes = [ctypes.POINTER(ctypes.c_float), ctypes.c_int]
    x = np.ascontiguousarray(logits, dtype=np.float32)
    return int(L.or_argmax(x.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), len(x)))


def test_split_argmax_equals_the_reference_scan():
    rng = np.random.default_rng(7)
    V = 1000
    for trial in range(40):
        x = (rng.standard_normal(V) * 3).astype(np.float32)
        if trial % 2:   # plant an exact tie of the maximum in two places, across slices
            m = np.float32(x.max() + 1.0)
            a, b = sorted(rng.choice(V, 2, replace=False))
            x[a] = x[b] = m
        if trial % 5 == 0:   # all logits negative
            x = -np.abs(x) - np.float32(1.0)
        want = reference_argmax(x)
        assert want == int(np.argmax(x))
        for world in (2, 3, 4, 7, 8):
            assert split_argmax(x, world) == want, (trial, world)


def test_tie_at_a_slice_boundary_keeps_the_lower_index():
    V, world = 64, 4
    x = np.full(V, -5.0, dtype=np.float32)
    x[15] = x[16] = 2.5   # the last row of slice 0 and the first of slice 1
    assert reference_argmax(x) == 15
    assert split_argmax(x, world) == 15
