"""ptc_sgemm_noalloc: the training GEMM for callers that cannot allocate.

Callers that run inside CUDA stream capture, inside an allocator callback,
or under a framework that owns every device allocation cannot call
cudaMalloc and may have no workspace to hand over. ptc_sgemm_noalloc keeps
its split-K partials in a static device array instead. This test calls it
through the C ABI and checks it against ptc_sgemm (given a caller workspace
of the same size) on two calls in a row, with different inputs each time so
that the partials the first call leaves in the shared array cannot leak into
the second, including products whose partials are read back from the array by
the split-K reduction kernel. The file is named to be collected last.
"""
import ctypes as C

import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu

MAX_MN = 1 << 20   # PTC_SGEMM_NOALLOC_MAX_MN in include/ptc.h
TOL = 1e-5         # the tolerance of tests/test_gemm_gpu.py


def test_noalloc_matches_sgemm_on_two_calls(ptlib):
    L = ptlib
    c = L.ptc_create(0, 0)
    try:
        stream = L.ptc_stream(c)
        # the classifier input-gradient shape of pt_train_step: K = vocab,
        # long enough that both entry points split K
        M, N, K = 255, 288, 32000

        def put(a):
            a = np.ascontiguousarray(a, np.float32)
            p = L.ptc_alloc(c, a.nbytes)
            L.ptc_h2d(c, p, a.ctypes.data, a.nbytes)
            return p

        def get(p):
            out = np.zeros((M, N), np.float32)
            L.ptc_d2h(c, out.ctypes.data, p, out.nbytes)
            return out

        ws = L.ptc_alloc(c, MAX_MN * 4)
        for call in range(2):
            rng = np.random.default_rng(100 + call)
            A = rng.standard_normal((M, K), dtype=np.float32)
            B = rng.standard_normal((K, N), dtype=np.float32)
            C0 = rng.standard_normal((M, N), dtype=np.float32)
            acc = call   # second call accumulates into C
            dA, dB = put(A), put(B)
            d_ref, d_na = put(C0), put(C0)
            L.ptc_sgemm(M, N, K, dA, K, 1, dB, N, 0, d_ref, N, acc, ws, MAX_MN, stream)
            rc = L.ptc_sgemm_noalloc(M, N, K, dA, K, 1, dB, N, 0, d_na, N, acc, stream)
            L.ptc_sync(c)
            assert rc == 0
            ref, got = get(d_ref), get(d_na)
            assert rel_err(got, ref) <= TOL, (call, rel_err(got, ref))
            want = A.astype(np.float64) @ B + (C0 if acc else 0.0)
            assert rel_err(got, want) <= TOL
    finally:
        L.ptc_destroy(c)


def counters(L):
    out = (C.c_longlong * 4)()
    L.ptc_gemm_counters(out)
    return list(out)   # tensor-core, SIMT, split-K reduction, cluster-reduced


def test_noalloc_split_k_partials_go_through_the_static_array(ptlib):
    """Products whose K-splits are summed by the reduction kernel, which
    reads the partials back from the static array: a 64x64 tile over
    K = 32000 (250 splits), then a smaller 32x32 product (so its partials
    sit at other offsets than the first call's), then a K that is not a
    multiple of 4 (the scalar-load kernel, 64 splits). Each call has fresh
    inputs, runs the reduction kernel exactly once and no cluster-summed
    split, and matches ptc_sgemm given a workspace of the same size."""
    L = ptlib
    c = L.ptc_create(0, 0)
    try:
        stream = L.ptc_stream(c)
        ws = L.ptc_alloc(c, MAX_MN * 4)
        shapes = [(64, 64, 32000), (32, 32, 32000), (64, 64, 32001)]
        for call, (M, N, K) in enumerate(shapes):
            rng = np.random.default_rng(200 + call)
            A = rng.standard_normal((M, K), dtype=np.float32)
            B = rng.standard_normal((K, N), dtype=np.float32)
            C0 = rng.standard_normal((M, N), dtype=np.float32)
            acc = call % 2

            def put(a):
                a = np.ascontiguousarray(a, np.float32)
                p = L.ptc_alloc(c, a.nbytes)
                L.ptc_h2d(c, p, a.ctypes.data, a.nbytes)
                return p

            def get(p):
                out = np.zeros((M, N), np.float32)
                L.ptc_d2h(c, out.ctypes.data, p, out.nbytes)
                return out

            dA, dB = put(A), put(B)
            d_ref, d_na = put(C0), put(C0)
            L.ptc_sgemm(M, N, K, dA, K, 1, dB, N, 0, d_ref, N, acc, ws, MAX_MN, stream)
            L.ptc_sync(c)
            before = counters(L)
            rc = L.ptc_sgemm_noalloc(M, N, K, dA, K, 1, dB, N, 0, d_na, N, acc, stream)
            L.ptc_sync(c)
            after = counters(L)
            assert rc == 0
            assert after[2] - before[2] == 1, (call, before, after)   # one reduction kernel
            assert after[3] == before[3] and after[0] == before[0], (call, before, after)
            ref, got = get(d_ref), get(d_na)
            assert rel_err(got, ref) <= TOL, (call, rel_err(got, ref))
            want = A.astype(np.float64) @ B + (C0 if acc else 0.0)
            assert rel_err(got, want) <= TOL, (call, rel_err(got, want))
    finally:
        L.ptc_destroy(c)


def test_noalloc_rejects_shapes_beyond_its_scratch(ptlib):
    # M*N above the static scratch is refused with -1 before any launch.
    rc = ptlib.ptc_sgemm_noalloc(2048, 1024, 64, None, 64, 1, None, 1024, 0, None, 1024, 0, None)
    assert rc == -1
