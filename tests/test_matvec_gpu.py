"""GPU parity of the fp32 matvec (the hot path's core) against the oracle.

Mirrors the reference's dev/tests/matvec/test_matvec.c: the same shapes and
LCG integer inputs (exact in fp32, so the GPU must match bit for bit), then
the BASELINE sweep shapes with N(0,0.02) weights and N(0,1) inputs, checked
at max|dy| / max|y_ref| <= 1e-5, plus shapes the vector path cannot take.
All calls go through the C ABI (ptc_matvec_host = the pt_matvec_fn path,
ptc_matvec = device pointers).
"""
import ctypes as C
import hashlib

import numpy as np
import pytest

import oracle
from conftest import rel_err
from test_oracle_pins import _lcg, matvec_kat_cases
from pitorch_b200.api import fp

pytestmark = pytest.mark.gpu

SWEEP = [(288, 288), (768, 288), (288, 768), (512, 512), (1376, 512), (2048, 768),
         (768, 2048), (32000, 288), (32000, 768)]
TOL = 1e-5


def gpu_matvec(L, W, x):
    y = np.zeros(W.shape[0], np.float32)
    L.ptc_matvec_host(fp(W), fp(x), fp(y), W.shape[0], W.shape[1])
    return y


@pytest.mark.parametrize("case", matvec_kat_cases(), ids=lambda c: f"{c['rows']}x{c['cols']}")
def test_matvec_known_answers_bitexact(ptlib, case):
    W = _lcg(case["rows"] * case["cols"], case["w_seed"]).reshape(case["rows"], case["cols"])
    x = _lcg(case["cols"], case["x_seed"])
    y = gpu_matvec(ptlib, W, x)
    assert hashlib.sha256(y.tobytes()).hexdigest() == case["y_sha256"]


@pytest.mark.parametrize("shape", SWEEP, ids=lambda s: f"{s[0]}x{s[1]}")
def test_matvec_sweep_vs_oracle(ptlib, shape):
    rng = np.random.default_rng(shape[0] * 7 + shape[1])
    W = (rng.standard_normal(shape, dtype=np.float32) * np.float32(0.02))
    x = rng.standard_normal(shape[1], dtype=np.float32)
    y = gpu_matvec(ptlib, W, x)
    assert rel_err(y, oracle.matvec(W, x)) <= TOL


@pytest.mark.parametrize("shape", [(1, 1), (3, 5), (17, 33), (16, 4097), (5, 9000), (1000, 2)],
                         ids=lambda s: f"{s[0]}x{s[1]}")
def test_matvec_ragged_shapes(ptlib, shape):
    rng = np.random.default_rng(11)
    W = rng.standard_normal(shape, dtype=np.float32)
    x = rng.standard_normal(shape[1], dtype=np.float32)
    assert rel_err(gpu_matvec(ptlib, W, x), oracle.matvec(W, x)) <= TOL


def test_matvec_zero_rows_is_noop(ptlib):
    y = np.full(4, 7.0, np.float32)
    W = np.zeros((0, 8), np.float32)
    x = np.ones(8, np.float32)
    ptlib.ptc_matvec_host(fp(W), fp(x), fp(y), 0, 8)
    assert (y == 7.0).all()


def test_matvec_device_pointers(ptlib):
    rng = np.random.default_rng(5)
    W = rng.standard_normal((2048, 768), dtype=np.float32)
    x = rng.standard_normal(768, dtype=np.float32)
    ctx = ptlib.ptc_create(0, 0)
    try:
        dW = ptlib.ptc_alloc(ctx, W.nbytes)
        dx = ptlib.ptc_alloc(ctx, x.nbytes)
        dy = ptlib.ptc_alloc(ctx, 2048 * 4)
        ptlib.ptc_h2d(ctx, dW, W.ctypes.data, W.nbytes)
        ptlib.ptc_h2d(ctx, dx, x.ctypes.data, x.nbytes)
        ptlib.ptc_matvec(dW, dx, dy, 2048, 768, ptlib.ptc_stream(ctx))
        y = np.zeros(2048, np.float32)
        ptlib.ptc_d2h(ctx, y.ctypes.data, dy, y.nbytes)
    finally:
        ptlib.ptc_destroy(ctx)
    assert rel_err(y, oracle.matvec(W, x)) <= TOL
