"""GPU parity of the tensor-core fp32 GEMM (ptc_gemm_tc.cu: CUTLASS's sm100
FastFP32 collective, bf16-split operands on tcgen05.mma) that runs the
classifier's training products (PTC_GEMM_TC=0 turns it off).

The switch is read once per process, so the checks run in a child process
with it set to 1: the three classifier products at the 15M training shapes
(forward X.W^T, input gradient dY.W split over K = 32000, weight gradient
dY^T.X accumulated) against a float64 product at max|dC| / max|C| <= 1e-5,
each shown by the launch counters (ptc_gemm_counters) to have run one
tensor-core kernel, and three pt_train_step losses against the reference's
at 1e-4. With PTC_GEMM_TC=1 a product the tensor-core kernel refuses is a
fatal error, so these cannot pass on the SIMT fallback.
"""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = r"""
import numpy as np, sys
sys.path.insert(0, "tests")
import pitorch_b200
from pitorch_b200 import api, synth
from conftest import golden, rel_err
from test_gemm_gpu import Dev, run
L = pitorch_b200.lib()
import ctypes
dev = Dev(L)
def tc_launches():
    out = (ctypes.c_longlong * 4)()
    L.ptc_gemm_counters(out)
    return out[0]
rng = np.random.default_rng(5)
V, D, T = 32000, 288, 256
W = rng.normal(0, 0.02, (V, D)).astype(np.float32)
X = rng.normal(0, 1, (T, D)).astype(np.float32)
n0 = tc_launches()
C = run(L, dev, X, W, 1, 1, T, V, D)
n1 = tc_launches()
e1 = rel_err(C, X.astype(np.float64) @ W.T.astype(np.float64))
dY = rng.normal(0, 1e-3, (T - 1, V)).astype(np.float32)
C = run(L, dev, dY, W, 1, 0, T - 1, D, V, workspace=8 * (T - 1) * D)
n2 = tc_launches()
e2 = rel_err(C, dY.astype(np.float64) @ W.astype(np.float64))
C0 = rng.normal(0, 1, (V, D)).astype(np.float32)
C = run(L, dev, dY, X[: T - 1], 0, 0, V, D, T - 1, C0=C0, accumulate=1)
n3 = tc_launches()
e3 = rel_err(C, C0.astype(np.float64) + dY.T.astype(np.float64) @ X[: T - 1].astype(np.float64))
dev.close()
print("TC", n1 - n0, n2 - n1, n3 - n2)
g = golden("train_stories15M.npz")
ctx = api.Context(synth.make_blob("stories15M"), max_T=int(g["T"]))
losses = [ctx.train_step(g["tokens"], float(g["lr"])) for _ in range(3)]
ref = g["losses"][:3].astype(np.float64)
e4 = float(np.max(np.abs(np.array(losses) - ref) / np.abs(ref)))
ctx.close()
print("ERRS", e1, e2, e3, e4)
"""


def test_tensor_core_gemm_classifier_products():
    env = dict(os.environ, PTC_GEMM_TC="1")
    r = subprocess.run([sys.executable, "-c", CHILD], cwd=ROOT, env=env, capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    # each product ran on the tensor cores: one CUTLASS launch each (the
    # input gradient as one batched launch over its K-slices)
    tc = [ln for ln in r.stdout.splitlines() if ln.startswith("TC")][-1]
    assert [int(v) for v in tc.split()[1:]] == [1, 1, 1], tc
    line = [ln for ln in r.stdout.splitlines() if ln.startswith("ERRS")][-1]
    e1, e2, e3, e4 = (float(v) for v in line.split()[1:])
    assert e1 <= 1e-5 and e2 <= 1e-5 and e3 <= 1e-5, (e1, e2, e3)
    assert e4 <= 1e-4, e4
