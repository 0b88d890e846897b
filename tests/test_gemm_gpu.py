"""GPU parity of ptc_sgemm, the fp32 GEMM behind pt_train_step's backward
pass (replacing sgemm_rect_tmu, pitorch/ops/gemm/gemm_rect.c:28-104).

As in the reference's dev/tests/gemm/test_gemm.c, square 16/32 products on
LCG integers 1..16 are exact in fp32 and must match bit for bit; the
training shapes (forward X.W^T, input grad dY.W, weight grad dY^T.X, and the
split-K classifier input gradient with K = 32000) are checked against a
float64 product at max|dC| / max|C| <= 1e-5.
"""
import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu


def lcg16(n, seed):
    out = np.empty(n, np.float32)
    s = seed
    for i in range(n):
        s = (s * 1103515245 + 12345) & 0xFFFFFFFF
        out[i] = float((s >> 16) & 0xF) + 1.0
    return out


class Dev:
    def __init__(self, L):
        self.L = L
        self.c = L.ptc_create(0, 0)

    def put(self, a):
        a = np.ascontiguousarray(a, np.float32)
        p = self.L.ptc_alloc(self.c, max(a.nbytes, 4))
        if a.nbytes:
            self.L.ptc_h2d(self.c, p, a.ctypes.data, a.nbytes)
        return p

    def get(self, p, shape):
        out = np.zeros(shape, np.float32)
        self.L.ptc_d2h(self.c, out.ctypes.data, p, out.nbytes)
        return out

    def close(self):
        self.L.ptc_destroy(self.c)


def run(L, dev, A, B, a_kc, b_kc, M, N, K, C0=None, accumulate=0, workspace=0):
    dA, dB = dev.put(A), dev.put(B)
    dC = dev.put(np.zeros((M, N), np.float32) if C0 is None else C0)
    ws = dev.put(np.zeros(workspace, np.float32)) if workspace else None
    lda = A.shape[1]
    ldb = B.shape[1]
    L.ptc_sgemm(M, N, K, dA, lda, a_kc, dB, ldb, b_kc, dC, N, accumulate, ws, workspace,
                L.ptc_stream(dev.c))
    L.ptc_sync(dev.c)
    return dev.get(dC, (M, N))


@pytest.mark.parametrize("dim", [16, 32])
def test_square_integer_exact(ptlib, dim):
    dev = Dev(ptlib)
    A = lcg16(dim * dim, 42).reshape(dim, dim)
    B = lcg16(dim * dim, 137).reshape(dim, dim)
    C = run(ptlib, dev, A, B, 1, 0, dim, dim, dim)   # A row-major [M,K], B row-major [K,N]
    assert np.array_equal(C, (A.astype(np.float64) @ B).astype(np.float32))
    dev.close()


# (M, N, K, a_kcontig, b_kcontig, workspace floats, accumulate)
CASES = [
    (256, 288, 288, 1, 1, 0, 0),        # forward q = x . Wq^T
    (256, 32000, 288, 1, 1, 0, 0),      # forward logits
    (255, 768, 288, 1, 0, 0, 0),        # input grad dX = dY . W
    (255, 288, 32000, 1, 0, 1 << 21, 0),  # classifier input grad, split-K
    (255, 288, 32000, 1, 0, 0, 0),      # same, no workspace: unsplit
    (32000, 288, 255, 0, 0, 0, 1),      # classifier weight grad, accumulate
    (768, 288, 255, 0, 0, 0, 1),        # w1 weight grad
    (37, 53, 4097, 1, 0, 1 << 20, 1),   # ragged, split-K + accumulate
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: "x".join(map(str, c[:3])) + f"_a{c[3]}b{c[4]}w{c[5]}acc{c[6]}")
def test_training_shapes(ptlib, case):
    M, N, K, akc, bkc, ws, acc = case
    rng = np.random.default_rng(M * 31 + N * 7 + K)
    A = rng.standard_normal((M, K) if akc else (K, M), dtype=np.float32)
    B = rng.standard_normal((N, K) if bkc else (K, N), dtype=np.float32)
    C0 = rng.standard_normal((M, N), dtype=np.float32) if acc else None
    dev = Dev(ptlib)
    got = run(ptlib, dev, A, B, akc, bkc, M, N, K, C0=C0, accumulate=acc, workspace=ws)
    dev.close()
    Am = A.astype(np.float64) if akc else A.astype(np.float64).T
    Bm = B.astype(np.float64).T if bkc else B.astype(np.float64)
    want = Am @ Bm + (C0.astype(np.float64) if acc else 0.0)
    assert rel_err(got, want) <= 1e-5
