"""Pins for the CPU oracle (CPU only).

The oracle (oracle/pt_oracle.c) is the checker for every GPU parity test, so
it is pinned first: against the known answers of the reference's own op
tests (dev/tests/ops/test_ops.c with dev/tests/ops/gen_refs.py's values),
against the reference's backward-op fixtures (gen_backward_refs.py), and
bit-for-bit against outputs of the reference's host C build on synthetic
models (tests/golden/*.npz, written by tests/golden/make_golden.py).
"""
import ctypes as C
import hashlib
import json
import os
import struct

import numpy as np
import pytest

import oracle
from conftest import GOLDEN, golden
from pitorch_b200 import synth

L = oracle.lib()


def fp(a):
    return a.ctypes.data_as(C.POINTER(C.c_float))


def approx_ok(got, ref, tol):
    # dev/tests/ops/test_ops.c:21-28: |d| < atol, or |d|/|ref| < rtol.
    got, ref = np.float32(got), np.float32(ref)
    d = abs(float(got) - float(ref))
    s = abs(float(ref))
    return d < tol if s < 1e-6 else (d < tol or d / s < tol)


@pytest.fixture(scope="module")
def ops():
    with open(os.path.join(GOLDEN, "ops_refs.json")) as f:
        return json.load(f)


def test_math_known_answers(ops):
    tol = ops["_tolerance"]
    for name, fn in (("exp", L.or_expf), ("sin", L.or_sinf), ("cos", L.or_cosf)):
        for x, r in zip(ops[f"{name}_in"], ops[f"{name}_ref"]):
            assert approx_ok(fn(x), r, tol[name]), (name, x, fn(x), r)


def test_elementwise_known_answers(ops):
    tol = ops["_tolerance"]
    x = np.array(ops["rms_x"], np.float32)
    w = np.array(ops["rms_w"], np.float32)
    o = np.zeros_like(x)
    L.or_rmsnorm(fp(o), fp(x), fp(w), len(x))
    assert all(approx_ok(a, b, tol["rms"]) for a, b in zip(o, ops["rms_ref"]))
    s = np.array(ops["sm_x"], np.float32)
    L.or_softmax(fp(s), len(s))
    assert all(approx_ok(a, b, tol["sm"]) for a, b in zip(s, ops["sm_ref"]))
    s = np.array(ops["silu_x"], np.float32)
    L.or_silu(fp(s), len(s))
    assert all(approx_ok(a, b, tol["silu"]) for a, b in zip(s, ops["silu_ref"]))
    q = np.array(ops["rope_q"], np.float32)
    k = np.array(ops["rope_k"], np.float32)
    r = ops["_rope"]
    L.or_rope(fp(q), fp(k), r["dim"], r["head_dim"], r["pos"])
    assert all(approx_ok(a, b, tol["rope"]) for a, b in zip(q, ops["rope_q_ref"]))
    assert all(approx_ok(a, b, tol["rope"]) for a, b in zip(k, ops["rope_k_ref"]))
    W = np.array(ops["mv_W"], np.float32).reshape(4, 6)
    y = oracle.matvec(W, np.array(ops["mv_x"], np.float32))
    assert all(approx_ok(a, b, tol["mv"]) for a, b in zip(y, ops["mv_ref"]))
    assert L.or_argmax(fp(np.array(ops["am_x"], np.float32)), 6) == ops["am_ref"]


def _read_backward_refs():
    # Layout written by dev/tests/train/gen_backward_refs.py.
    data = open(os.path.join(GOLDEN, "backward_refs.bin"), "rb").read()
    off = 0

    def floats():
        nonlocal off
        n = struct.unpack_from("i", data, off)[0]
        off += 4
        a = np.frombuffer(data, np.float32, n, off).copy()
        off += 4 * n
        return a

    def integer():
        nonlocal off
        v = struct.unpack_from("i", data, off)[0]
        off += 4
        return v

    r = {}
    r["rms"] = [floats() for _ in range(5)]
    r["mm"] = [floats() for _ in range(5)]
    r["rope_pos"] = integer()
    r["rope"] = [floats() for _ in range(4)]
    r["sm"] = [floats() for _ in range(3)]
    r["silu"] = [floats() for _ in range(3)]
    n = integer()
    r["emb_tokens"] = [integer() for _ in range(n)]
    r["emb_d"] = [floats() for _ in range(n)]
    r["emb_ref"] = floats()
    return r


def test_backward_primitives_against_reference_fixture():
    # Tolerances of dev/tests/train/test_backward_ops.c:82-177.
    r = _read_backward_refs()
    DIM, HDIM, HD = 16, 32, 4
    x, w, d_o, dx_ref, dw_ref = r["rms"]
    dx = np.zeros(DIM, np.float32)
    dw = np.zeros(DIM, np.float32)
    L.or_rmsnorm_backward(fp(dx), fp(dw), fp(d_o), fp(x), fp(w), DIM)
    assert np.abs(dx - dx_ref).max() < 1e-4 and np.abs(dw - dw_ref).max() < 1e-4
    W, xm, dy, dxm_ref, dW_ref = r["mm"]
    W = W.reshape(HDIM, DIM)
    assert np.abs(oracle.matvec(np.ascontiguousarray(W.T), dy) - dxm_ref).max() < 1e-4
    assert np.abs(np.outer(dy, xm).ravel() - dW_ref).max() < 1e-4
    dqo, dko, dq_ref, dk_ref = r["rope"]
    dq = np.zeros(DIM, np.float32)
    dk = np.zeros(DIM, np.float32)
    L.or_rope_backward(fp(dq), fp(dk), fp(dqo), fp(dko), DIM, HD, r["rope_pos"])
    assert np.abs(dq - dq_ref).max() < 5e-3 and np.abs(dk - dk_ref).max() < 5e-3
    y, dys, dxs_ref = r["sm"]
    dxs = np.zeros(DIM, np.float32)
    L.or_softmax_backward(fp(dxs), fp(dys), fp(y), DIM)
    assert np.abs(dxs - dxs_ref).max() < 1e-5


def _lcg(n, seed):
    out = np.empty(n, dtype=np.uint64)
    a, c, m = 1103515245, 12345, 1 << 32
    s = seed
    A = np.empty(4096, np.uint64)
    Cc = np.empty(4096, np.uint64)
    ak, ck = 1, 0
    for k in range(4096):
        ak, ck = (a * ak) % m, (a * ck + c) % m
        A[k], Cc[k] = ak, ck
    for st in range(0, n, 4096):
        cnt = min(4096, n - st)
        v = (A[:cnt] * np.uint64(s) + Cc[:cnt]) % np.uint64(m)
        out[st:st + cnt] = v
        s = int(v[cnt - 1])
    return (((out >> np.uint64(16)) & np.uint64(7)).astype(np.float32) + 1.0)


def matvec_kat_cases():
    with open(os.path.join(GOLDEN, "matvec_kat.json")) as f:
        return json.load(f)["cases"]


@pytest.mark.parametrize("case", matvec_kat_cases(), ids=lambda c: f"{c['rows']}x{c['cols']}")
def test_oracle_matvec_known_answers(case):
    W = _lcg(case["rows"] * case["cols"], case["w_seed"]).reshape(case["rows"], case["cols"])
    x = _lcg(case["cols"], case["x_seed"])
    y = oracle.matvec(W, x)
    assert hashlib.sha256(y.tobytes()).hexdigest() == case["y_sha256"]


def test_oracle_tiny_decode_bitwise():
    g = golden("decode_tiny.npz")
    m = oracle.Model(synth.make_blob("tiny"))
    toks, logits = m.decode_greedy(g["prompt"], int(g["n_pos"]), want_logits=True)
    assert np.array_equal(toks, g["tokens"])
    assert np.array_equal(logits[g["rows"]].view(np.int32), g["logits_rows"].view(np.int32))


def test_oracle_tiny_train_bitwise():
    g = golden("train_tiny.npz")
    m = oracle.Model(synth.make_blob("tiny"), max_T=int(g["T"]))
    losses = [m.train_step(g["tokens"], float(g["lr"])) for _ in range(int(g["steps"]))]
    assert np.array_equal(np.array(losses, np.float32).view(np.int32), g["losses"].view(np.int32))
    assert hashlib.sha256(m.blob()).hexdigest() == g["final_blob_sha256"].item().decode()


def test_oracle_15M_decode_bitwise():
    g = golden("decode_stories15M.npz")
    m = oracle.Model(synth.make_blob("stories15M"))
    toks, logits = m.decode_greedy(g["prompt"], int(g["n_pos"]), want_logits=True)
    assert np.array_equal(toks, g["tokens"])
    assert np.array_equal(logits[g["rows"]].view(np.int32), g["logits_rows"].view(np.int32))


@pytest.mark.slow
def test_oracle_15M_train_first_step_bitwise():
    path = os.path.join(GOLDEN, "train_stories15M.npz")
    if not os.path.exists(path):
        pytest.skip("15M training fixture not generated")
    g = np.load(path)
    m = oracle.Model(synth.make_blob("stories15M"), max_T=int(g["T"]))
    loss = m.train_step(g["tokens"], float(g["lr"]))
    assert np.float32(loss).view(np.int32) == g["losses"][:1].view(np.int32)[0]


@pytest.mark.skipif(not oracle.ref_available(), reason="reference host build not present")
def test_oracle_equals_reference_build_on_tiny():
    blob = synth.make_blob("tiny")
    prompt = synth.make_prompt(1024)
    a, b = oracle.Model(blob), oracle.Model(blob, impl="reference")
    ta, la = a.decode_greedy(prompt, 64, True)
    tb, lb = b.decode_greedy(prompt, 64, True)
    assert np.array_equal(ta, tb) and np.array_equal(la.view(np.int32), lb.view(np.int32))
    toks = synth.make_tokens(1024, 16)
    a, b = oracle.Model(blob, 16), oracle.Model(blob, 16, impl="reference")
    for _ in range(3):
        assert a.train_step(toks, 1e-3) == b.train_step(toks, 1e-3)
    assert np.array_equal(a.grads().view(np.int32), b.grads().view(np.int32))
    assert a.blob() == b.blob()


def test_oracle_staged_equals_monolithic():
    # dev/host/test_stage_forward.c:49-80 -- staged forward is bitwise the
    # monolithic one; the pipeline relies on this.
    blob = synth.make_blob("tiny")
    a, b = oracle.Model(blob), oracle.Model(blob)
    tok = 5
    for pos in range(6):
        a.forward_embed(tok)
        a.forward_layers_range(pos, 0, 1)
        a.forward_layers_range(pos, 1, 2)
        a.forward_head()
        la = a.logits()
        b.forward_embed(tok)
        b.forward_layers_range(pos, 0, 2)
        b.forward_head()
        assert np.array_equal(la.view(np.int32), b.logits().view(np.int32))
        tok = int(np.argmax(la))
