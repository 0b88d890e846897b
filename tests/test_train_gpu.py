"""GPU parity of pt_train_step (forward with saved activations, the
7-operator backward as fp32 GEMMs, SGD) against the reference's host C.

Losses are checked per step at |dloss| / |loss| <= 1e-4, the tolerance of
the north star; gradients and updated weights at max|d| / max|ref| <= 1e-4
per tensor against the oracle (pinned bitwise to the reference build).
"""
import ctypes as C

import numpy as np
import pytest

import oracle
from conftest import golden, rel_err
from pitorch_b200 import api, synth

pytestmark = pytest.mark.gpu
TOL = 1e-4


def grads_of(ctx):
    ctx.L.pt_sync_grads(C.byref(ctx.ctx))
    n = ctx.ctx.grads._n_params
    return np.ctypeslib.as_array(ctx.ctx.grads._mem, shape=(n,)).copy()


def tensor_slices(cfg):
    dim, hidden, L, nh, nkv, V, seq = cfg
    kvd = nkv * (dim // nh)
    sizes = [("emb", V * dim), ("rms_att", L * dim), ("wq", L * dim * dim), ("wk", L * kvd * dim),
             ("wv", L * kvd * dim), ("wo", L * dim * dim), ("rms_ffn", L * dim),
             ("w1", L * hidden * dim), ("w2", L * dim * hidden), ("w3", L * hidden * dim),
             ("rms_final", dim)]
    off = 0
    for name, n in sizes:
        yield name, slice(off, off + n)
        off += n


def test_tiny_train_losses_grads_weights(ptlib):
    g = golden("train_tiny.npz")
    blob = synth.make_blob("tiny")
    T = int(g["T"])
    ctx = api.Context(blob, max_T=T)
    ref = oracle.Model(blob, max_T=T)
    for step in range(int(g["steps"])):
        loss = ctx.train_step(g["tokens"], float(g["lr"]))
        rl = ref.train_step(g["tokens"], float(g["lr"]))
        assert abs(loss - g["losses"][step]) <= TOL * abs(g["losses"][step]), (step, loss)
        assert abs(loss - rl) <= TOL * abs(rl)
        gg, rg = grads_of(ctx), ref.grads()
        for name, sl in tensor_slices(synth.CONFIGS["tiny"]):
            assert rel_err(gg[sl], rg[sl]) <= TOL, (step, name, rel_err(gg[sl], rg[sl]))
    w = np.frombuffer(ctx.blob()[28:], np.float32)
    rw = np.frombuffer(ref.blob()[28:], np.float32)
    assert rel_err(w, rw) <= TOL
    ctx.close()


def test_15M_train_20_steps_T256(ptlib):
    g = golden("train_stories15M.npz")
    T = int(g["T"])
    ctx = api.Context(synth.make_blob("stories15M"), max_T=T)
    losses = [ctx.train_step(g["tokens"], float(g["lr"])) for _ in range(int(g["steps"]))]
    ref = g["losses"].astype(np.float64)
    err = np.abs(np.array(losses) - ref) / np.abs(ref)
    assert err.max() <= TOL, err
    ctx.close()


def test_decode_after_training_uses_updated_weights(ptlib):
    blob = synth.make_blob("tiny")
    toks = synth.make_tokens(1024, 16)
    ctx = api.Context(blob, max_T=16)
    ref = oracle.Model(blob, max_T=16)
    for _ in range(3):
        ctx.train_step(toks, 1e-2)
        ref.train_step(toks, 1e-2)
    prompt = synth.make_prompt(1024)
    got = ctx.decode_greedy(prompt, 24)
    want = oracle.Model(ref.blob()).decode_greedy(prompt, 24)
    assert np.array_equal(got, want)
    ctx.close()


def test_staged_training_equals_train_step(ptlib):
    """pt_forward_train_embed / _layers_range / _head + staged backward + the
    split SGD (the pipeline rank path, pt_dist_pipeline.c:128-278) is the
    same computation as pt_train_step."""
    blob = synth.make_blob("tiny")
    toks = synth.make_tokens(1024, 16)
    a = api.Context(blob, max_T=16)
    b = api.Context(blob, max_T=16)
    L = a.L
    la = a.train_step(toks, 1e-3)
    c = b.ctx
    tp = api.ip(toks)
    Lyr = c.cfg.n_layers
    L.pt_zero_grads(C.byref(c.grads))
    L.pt_forward_train_embed(C.byref(c.w), C.byref(c.acts), tp, 16, c.cfg.dim)
    L.pt_forward_train_layers_range(C.byref(c.cfg), C.byref(c.w), C.byref(c.acts), 16, 0, 1, None, None)
    L.pt_forward_train_layers_range(C.byref(c.cfg), C.byref(c.w), C.byref(c.acts), 16, 1, Lyr, None, None)
    lb = L.pt_forward_train_head(C.byref(c.cfg), C.byref(c.w), C.byref(c.acts), tp, 16, None, None)
    L.pt_backward_head(C.byref(c.cfg), C.byref(c.w), C.byref(c.grads), C.byref(c.acts), C.byref(c.bb), tp, 16,
                       None, None)
    L.pt_backward_layers_range(C.byref(c.cfg), C.byref(c.w), C.byref(c.grads), C.byref(c.acts), C.byref(c.bb),
                               16, 1, Lyr, None, None)
    L.pt_backward_layers_range(C.byref(c.cfg), C.byref(c.w), C.byref(c.grads), C.byref(c.acts), C.byref(c.bb),
                               16, 0, 1, None, None)
    L.pt_backward_embed(C.byref(c.grads), C.byref(c.bb), tp, 16, c.cfg.dim)
    L.pt_sgd_update_head(C.byref(c.w), C.byref(c.grads), C.c_float(1e-3), C.byref(c.cfg))
    L.pt_sgd_update_layers(C.byref(c.w), C.byref(c.grads), C.c_float(1e-3), C.byref(c.cfg), 0, Lyr)
    assert la == lb
    assert np.array_equal(grads_of(a), grads_of(b))
    assert a.blob() == b.blob()
    a.close()
    b.close()
