"""GPU parity of pt_train_step (forward with saved activations, the
7-operator backward as fp32 GEMMs, SGD) against the reference's host C.

Losses are checked per step at |dloss| / |loss| <= 1e-4, the tolerance of
the north star; gradients and updated weights at max|d| / max|ref| <= 1e-4
per tensor against the oracle (pinned bitwise to the reference build).
"""
import ctypes as C
import os

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


def test_train_beyond_256_positions(ptlib):
    """T > 256 takes the per-row attention kernels (the row-block ones cover
    T <= 256): a narrow model with seq_len 320 trained at T = 300."""
    cfg = (64, 176, 2, 4, 4, 1024, 320)
    blob = synth.make_blob(cfg)
    T = 300
    toks = synth.make_tokens(1024, T, seed=7)
    ctx = api.Context(blob, max_T=T)
    ref = oracle.Model(blob, max_T=T)
    for step in range(2):
        loss = ctx.train_step(toks, 1e-3)
        rl = ref.train_step(toks, 1e-3)
        assert abs(loss - rl) <= TOL * abs(rl), (step, loss, rl)
        gg, rg = grads_of(ctx), ref.grads()
        for name, sl in tensor_slices(cfg):
            assert rel_err(gg[sl], rg[sl]) <= TOL, (step, name, rel_err(gg[sl], rg[sl]))
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


def accumulate_step(ctx, token_mbs, lr):
    """One accumulated step on one GPU: zero, forward + backward of every
    microbatch (pt_backward adds into the gradients), then SGD with lr times
    the mean gradient. Returns the mean loss."""
    L, c = ctx.L, ctx.ctx
    L.pt_zero_grads(C.byref(c.grads))
    total = 0.0
    for toks in token_mbs:
        tp = api.ip(toks)
        T = len(toks)
        total += L.pt_forward_train(C.byref(c.cfg), C.byref(c.w), C.byref(c.acts), tp, T, None, None)
        L.pt_backward(C.byref(c.cfg), C.byref(c.w), C.byref(c.grads), C.byref(c.acts), C.byref(c.bb), tp, T,
                      None, None)
    L.pt_sgd_update(C.byref(c.w), C.byref(c.grads), C.c_float(lr / len(token_mbs)), C.byref(c.cfg))
    return total / len(token_mbs)


def test_checkpoint_round_trip(ptlib, tmp_path):
    """pt_save_weights after training writes a .bin that loads into a new
    context with the trained weights (same logits as the trained context)."""
    blob = synth.make_blob("tiny")
    toks = synth.make_tokens(1024, 16)
    a = api.Context(blob, max_T=16)
    for _ in range(3):
        a.train_step(toks, 1e-2)
    path = str(tmp_path / "tiny_trained.bin")
    assert ptlib.pt_save_weights(C.byref(a.ctx), path.encode()) == 0
    saved = open(path, "rb").read()
    assert saved == a.blob()
    assert saved != blob
    b = api.Context(saved)
    for p, t in enumerate([1, 5, 9, 13]):
        a.L.pt_forward_step(C.byref(a.ctx), t)
        la = np.ctypeslib.as_array(a.ctx.state.logits, shape=(1024,)).copy()
        b.L.pt_forward_step(C.byref(b.ctx), t)
        lb = np.ctypeslib.as_array(b.ctx.state.logits, shape=(1024,)).copy()
        assert rel_err(lb, la) <= 1e-5, p
    a.close()
    b.close()


def test_microbatch_sets_match_accumulation(ptlib):
    """The trainer's microbatch activation sets (ptc_trainer_set_microbatches
    / ptc_trainer_select), driven in the GPipe order on one GPU -- every
    forward, then every backward in reverse -- equal plain gradient
    accumulation (accumulate_step): mean losses of 3 steps within 1e-4."""
    L = ptlib
    cfg = synth.CONFIGS["stories15M"]
    T, n_mb, lr = 64, 4, 1e-2
    mbs = [synth.make_tokens(cfg[5], T, seed=100 + m) for m in range(n_mb)]
    ref_ctx = api.Context(synth.make_blob(cfg), max_T=T)
    ref = np.array([accumulate_step(ref_ctx, mbs, lr) for _ in range(3)], dtype=np.float64)
    ref_ctx.close()
    ctx = api.Context(synth.make_blob(cfg), max_T=T)
    tr = L.pt_ptc_trainer(C.byref(ctx.ctx))
    nl = cfg[2]
    L.ptc_trainer_set_microbatches(tr, n_mb)
    for m in range(n_mb):
        L.ptc_trainer_select(tr, m)
        L.ptc_trainer_set_tokens(tr, api.ip(mbs[m]), T)
    got = []
    for _ in range(3):
        L.ptc_trainer_zero_grads(tr)
        total = 0.0
        for m in range(n_mb):
            L.ptc_trainer_select(tr, m)
            L.ptc_trainer_fwd_embed(tr)
            L.ptc_trainer_fwd_layers(tr, 0, nl)
            total += L.ptc_trainer_fwd_head(tr)
        for m in reversed(range(n_mb)):
            L.ptc_trainer_select(tr, m)
            L.ptc_trainer_bwd_head(tr)
            L.ptc_trainer_bwd_layers(tr, 0, nl)
            L.ptc_trainer_bwd_embed(tr)
        L.ptc_trainer_sgd_head(tr, C.c_float(lr / n_mb))
        L.ptc_trainer_sgd_layers(tr, C.c_float(lr / n_mb), 0, nl)
        L.ptc_trainer_sync(tr)
        got.append(total / n_mb)
    L.ptc_trainer_select(tr, 0)
    ctx.close()
    got = np.array(got)
    assert np.all(np.abs(got - ref) <= 1e-4 * np.abs(ref)), (got, ref)
    assert ref[2] < ref[0]


def test_microbatch_set_without_length_is_refused(ptlib):
    """A microbatch set that has neither tokens nor a length has T = 0; a
    pass on it is refused on the host with a message (its kernels would
    index row T - 1 = -1). Checked in a child process, which aborts before
    any kernel of the pass is launched."""
    import subprocess
    import sys
    code = (
        "import ctypes as C, pitorch_b200\n"
        "from pitorch_b200 import api, synth\n"
        "L = pitorch_b200.lib()\n"
        "ctx = api.Context(synth.make_blob('tiny'), max_T=16)\n"
        "tr = L.pt_ptc_trainer(C.byref(ctx.ctx))\n"
        "L.ptc_trainer_set_microbatches(tr, 2)\n"
        "L.ptc_trainer_select(tr, 1)\n"
        "L.ptc_trainer_fwd_layers(tr, 0, 1)\n"
        "L.ptc_trainer_sync(tr)\n"
        "print('NOT REFUSED')\n")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "-c", code], cwd=root, capture_output=True, text=True, timeout=300)
    assert r.returncode != 0 and "NOT REFUSED" not in r.stdout, (r.returncode, r.stdout[-500:])
    assert "set the tokens or the length first" in r.stderr, r.stderr[-1000:]
