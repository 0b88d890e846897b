"""Text layer (tokenizer, sampler, pt_generate) against the reference's own
text code (pitorch/text/pt_text.c, built into oracle/_ref) on a seeded
synthetic tokenizer.bin; plus pt_generate on the GPU."""
import ctypes as C
import os
import sys
import tempfile

import numpy as np
import pytest

import oracle
from pitorch_b200 import api, synth
from tokenizer_synth import make_tokenizer

Tok, Sampler = api.pt_tokenizer_t, api.pt_sampler_t
bind = api.declare_text


@pytest.fixture(scope="module")
def libs():
    import pitorch_b200
    ours = bind(pitorch_b200.lib())
    if not oracle.ref_available():
        pytest.skip("reference host build not present")
    return ours, bind(oracle.ref_lib())


def encode(L, tok, text):
    out = (C.c_int * (len(text.encode()) + 8))()
    n = C.c_int(0)
    L.pt_encode(C.byref(tok), text.encode(), 1, 0, out, C.byref(n))
    return list(out[:n.value])


TEXTS = ["Once upon a time", "the rain in spain", "Hello, world!", "", "zz", "héllo ünïcode ✓",
         "a" * 40, "teat oin shrdlu eta"]


def test_tokenizer_matches_reference(libs):
    ours, ref = libs
    data, pieces = make_tokenizer()
    buf = C.create_string_buffer(data, len(data))
    ta, tb = Tok(), Tok()
    ours.pt_tokenizer_init(C.byref(ta), C.cast(buf, C.c_void_p), 1024)
    ref.pt_tokenizer_init(C.byref(tb), C.cast(buf, C.c_void_p), 1024)
    for t in TEXTS:
        ea, eb = encode(ours, ta, t), encode(ref, tb, t)
        assert ea == eb, t
    for prev in (1, 5):
        for tk in list(range(0, 1024, 37)) + [3, 13, 258, 259]:
            assert ours.pt_decode(C.byref(ta), prev, tk) == ref.pt_decode(C.byref(tb), prev, tk), (prev, tk)
    ours.pt_tokenizer_free(C.byref(ta))


@pytest.mark.parametrize("temp,topp", [(0.0, 0.9), (1.0, 0.9), (0.7, 0.5), (1.3, 1.0)])
def test_sampler_matches_reference(libs, temp, topp):
    ours, ref = libs
    rng = np.random.default_rng(3)
    sa, sb = Sampler(), Sampler()
    ours.pt_sampler_init(C.byref(sa), 1024, temp, topp, 1234)
    ref.pt_sampler_init(C.byref(sb), 1024, temp, topp, 1234)
    for _ in range(50):
        lg = (rng.standard_normal(1024) * 3).astype(np.float32)
        la, lb = lg.copy(), lg.copy()
        assert ours.pt_sample(C.byref(sa), api.fp(la)) == ref.pt_sample(C.byref(sb), api.fp(lb))
        assert sa.rng_state == sb.rng_state


@pytest.mark.gpu
def test_generate_greedy_text_matches_oracle(ptlib):
    """pt_generate at temperature 0 prints the pieces of the reference's greedy
    stream (oracle decode + the tokenizer checked above)."""
    L = bind(ptlib)
    data, _ = make_tokenizer()
    tbuf = C.create_string_buffer(data, len(data))
    tok = Tok()
    L.pt_tokenizer_init(C.byref(tok), C.cast(tbuf, C.c_void_p), 1024)
    blob = synth.make_blob("tiny")
    ctx = api.Context(blob)
    sampler = Sampler()
    L.pt_sampler_init(C.byref(sampler), 1024, 0.0, 0.9, 42)
    prompt = "the rain in spain"
    ids = encode(L, tok, prompt)
    # expected: teacher-forced prompt then greedy, stopping at BOS/EOS
    m = oracle.Model(blob)
    stream = m.decode_greedy(np.array(ids, np.int32), 48)
    want, prev = [], ids[-1]
    for p in range(len(ids) - 1, 48):
        nxt = int(stream[p])
        if nxt in (1, 2):
            break
        want.append(L.pt_decode(C.byref(tok), prev, nxt))
        prev = nxt
    sys.stdout.flush()
    with tempfile.TemporaryFile() as f:
        saved = os.dup(1)
        os.dup2(f.fileno(), 1)
        try:
            L.pt_generate(C.byref(ctx.ctx.cfg), C.byref(ctx.ctx.w), C.byref(ctx.ctx.state), C.byref(tok),
                          C.byref(sampler), prompt.encode(), 48, None)
        finally:
            os.dup2(saved, 1)
            os.close(saved)
        f.seek(0)
        out = f.read()
    text = out.split(b"\n[")[0]
    assert text == b"".join(want)
    L.pt_tokenizer_free(C.byref(tok))
    ctx.close()
