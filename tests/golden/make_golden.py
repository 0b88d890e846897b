"""Regenerate the committed golden fixtures under tests/golden/.

Run in a checkout that has the reference sources next to it and
``oracle/_ref/libptref.so`` built (``make -C oracle``)::

    python tests/golden/make_golden.py [--ref-root PATH] [--skip-slow]

Sources of truth, all the reference's own:

* ``ops_refs.json``  -- the known answers of the reference's op tests,
  printed by its generator ``dev/tests/ops/gen_refs.py``, with the
  tolerances its ``dev/tests/ops/test_ops.c`` applies to each op.
* ``backward_refs.bin`` -- written by the reference's
  ``dev/tests/train/gen_backward_refs.py`` (torch autograd, seed 42); the
  tolerances are those of ``dev/tests/train/test_backward_ops.c``.
* ``matvec_kat.json`` and ``decode_*.npz`` / ``train_*.npz`` -- outputs of
  the reference's own host C (pitorch/pt.c host branch and below, compiled
  unchanged into oracle/_ref) on this repository's seeded synthetic inputs.

Nothing at test time reads the reference tree; only these files.
"""
import argparse
import hashlib
import json
import os
import re
import shutil
import subprocess
import sys
import tempfile
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

import oracle  # noqa: E402
from pitorch_b200 import synth  # noqa: E402

# Tolerance each reference op test uses (dev/tests/ops/test_ops.c).
OP_TOL = {"exp": 1e-4, "sin": 5e-4, "cos": 5e-4, "rms": 1e-4, "sm": 1e-4,
          "silu": 1e-4, "rope": 5e-3, "va": 1e-5, "vm": 1e-5, "emb": 1e-6,
          "mv": 1e-4}


def parse_c_arrays(text):
    out = {}
    for m in re.finditer(r"float (\w+)\[\]\s*=\s*\{([^}]*)\};", text):
        vals = [float(v.strip().rstrip("f")) for v in m.group(2).split(",") if v.strip()]
        out[m.group(1)] = vals
    for m in re.finditer(r"int (\w+)\s*=\s*(-?\d+);", text):
        out[m.group(1)] = int(m.group(2))
    return out


def make_ops(ref_root):
    script = os.path.join(ref_root, "dev", "tests", "ops", "gen_refs.py")
    text = subprocess.run([sys.executable, script], check=True, capture_output=True,
                          text=True).stdout
    arrays = parse_c_arrays(text)
    arrays["_tolerance"] = OP_TOL
    arrays["_rope"] = {"dim": 12, "head_dim": 6, "pos": 3}
    arrays["_source"] = "dev/tests/ops/gen_refs.py output; tolerances from dev/tests/ops/test_ops.c"
    with open(os.path.join(HERE, "ops_refs.json"), "w") as f:
        json.dump(arrays, f, indent=1)


def make_backward(ref_root):
    script = os.path.join(ref_root, "dev", "tests", "train", "gen_backward_refs.py")
    with tempfile.TemporaryDirectory() as td:
        subprocess.run([sys.executable, script], check=True, cwd=td, capture_output=True)
        shutil.copy(os.path.join(td, "backward_refs.bin"), os.path.join(HERE, "backward_refs.bin"))


def lcg_fill(n, seed):
    """Integer values 1..8 from the LCG of dev/tests/matvec/test_matvec.c:25-35."""
    out = np.empty(n, dtype=np.float32)
    s = seed & 0xFFFFFFFF
    for i in range(n):
        s = (s * 1103515245 + 12345) & 0xFFFFFFFF
        out[i] = float((s >> 16) & 0x7) + 1.0
    return out


def lcg_fill_fast(n, seed):
    # Same sequence as lcg_fill, computed in numpy blocks via the affine jump.
    out = np.empty(n, dtype=np.uint64)
    a, c, m = 1103515245, 12345, 1 << 32
    s = seed
    block = 4096
    # powers for a block: s_k = A_k s + C_k
    A = np.empty(block, dtype=np.uint64)
    C = np.empty(block, dtype=np.uint64)
    ak, ck = 1, 0
    for k in range(block):
        ak, ck = (a * ak) % m, (a * ck + c) % m
        A[k], C[k] = ak, ck
    for start in range(0, n, block):
        cnt = min(block, n - start)
        vals = (A[:cnt] * np.uint64(s) + C[:cnt]) % np.uint64(m)
        out[start:start + cnt] = vals
        s = int(vals[cnt - 1])
    return (((out >> np.uint64(16)) & np.uint64(7)).astype(np.float32) + 1.0)


def make_matvec_kat():
    shapes = [(48, 48), (288, 288), (768, 288), (288, 768), (32000, 288)]
    assert np.array_equal(lcg_fill(1000, 42), lcg_fill_fast(1000, 42))
    entries = []
    for rows, cols in shapes:
        W = lcg_fill_fast(rows * cols, 42).reshape(rows, cols)
        x = lcg_fill_fast(cols, 137)
        y = oracle.matvec(W, x, impl="reference")
        entries.append({"rows": rows, "cols": cols, "w_seed": 42, "x_seed": 137,
                        "y_sha256": hashlib.sha256(y.tobytes()).hexdigest(),
                        "y_head": [float(v) for v in y[:8]], "y_sum": float(y.astype(np.float64).sum())})
    with open(os.path.join(HERE, "matvec_kat.json"), "w") as f:
        json.dump({"source": "smatvec_cpu of the reference host build; inputs from the LCG of "
                             "dev/tests/matvec/test_matvec.c:25-35 (values 1..8, exact in fp32)",
                   "cases": entries}, f, indent=1)


def make_decode(name, n_pos, keep_rows, suffix=""):
    cfg = synth.CONFIGS[name]
    blob = synth.make_blob(cfg)
    prompt = synth.make_prompt(cfg[5])
    m = oracle.Model(blob, impl="reference")
    t0 = time.time()
    toks, logits = m.decode_greedy(prompt, n_pos, want_logits=True)
    dt = time.time() - t0
    srt = np.sort(logits, axis=1)
    np.savez_compressed(
        os.path.join(HERE, f"decode_{name}{suffix}.npz"),
        prompt=prompt, tokens=toks, n_pos=np.int32(n_pos), seed=np.int32(synth.DEFAULT_SEED),
        logit_absmax=np.abs(logits).max(axis=1), logit_sum=logits.astype(np.float64).sum(axis=1),
        top2_gap=srt[:, -1] - srt[:, -2], rows=np.array(keep_rows, dtype=np.int32),
        logits_rows=logits[keep_rows])
    print(f"decode {name}: {n_pos} positions in {dt:.1f}s ({n_pos / dt:.1f} tok/s, reference host C)")


def make_train(name, T, steps, lr=1e-3):
    cfg = synth.CONFIGS[name]
    blob = synth.make_blob(cfg)
    tokens = synth.make_tokens(cfg[5], T)
    m = oracle.Model(blob, max_T=T, impl="reference")
    losses = []
    t0 = time.time()
    for _ in range(steps):
        losses.append(m.train_step(tokens, lr))
    dt = time.time() - t0
    g = m.grads()
    np.savez_compressed(os.path.join(HERE, f"train_{name}.npz"), tokens=tokens,
                        losses=np.array(losses, dtype=np.float32), lr=np.float32(lr),
                        T=np.int32(T), steps=np.int32(steps),
                        final_blob_sha256=np.bytes_(hashlib.sha256(m.blob()).hexdigest()),
                        grad_absmax=np.float32(np.abs(g).max()),
                        grad_sum=np.float64(g.astype(np.float64).sum()))
    print(f"train {name}: T={T} {steps} steps in {dt:.1f}s ({dt / steps:.2f} s/step); losses {losses[0]:.6f}..{losses[-1]:.6f}")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref-root", default=os.path.join(REPO, "..", "reference"))
    ap.add_argument("--skip-slow", action="store_true")
    ap.add_argument("--only-110M-long", action="store_true",
                    help="regenerate decode_stories110M_long.npz alone (about 100 s)")
    args = ap.parse_args()
    if not oracle.ref_available():
        sys.exit("oracle/_ref/libptref.so missing: run make -C oracle first")
    if args.only_110M_long:
        make_decode("stories110M", 1024, [255, 511, 767, 1023], suffix="_long")
        return
    make_ops(args.ref_root)
    make_backward(args.ref_root)
    make_matvec_kat()
    make_decode("tiny", 64, [0, 1, 7, 8, 31, 63])
    make_train("tiny", 16, 5)
    make_decode("stories15M", 256, [0, 255])
    if not args.skip_slow:
        make_decode("stories42M", 64, [63])
        make_decode("stories110M", 64, [63])
        # the whole 1024-position cache: attention over more than 512 positions
        make_decode("stories42M", 1024, [511, 700, 1023], suffix="_long")
        # the benchmark's configuration: 110M over the whole 1024-position cache
        make_decode("stories110M", 1024, [255, 511, 767, 1023], suffix="_long")
        make_train("stories15M", 256, 20)


if __name__ == "__main__":
    main()
