"""The low-level training API on structs the CALLER allocates: a C program
(tests/c/stage_train_dropin.c) compiled with gcc against include/ and linked
to libpitorch_b200.so makes the reference's call sequence for caller-owned
pt_activations_t / pt_grads_t / pt_backward_buf_t (pitorch/train/pt_train.h;
dev/host/test_stage_train.c drives the same calls): the whole-model passes,
the staged passes split at a layer, and a two-stage pipeline whose stages
hand residual rows and d_res over through their host arrays.

Checks: staged and pipeline losses equal the whole-model ones bit for bit
and the staged run leaves the same weight image byte for byte (all checked
inside the program), and the losses match the reference's own host C
(tests/golden/train_tiny.npz) within 1e-4.
"""
import os
import subprocess

import numpy as np
import pytest

import pitorch_b200
from conftest import golden
from pitorch_b200 import synth

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SRC = os.path.join(ROOT, "tests", "c", "stage_train_dropin.c")


def build(tmp_path):
    exe = tmp_path / "stage_train_dropin"
    lib_dir = os.path.dirname(pitorch_b200.LIB_PATH)
    subprocess.run(["gcc", "-O2", "-std=gnu11", "-I", os.path.join(ROOT, "include"), SRC,
                    pitorch_b200.LIB_PATH, f"-Wl,-rpath,{lib_dir}", "-o", str(exe)], check=True)
    return exe


def test_caller_owned_structs_train_like_the_reference(ptlib, tmp_path):
    g = golden("train_tiny.npz")
    T, steps, lr = int(g["T"]), int(g["steps"]), float(g["lr"])
    model = tmp_path / "tiny.bin"
    model.write_bytes(bytes(synth.make_blob("tiny")))
    toks = tmp_path / "tokens.i32"
    toks.write_bytes(np.ascontiguousarray(g["tokens"], dtype=np.int32).tobytes())
    exe = build(tmp_path)
    r = subprocess.run([str(exe), str(model), str(toks), str(T), str(steps), repr(lr), "1"],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and r.stdout.strip().endswith("OK"), r.stdout[-2000:] + r.stderr[-2000:]
    losses = np.array([float(ln.split()[2]) for ln in r.stdout.splitlines() if ln.startswith("step ")])
    ref = g["losses"].astype(np.float64)
    assert len(losses) == steps
    assert np.all(np.abs(losses - ref) <= 1e-4 * np.abs(ref)), (losses, ref)
