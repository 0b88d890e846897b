"""The layer pipeline on 2+ GPUs (pt_dist_setup / pt_dist_forward_step /
pt_dist_train_step), one process per GPU as the reference runs one program
per Pi (pitorch/dist/pt_dist_pipeline.c).

Parity targets are the reference's host C on the same weights (decode
fixtures), and -- for training -- the single-context pt_train_step, which is
the same arithmetic split differently (dev/tests/host/test_shard_train.c
checks the shard pipeline against the full model the same way).
Skipped when fewer GPUs are visible than the case needs.
"""
import multiprocessing as mp
import os
import socket

import numpy as np
import pytest

from conftest import golden

pytestmark = pytest.mark.gpu


def n_gpus():
    import pitorch_b200
    return pitorch_b200.lib().ptc_device_count()


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, task, q):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["PT_DIST_PORT"] = str(port)
        os.environ["PT_DIST_TIMEOUT_MS"] = "60000"
        from pitorch_b200 import api, synth
        name, kind = task[:2]
        if len(task) > 2:
            os.environ["PT_DIST_P2P"] = task[2]
        cfg = synth.CONFIGS[name]
        blob = synth.make_blob(cfg)
        if kind == "decode":
            g = golden(f"decode_{name}.npz")
            n = int(g["n_pos"])
            pipe = api.Pipeline(blob, rank, world, device=rank)
            dev = pipe.generate_greedy(g["prompt"], n)
            host = pipe.decode_greedy(g["prompt"], n)
            q.put((rank, pipe.is_head, dev.tolist(), host.tolist()))
            pipe.close()
        elif kind == "decode_vp":   # the classifier split over all ranks
            g = golden(f"decode_{name}.npz")
            n = int(g["n_pos"])
            pipe = api.Pipeline(blob, rank, world, device=rank)
            pipe.vocab_parallel()
            dev = pipe.generate_greedy(g["prompt"], n)
            rows = tuple(int(r) for r in g["rows"] if r < n)
            host, kept = pipe.decode_greedy(g["prompt"], n, logit_rows=rows)
            again = pipe.generate_greedy(g["prompt"], n)   # a second decode on the same links
            q.put((rank, pipe.is_head, dev.tolist(),
                   (host.tolist(), {k: v.tolist() for k, v in kept.items()}, again.tolist())))
            pipe.close()
        elif kind == "train":
            g = golden(f"train_{name}.npz")
            T = int(g["T"])
            pipe = api.Pipeline(blob, rank, world, device=rank, max_T=T)
            losses = [pipe.train_step(g["tokens"], float(g["lr"])) for _ in range(3)]
            q.put((rank, pipe.is_head, losses, None))
            pipe.close()
        else:   # "train_mb": GPipe over 4 microbatches of the same tokens, lr / 4
            g = golden(f"train_{name}.npz")
            T, M = int(g["T"]), 4
            pipe = api.Pipeline(blob, rank, world, device=rank, max_T=T)
            toks = np.tile(np.asarray(g["tokens"], dtype=np.int32), M)
            losses = [pipe.train_step_mb(toks, M, float(g["lr"]) / M) for _ in range(3)]
            q.put((rank, pipe.is_head, losses, None))
            pipe.close()
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, None, repr(e), None))


def run_ranks(world, task):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, task, q)) for r in range(world)]
    for p in ps:
        p.start()
    out = []
    try:
        for _ in range(world):
            out.append(q.get(timeout=240))
    finally:
        for p in ps:   # a rank that died leaves the others waiting: end them
            p.join(timeout=60)
            if p.is_alive():
                p.terminate()
                p.join(timeout=30)
    assert len(out) == world, f"only {len(out)} of {world} ranks reported"
    for r, head, a, b in out:
        assert head is not None, f"rank {r} failed: {a}"
    return out


@pytest.mark.parametrize("name,world,transport", [("tiny", 2, "1"), ("stories15M", 2, "1"), ("stories15M", 2, "0"),
                                                  ("stories15M", 4, "1"), ("stories110M", 4, "1"),
                                                  ("stories110M", 4, "0")])
def test_pipeline_decode_matches_reference(ptlib, name, world, transport):
    """transport "1": decode hops as peer stores over NVLink (ptc_hop_*, the
    default); "0": NCCL send/recv (PT_DIST_P2P=0)."""
    if n_gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    out = run_ranks(world, (name, "decode", transport))
    g = golden(f"decode_{name}.npz")
    n = int(g["n_pos"])
    head = [o for o in out if o[1]]
    assert len(head) == 1
    _, _, dev, host = head[0]
    assert np.array_equal(np.array(dev), g["tokens"][:n])
    assert np.array_equal(np.array(host), g["tokens"][:n])


@pytest.mark.parametrize("name,world", [("tiny", 2), ("stories15M", 2), ("stories15M", 4), ("stories110M", 4),
                                        ("stories110M", 8)])
def test_pipeline_vocab_parallel_matches_reference(ptlib, name, world):
    """The classifier split over all ranks (pt_dist_vocab_parallel): each
    rank's rows, the argmax combined across ranks on the GPU. The token
    streams of the device loop, of host-driven steps and of a second decode
    equal the reference's, and the host logits the head gathers match the
    reference's rows within 1e-4 of their max."""
    if n_gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    out = run_ranks(world, (name, "decode_vp"))
    g = golden(f"decode_{name}.npz")
    n = int(g["n_pos"])
    head = [o for o in out if o[1]]
    assert len(head) == 1
    _, _, dev, (host, kept, again) = head[0]
    assert np.array_equal(np.array(dev), g["tokens"][:n])
    assert np.array_equal(np.array(host), g["tokens"][:n])
    assert np.array_equal(np.array(again), g["tokens"][:n])
    for r, row in zip(g["rows"], g["logits_rows"]):
        if r < n:
            got = np.array(kept[int(r)], dtype=np.float64)
            assert np.abs(got - row).max() <= 1e-4 * np.abs(row).max(), int(r)


@pytest.mark.parametrize("world", [2, 4])
def test_pipeline_training_matches_single_gpu(ptlib, world):
    if n_gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    out = run_ranks(world, ("stories15M", "train"))
    g = golden("train_stories15M.npz")
    head = [o for o in out if o[1]]
    losses = np.array(head[0][2], dtype=np.float64)
    ref = g["losses"][:3].astype(np.float64)
    assert np.all(np.abs(losses - ref) <= 1e-4 * np.abs(ref)), (losses, ref)


@pytest.mark.parametrize("world", [2, 4])
def test_pipeline_microbatch_training_matches_single_gpu(ptlib, world):
    """GPipe (pt_dist_train_step_mb, the schedule of the reference's
    dev/tests/dist/train_pp/test_train_pp_mb_rank{0,1}.c): 4 microbatches of
    the fixture's tokens with lr / 4 accumulate to the same update as one
    pt_train_step with lr, so the losses of 3 steps equal the reference's
    single-step losses within 1e-4."""
    if n_gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    out = run_ranks(world, ("stories15M", "train_mb"))
    g = golden("train_stories15M.npz")
    head = [o for o in out if o[1]]
    losses = np.array(head[0][2], dtype=np.float64)
    ref = g["losses"][:3].astype(np.float64)
    assert np.all(np.abs(losses - ref) <= 1e-4 * np.abs(ref)), (losses, ref)
