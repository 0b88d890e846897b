"""bench.py's reference arm (--impl reference) on the host CPU: the JSON line
the driver reads, at N = 1 and under torchrun with two ranks (rank 0 alone
times and prints; the other rank exits 0 without work)."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def last_json(out):
    lines = [ln for ln in out.splitlines() if ln.startswith("{")]
    assert lines, out[-2000:]
    return [json.loads(ln) for ln in lines]


def check_line(d, n_gpus):
    assert d["impl"] == "reference" and d["n_gpus"] == n_gpus
    assert d["metric"] == "batch-1 decode tokens/s (stories110M shape)" and d["unit"] == "tokens/s"
    assert d["value"] > 0 and d["higher_is_better"] is True and d["scaling"] == "strong"
    assert d["config"]["model"] == "stories110M" and d["config"]["seq_len"] == 1024
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["cores"] == 1 and cb["kind"] in ("reference", "port") and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_one_process():
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "0"],
                       cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = last_json(r.stdout)
    assert len(lines) == 1
    check_line(lines[0], 1)


def test_reference_arm_two_ranks_rank0_only():
    env = dict(os.environ, OMP_NUM_THREADS="1")
    r = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
                        "--master-addr", "127.0.0.1", "--master-port", "29671", "bench.py", "--impl", "reference",
                        "--gpus", "2", "--steps", "1", "--warmup", "0"],
                       cwd=ROOT, env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = last_json(r.stdout)
    assert len(lines) == 1
    check_line(lines[0], 2)


def _bench():
    sys.path.insert(0, ROOT)
    import bench
    return bench


def test_stream_parity_against_the_fixture():
    """The N = 1 line's parity key: the reference stream itself matches all
    1024 positions; a stream changed at position p matches p positions and
    counts as equal only when p lies past the reference's first near-tie."""
    import numpy as np
    bench = _bench()
    g = np.load(os.path.join(ROOT, "tests", "golden", "decode_stories110M_long.npz"))
    ref = np.asarray(g["tokens"], dtype=np.int32)
    seq = len(ref)
    p = bench.stream_parity(ref.copy(), seq)
    assert p["matched_positions"] == seq and p["equal_positions"] == seq and p["equal_up_to_first_near_tie"]
    first_tie = p["first_near_tie"]
    early = min(first_tie, seq) // 2
    bad = ref.copy()
    bad[early] = (bad[early] + 1) % 32000
    q = bench.stream_parity(bad, seq)
    assert q["matched_positions"] == early and q["equal_positions"] == seq - 1
    assert q["equal_up_to_first_near_tie"] is False


def test_decode_byte_model():
    """Algorithmic bytes per token of the 110M decode: 438.04 MB of weights
    (tied classifier read once) plus the K/V rows read and written; the mean
    over 1024 positions is the 475.98 MB the roofline uses."""
    import numpy as np
    bench = _bench()
    cfg = bench.synth.CONFIGS["stories110M"]
    b0 = bench.decode_bytes_per_token(cfg, 0)
    mean = np.mean([bench.decode_bytes_per_token(cfg, p) for p in range(cfg[6])])
    assert abs(b0 / 1e6 - 438.1) < 0.2, b0
    assert abs(mean / 1e6 - 475.98) < 0.01, mean


def test_cpu_sample_positions_cover_the_decode():
    bench = _bench()
    pos = bench.stratified_positions(96, 1024)
    assert len(pos) == 96 and pos == sorted(pos) and pos[0] >= 0 and pos[-1] < 1024
    assert abs(sum(pos) / len(pos) - 511.5) < 1.0   # mean position of the whole decode
