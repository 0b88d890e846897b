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
