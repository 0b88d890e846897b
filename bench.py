#!/usr/bin/env python3
"""Benchmark: batch-1 greedy decode tokens/s, stories110M shape, on B200.

One step = one full greedy decode of seq_len = 1024 positions (8 seeded prompt
tokens teacher-forced, then argmax feedback), from a reset KV cache, on
seeded N(0, 0.02) fp32 weights of the stories110M shape (438 MB of weights,
larger than the 126 MB L2, so every token streams its weights from HBM).

  value  device-resident run: the decode's CUDA graph chain is enqueued with
         inputs already on the GPU, timed with CUDA events on its stream.
  e2e    the drop-in C API path: pt_forward_step(ctx, token) per position
         (host token in, host token out), timed with CUDA events around the
         whole loop.

After the decode's timed region the N = 1 line also carries the isolated
matvec sweep (`matvec_sweep`, cold column of the 9 shapes; --sweep prints the
full per-shape lines) and the stories15M training step (`train`; --train
prints it alone). --no-extras leaves both out.

N > 1 (torchrun): the layer pipeline over N GPUs (pt_dist_forward_step), the
last rank holding embedding + classifier as in the pitorch ring.

--impl reference times the reference's own host C decode (oracle/_ref, built
from the reference sources) on this host's CPU on a bounded sample of
positions per step.
"""
import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

from pitorch_b200 import synth  # noqa: E402

MODEL = "stories110M"
N_PROMPT = 8
METRIC = "batch-1 decode tokens/s (stories110M shape)"


def peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.device = device
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# DRAM bytes (read + write) per launch of each decode kernel from one ncu
# capture of the 16-position bench case (positions 0-15, so the attention
# block's KV share is that of those positions, not of the mean position):
# dram__bytes_read.sum + dram__bytes_write.sum.
TRAFFIC = {"attention block": 9518592, "ffn block": 18916608, "classifier": 102142208}
TRAFFIC_SOURCE = ("ncu --set full --clock-control none -k regex:'k_attn_fused|k_ffn' -s 44 -c 2 "
                  "-o layer python bench.py --positions 16 --steps 1 --warmup 1 --no-cpu-baseline "
                  "(profiles/k_attn_fused_k_ffn_110M.md: layer 10 of position 1, so the attention block's "
                  "KV bytes are those of that position; the classifier from "
                  "profiles/k_mv_cls_110M.md)")


def decode_bytes_per_token(cfg, pos):
    """Algorithmic HBM bytes of one decode position: all weights read once
    (tied classifier = embedding table, read once by the classifier, plus one
    embedding row), the KV cache read for positions <= pos and one KV row
    written per layer."""
    dim, hidden, L, nh, nkv, V, seq = cfg
    kvd = nkv * (dim // nh)
    weights = 4 * (V * dim + L * (2 * dim + 2 * dim * dim + 2 * kvd * dim + 3 * hidden * dim) + dim)
    kv = 4 * (2 * L * (pos + 1) * kvd + 2 * L * kvd)
    return weights + kv + 4 * dim


def stratified_positions(n, seq):
    """n decode positions spread evenly over [0, seq): a CPU sample whose
    mean cost per token is that of the whole decode (attention grows with
    the position)."""
    return [int((k + 0.5) * seq / n) for k in range(n)]


def time_cpu_positions(m, positions, n_layers, token=1):
    """The reference's own forward (pt_forward_embed, pt_forward_layers_range,
    pt_forward_head: llama2.c:201-206) at each sampled position; the KV rows
    of earlier positions are whatever the cache holds, which changes no
    arithmetic cost. Returns seconds."""
    t0 = time.perf_counter()
    for p in positions:
        m.forward_embed(token)
        m.forward_layers_range(p, 0, n_layers)
        m.forward_head()
    return time.perf_counter() - t0


def run_reference(args, rank):
    if rank != 0:
        return 0
    import oracle
    cfg = synth.CONFIGS[MODEL]
    blob = synth.make_blob(cfg)
    impl = "reference" if oracle.ref_available() else "port"
    m = oracle.Model(blob, impl=impl)
    sample = 24   # positions per step: a bounded sample of the 1024-position decode
    positions = stratified_positions(sample, cfg[6])
    for _ in range(args.warmup):
        time_cpu_positions(m, positions, cfg[2])
    dt = 0.0
    for _ in range(args.steps):
        dt += time_cpu_positions(m, positions, cfg[2])
    v = sample * args.steps / dt
    line = {
        "metric": METRIC, "value": v, "unit": "tokens/s", "impl": "reference",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000 * dt / args.steps, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        # the device arm's workload; each step times a bounded sample of it
        "config": {"workload": f"{MODEL} batch-1 greedy decode, {cfg[6]} positions per step",
                   "model": MODEL, "global_batch": 1, "seq_len": cfg[6], "parallelism": "cpu-1thread",
                   "sample_positions_per_step": sample, "prompt": N_PROMPT},
        "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": 1, "kind": impl,
                         "sample": f"{sample} positions per step spread evenly over the 1024-position "
                                   f"decode ({positions[0]}, {positions[1]}, ..., {positions[-1]}), the "
                                   "reference's staged forward at each, single thread"},
        "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def cpu_baseline_sample(blob, cfg):
    import oracle
    impl = "reference" if oracle.ref_available() else "port"
    m = oracle.Model(blob, impl=impl)
    n = 96
    positions = stratified_positions(n, cfg[6])
    dt = time_cpu_positions(m, positions, cfg[2])
    return {"value": n / dt, "unit": "tokens/s", "cores": 1, "kind": impl,
            "sample": f"{n} positions spread evenly over the 1024-position decode ({positions[0]}, "
                      f"{positions[1]}, ..., {positions[-1]}), the reference's staged forward at each "
                      "(pt_forward_embed, pt_forward_layers_range, pt_forward_head), single thread"}


NEAR_TIE = 1e-5   # top-2 gap / max|logit| below which another fp32 order may flip the argmax


def stream_parity(tokens, seq):
    """The timed decode's token stream against the reference host C's
    1024-position stream (tests/golden/decode_stories110M_long.npz): equal up
    to the reference's first near-tie, after which a different fp32
    summation order may legitimately pick the other token."""
    path = os.path.join(REPO, "tests", "golden", "decode_stories110M_long.npz")
    if not os.path.exists(path):
        return {"fixture": None}
    g = np.load(path)
    ref = g["tokens"][:seq]
    clear = g["top2_gap"][:seq] >= NEAR_TIE * g["logit_absmax"][:seq]
    clear[: N_PROMPT - 1] = True
    first_tie = int(np.argmin(clear)) if not clear.all() else seq
    eq = tokens[:seq] == ref
    matched = int(np.argmin(eq)) if not eq.all() else seq
    return {"fixture": "tests/golden/decode_stories110M_long.npz (reference host C)",
            "compared": "token stream of the last timed step", "first_near_tie": first_tie,
            "matched_positions": matched, "equal_up_to_first_near_tie": bool(matched >= min(first_tie + 1, seq)),
            "equal_positions": int(eq.sum()), "positions": int(seq)}


def run_single(args):
    import ctypes as C
    import pitorch_b200
    from pitorch_b200 import api
    L = pitorch_b200.lib()
    cfg = synth.CONFIGS[MODEL]
    dim, hidden, nl, nh, nkv, V, seq = cfg
    if args.positions:
        seq = min(args.positions, seq)
    blob = synth.make_blob(cfg)
    prompt = synth.make_prompt(V, N_PROMPT)
    ctx = api.Context(blob)
    dec = ctx.ptc_decoder()
    pctx = ctx.ptc_ctx()
    timer = L.ptc_timer_create(pctx)

    def device_run(n_steps):
        for _ in range(n_steps):
            L.ptc_decoder_reset(dec)
            L.ptc_decoder_generate_begin(dec, api.ip(prompt), N_PROMPT)
            L.ptc_decoder_enqueue_steps(dec, seq)

    # warm-up (also checks the stream against the host path below)
    for _ in range(args.warmup):
        device_run(1)
    L.ptc_sync(pctx)
    toks_dev = np.zeros(seq, np.int32)
    L.ptc_decoder_read_tokens(dec, api.ip(toks_dev), seq)

    # ---- device-resident timed region (CUDA events on the decode stream) ----
    # Per-step resets/prompt loads are part of each step (tiny H2D copies).
    L.ptc_sync(pctx)
    with ClockSampler(0) as clk:
        ms_total = 0.0
        for _ in range(args.steps):
            L.ptc_decoder_reset(dec)
            L.ptc_decoder_generate_begin(dec, api.ip(prompt), N_PROMPT)
            L.ptc_timer_start(timer)
            L.ptc_decoder_enqueue_steps(dec, seq)
            L.ptc_timer_stop(timer)
            ms_total += L.ptc_timer_ms(timer)
    ms_per_step = ms_total / args.steps
    toks_timed = np.zeros(seq, np.int32)
    L.ptc_decoder_read_tokens(dec, api.ip(toks_timed), seq)
    value = seq / (ms_per_step / 1000.0)

    # ---- e2e through pt_forward_step (host token in / host token out) -------
    ctx.ctx.sync_logits = 0
    e2e_steps = max(1, min(args.steps, 3))
    L.ptc_sync(pctx)
    t0 = time.perf_counter()
    L.ptc_timer_start(timer)
    toks_host = None
    for _ in range(e2e_steps):
        toks_host = ctx.decode_greedy(prompt, seq)
    L.ptc_timer_stop(timer)
    e2e_ms = L.ptc_timer_ms(timer) / e2e_steps
    e2e_wall_ms = 1000 * (time.perf_counter() - t0) / e2e_steps
    e2e_value = seq / (e2e_ms / 1000.0)
    streams_match = bool(np.array_equal(toks_host, toks_dev))

    # ---- per-kernel rooflines: each decode kernel alone, 50 back-to-back
    # launches at the mean position (CUDA events on the decoder's stream) ----
    hbm, src = peaks()
    launches_per_step = L.ptc_decoder_launches_per_step(dec)
    kvd = nkv * (dim // nh)
    pos_mid = seq // 2
    n_rep = 50

    def time_kernel(kind, layer):
        L.ptc_sync(pctx)
        L.ptc_timer_start(timer)
        for _ in range(n_rep):
            L.ptc_decoder_enqueue_kernel(dec, kind, layer, pos_mid)
        L.ptc_timer_stop(timer)
        return L.ptc_timer_ms(timer) / n_rep

    fused = launches_per_step == 2 * nl + 1
    kern = {
        # attention block: q/k/v and wo rows, the rms gain, K/V rows of
        # positions <= pos read, one K/V row written, x read
        "attention block": (0, 4 * (dim * (dim + 2 * kvd) + dim * dim + dim + 2 * (pos_mid + 1) * kvd + 2 * kvd + dim),
                            "k_attn_fused: per-head clusters; q/k/v rows, RoPE, KV attention, wo" if fused
                            else "q/k/v, attention and wo kernels"),
        "ffn block": (1, 4 * (3 * hidden * dim + dim + dim),
                      "k_ffn: rmsnorm, w1/w3 rows, silu, transposed-w2 split-K"),
        "classifier": (2, 4 * (V * dim + V + 2 * dim), "k_mv<CLS>: final rmsnorm, 32000 rows, argmax"),
    }
    kernels = {}
    for name, (kind, nbytes, what) in kern.items():
        ms_k = time_kernel(kind, nl // 2)
        gbs = nbytes / (ms_k / 1000.0) / 1e9
        kernels[name] = {"kernel": what, "bytes_per_launch": nbytes, "ms_per_launch": ms_k,
                         "achieved": gbs, "frac": gbs / hbm,
                         "launches_per_step": (nl if kind < 2 else 1) * seq}
    L.ptc_decoder_reset(dec)
    # dominant kernel: the largest share of the step's kernel time
    dom = max(kernels, key=lambda k: kernels[k]["ms_per_launch"] * kernels[k]["launches_per_step"])
    dk = kernels[dom]

    # whole-step roofline (bytes per token over the decode)
    mean_bytes = np.mean([decode_bytes_per_token(cfg, p) for p in range(seq)])
    step_gbs = mean_bytes * seq / (ms_per_step / 1000.0) / 1e9
    L.ptc_timer_destroy(timer)
    ctx.close()
    clocks = clk.summary()
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
        # one whole decode per step whatever the GPU count (the N > 1 line is
        # the layer pipeline over the same decode): total work is fixed
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,0.02) fp32 weights, seeded 8-token prompt)",
        "config": {"workload": f"{MODEL} batch-1 greedy decode, {seq} positions per step",
                   "model": MODEL, "global_batch": 1, "seq_len": seq, "parallelism": "none",
                   "l2_policy": "weights 438 MB > 126 MB L2: every token re-streams from HBM"},
        "e2e": {"value": e2e_value, "unit": "tokens/s", "api": "pt_forward_step per position",
                "h2d_bytes_per_step": 8 * seq, "d2h_bytes_per_step": 4 * seq,
                "wall_ms_per_step": e2e_wall_ms, "token_stream_equals_device_loop": streams_match},
        "roofline": {"kernel": f"{dom}: {dk['kernel']}", "bound": "hbm", "achieved": dk["achieved"],
                     "peak": hbm, "unit": "GB/s", "frac": dk["frac"], "peak_source": f"{src} hbm_gbs (burst copy)",
                     "traffic": TRAFFIC.get(dom), "traffic_source": TRAFFIC_SOURCE,
                     "bytes_per_launch": dk["bytes_per_launch"], "ms_per_launch": dk["ms_per_launch"],
                     "position": pos_mid, "timing": f"{n_rep} back-to-back launches, CUDA events"},
        "kernels": kernels,
        "step_roofline": {"bytes_per_token": float(mean_bytes), "achieved": step_gbs, "peak": hbm,
                          "unit": "GB/s", "frac": step_gbs / hbm,
                          "roofline_tokens_per_s": hbm * 1e9 / mean_bytes},
        "gpu_launches": args.steps * seq * launches_per_step,
        "clocks": clocks,
        "parity": stream_parity(toks_timed, seq),
    }
    if not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_sample(blob, cfg)
    if not args.no_extras:
        # the path's two other measured workloads, after the decode's timed
        # region: the isolated matvec sweep (cold column) and the training step
        sw = MatvecSweep()
        line["matvec_sweep"] = sw.summary(3, 3)
        sw.close()
        line["train"] = train_line(3, 10, not args.no_cpu_baseline)
    print(json.dumps(line), flush=True)
    return 0


ATTN_PHASES = [("release after the previous kernel's end", None, 1),
               ("x read + rmsnorm", 1, 2), ("q/k/v rows resident", 2, 3),
               ("q/k/v row pairs + RoPE + stores to the cluster", 3, 8),
               ("ticket + wo / K/V copy issue", 8, 9), ("q/k/v cluster barrier wait", 9, 4),
               ("attention rounds", 4, 5), ("partial exchange (cluster)", 5, 6),
               ("merge of the partials", 6, 10), ("wo slice resident", 10, 11),
               ("wo rows + reductions", 11, 7)]
FFN_PHASES = [("release after the previous kernel's end", None, 1), ("x read + rmsnorm", 1, 2),
              ("w1/w3 rows resident", 2, 3), ("h1, h3 rows + silu", 3, 8), ("w2t rows resident", 8, 4),
              ("w2t product + reductions", 4, 7)]
CLS_PHASES = [("release after the previous kernel's end", None, 1), ("x read + rmsnorm", 1, 2),
              ("32000 rows + logits", 2, 6), ("argmax + step state (last CTA)", 6, 7)]


def run_timeline(args):
    """Phase timeline of the decode kernels (ptc_decoder_trace): the 110M
    device loop runs to position `start` untraced, then 16 positions with
    every kernel stamping %globaltimer at its phase points. Each phase is the
    time between the LAST CTA of the kernel passing one point and the last
    CTA passing the next, so the sum over a position's kernels is its
    critical path. Medians over the 16 positions (and over layers 1..L-1 for
    the layer kernels). Stamping adds two atomics per CTA per point, so the
    traced positions run slightly slower than untraced ones."""
    import ctypes as C
    import pitorch_b200
    from pitorch_b200 import api
    L = pitorch_b200.lib()
    cfg = synth.CONFIGS[MODEL]
    dim, hidden, nl, nh, nkv, V, seq = cfg
    blob = synth.make_blob(cfg)
    prompt = synth.make_prompt(V, N_PROMPT)
    ctx = api.Context(blob)
    dec = ctx.ptc_decoder()
    pctx = ctx.ptc_ctx()
    start = args.timeline_start - args.timeline_start % 8
    L.ptc_decoder_reset(dec)
    L.ptc_decoder_generate_begin(dec, api.ip(prompt), N_PROMPT)
    L.ptc_decoder_enqueue_steps(dec, start)
    L.ptc_sync(pctx)
    n = L.ptc_decoder_trace(dec, 1)
    L.ptc_decoder_enqueue_steps(dec, 16)
    L.ptc_sync(pctx)
    buf = (C.c_ulonglong * n)()
    L.ptc_decoder_read_trace(dec, buf, n)
    L.ptc_decoder_trace(dec, 0)
    ctx.close()
    t = np.frombuffer(buf, dtype=np.uint64).astype(np.float64).reshape(16, 2 * nl + 1, 12, 2)
    last = t[..., 1]    # latest CTA per event (ns)
    first = t[..., 0]
    order = [(start + i) % 16 for i in range(16)]

    def phase_stats(k_list, phases, skip_first_pos=False):
        out = {}
        for name, a, b in phases:
            vals = []
            for i, slot in enumerate(order):
                if skip_first_pos and i == 0:
                    continue
                for k in k_list:
                    if a is None:   # previous kernel's end: k-1, or the previous position's classifier
                        if k > 0:
                            prev = last[slot, k - 1, 7]
                        elif i > 0:
                            prev = last[order[i - 1], 2 * nl, 7]
                        else:
                            continue
                        vals.append(last[slot, k, b] - prev)
                    else:
                        vals.append(last[slot, k, b] - last[slot, k, a])
            out[name] = float(np.median(vals)) / 1000.0 if vals else None
        return out

    attn = phase_stats([2 * l for l in range(1, nl)], ATTN_PHASES)
    ffn = phase_stats([2 * l + 1 for l in range(1, nl)], FFN_PHASES)
    cls = phase_stats([2 * nl], CLS_PHASES)
    per_pos = [(last[order[i], 2 * nl, 7] - last[order[i - 1], 2 * nl, 7]) / 1000.0 for i in range(1, 16)]
    layer = [(last[slot, 2 * l + 1, 7] - last[slot, 2 * l - 1, 7]) / 1000.0
             for slot in order[1:] for l in range(1, nl)]
    # how early each kernel's CTAs are resident before their release: the
    # window the weight copies issued before griddepcontrol.wait have
    lead = {nm: float(np.median([(last[s_, k, 1] - first[s_, k, 0]) / 1000.0 for s_ in order
                                 for k in ks]))
            for nm, ks in (("attention block", [2 * l for l in range(1, nl)]),
                           ("ffn block", [2 * l + 1 for l in range(1, nl)]), ("classifier", [2 * nl]))}
    line = {"metric": "decode phase timeline (us, median)", "model": MODEL,
            "positions": [start, start + 15], "us_per_position": float(np.median(per_pos)),
            "us_per_layer": float(np.median(layer)), "attention_block": attn, "ffn_block": ffn,
            "classifier": cls, "first_cta_start_to_release_us": lead,
            "note": "latest CTA per phase point; traced positions pay two atomics per CTA per point"}
    print(json.dumps(line), flush=True)
    return 0


SWEEP_SHAPES = [(288, 288), (768, 288), (288, 768), (512, 512), (1376, 512), (2048, 768), (768, 2048),
                (32000, 288), (32000, 768)]
L2_BYTES = 126 * 1024 * 1024


def sweep_references(L, pc, stream, graph_time, hbm, src):
    """The sweep's two measured references: the L2 read bandwidth (48 MiB,
    L2-resident, read 20 times per graph replay by ptc_read_probe) and the
    per-call floor of a chain of dependent matvec launches (8 x 4, 512 per
    graph). Prints them as one JSON line and returns both."""
    l2_bytes = 48 << 20
    probe = L.ptc_alloc(pc, l2_bytes)
    sink = L.ptc_alloc(pc, 256)
    L.ptc_memset(pc, probe, 0, l2_bytes)
    ms = graph_time(lambda: [L.ptc_read_probe(probe, l2_bytes, sink, stream) for _ in range(20)], 10)
    l2_gbs = 20 * l2_bytes / (ms / 1000.0) / 1e9
    # per-call floor of dependent matvec launches (PDL chain in a graph)
    tW, tx, ty = L.ptc_alloc(pc, 8 * 4 * 4), L.ptc_alloc(pc, 64), L.ptc_alloc(pc, 64)
    L.ptc_memset(pc, tW, 0, 128)
    L.ptc_memset(pc, tx, 0, 64)
    floor_us = 1000 * graph_time(lambda: [L.ptc_matvec(tW, tx, ty, 8, 4, stream) for _ in range(512)], 10) / 512
    print(json.dumps({"metric": "matvec sweep references", "l2_read_gbs": l2_gbs,
                      "l2_probe": f"ptc_read_probe over {l2_bytes >> 20} MiB, 20 reads per graph replay",
                      "launch_floor_us": floor_us,
                      "launch_floor": "8x4 matvec, 512 dependent launches per graph (PDL)",
                      "hbm_peak_gbs": hbm, "hbm_peak_source": f"{src} hbm_gbs"}), flush=True)
    return l2_gbs, floor_us


class MatvecSweep:
    """The isolated fp32 matvec sweep y = W.x (W rows x cols, W ~ N(0,0.02),
    x ~ N(0,1), seeded) through the C ABI's ptc_matvec. Per shape:
      cold  back-to-back calls, each on a different copy of W, the copies
            together >= 2x L2 so every call streams W from HBM; the calls are
            one CUDA graph, timed with CUDA events (launches overlap through
            programmatic dependent launch, as in a decode step);
      hot   the same, always the same W (L2-resident when it fits);
      cpu_baseline  the reference's own smatvec_cpu (oracle/_ref), 1 thread.
    Algorithmic bytes per call: 4*(rows*cols + rows + cols).
    Two measured references come first: the L2 read bandwidth (ptc_read_probe
    over a 48 MiB buffer read back to back, L2-resident) for the hot column,
    and the per-call floor of a chain of dependent matvec launches (an 8 x 4
    matvec, whose bytes take no time), so that every shape's attainable time
    is max(bytes / peak, floor)."""

    def __init__(self, refs=True):
        import pitorch_b200
        self.L = L = pitorch_b200.lib()
        self.pc = L.ptc_create(0, 0)
        self.stream = L.ptc_stream(self.pc)
        self.timer = L.ptc_timer_create(self.pc)
        self.hbm, self.src = peaks()
        self.l2_gbs, self.floor_us = None, 0.0
        if refs:
            self.l2_gbs, self.floor_us = sweep_references(L, self.pc, self.stream, self.graph_time,
                                                          self.hbm, self.src)

    def graph_time(self, calls, reps):
        """ms per replay of a captured graph of the (callable) enqueues."""
        L, pc = self.L, self.pc
        L.ptc_capture_begin(pc)
        calls()
        g = L.ptc_capture_end(pc)
        for _ in range(3):
            L.ptc_graph_launch(g)
        L.ptc_sync(pc)
        L.ptc_timer_start(self.timer)
        for _ in range(reps):
            L.ptc_graph_launch(g)
        L.ptc_timer_stop(self.timer)
        ms = L.ptc_timer_ms(self.timer) / reps
        L.ptc_graph_destroy(g)
        return ms

    def shape(self, rows, cols, warmup, steps, modes=("cold", "hot"), cpu_s=0.3):
        """One shape's JSON record (see the class docstring)."""
        import oracle
        L, pc, stream, hbm = self.L, self.pc, self.stream, self.hbm
        rng = np.random.default_rng(1000 + rows + cols)
        W = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
        x = rng.standard_normal(cols).astype(np.float32)
        wbytes = W.nbytes
        n_copies = max(2, -(-2 * L2_BYTES // wbytes))
        dW = L.ptc_alloc(pc, wbytes * n_copies)
        dx = L.ptc_alloc(pc, cols * 4)
        dy = L.ptc_alloc(pc, rows * 4)
        L.ptc_h2d(pc, dW, W.ctypes.data, wbytes)
        for k in range(1, n_copies):
            L.ptc_d2d(pc, dW + k * wbytes, dW, wbytes)
        L.ptc_h2d(pc, dx, x.ctypes.data, cols * 4)
        L.ptc_sync(pc)
        # parity against the oracle (smatvec_cpu order), tolerance 1e-5
        L.ptc_matvec(dW, dx, dy, rows, cols, stream)
        y = np.zeros(rows, np.float32)
        L.ptc_d2h(pc, y.ctypes.data, dy, rows * 4)
        ref = oracle.matvec(W, x)
        err = float(np.abs(y - ref).max() / np.abs(ref).max())
        bytes_call = 4 * (rows * cols + rows + cols)
        res = {}
        for mode in modes:
            n_calls = n_copies if mode == "cold" else max(64, n_copies)
            while n_calls * bytes_call < 1.5e9 and n_calls < 4096:   # >= ~0.25 ms of work per replay
                n_calls *= 2
            L.ptc_capture_begin(pc)
            for i in range(n_calls):
                Wi = dW + (i % n_copies) * wbytes if mode == "cold" else dW
                L.ptc_matvec(Wi, dx, dy, rows, cols, stream)
            g = L.ptc_capture_end(pc)
            for _ in range(max(3, warmup)):
                L.ptc_graph_launch(g)
            L.ptc_sync(pc)
            reps = max(3, steps)
            L.ptc_timer_start(self.timer)
            for _ in range(reps):
                L.ptc_graph_launch(g)
            L.ptc_timer_stop(self.timer)
            ms = L.ptc_timer_ms(self.timer)
            L.ptc_graph_destroy(g)
            us_call = 1000 * ms / (reps * n_calls)
            gbs = bytes_call / (us_call * 1e-6) / 1e9
            peak_mode = hbm if (mode == "cold" or not self.l2_gbs or wbytes > L2_BYTES // 2) else self.l2_gbs
            attain_us = max(bytes_call / (peak_mode * 1e3), self.floor_us)
            res[mode] = {"GB/s": gbs, "us_per_call": us_call, "calls_per_graph": n_calls,
                         "frac_of_hbm": gbs / hbm, "peak": peak_mode,
                         "peak_kind": "hbm" if peak_mode == hbm else "l2 (measured)",
                         "frac_of_peak": gbs / peak_mode,
                         "attainable_us": attain_us, "frac_of_attainable": attain_us / us_call}
        rec = {"shape": f"{rows}x{cols}", "bytes_per_call": bytes_call, "parity_rel_err": err,
               "cold_copies": n_copies, "w_bytes": wbytes, **res}
        if cpu_s > 0:
            # CPU: the reference's smatvec_cpu on a bounded sample
            impl = "reference" if oracle.ref_available() else "port"
            n_cpu, t0 = 0, time.perf_counter()
            while time.perf_counter() - t0 < cpu_s or n_cpu < 2:
                oracle.matvec(W, x, impl=impl)
                n_cpu += 1
            cpu_us = 1e6 * (time.perf_counter() - t0) / n_cpu
            rec["cpu_baseline"] = {"value": bytes_call / (cpu_us * 1e-6) / 1e9, "unit": "GB/s", "cores": 1,
                                   "kind": impl, "us_per_call": cpu_us,
                                   "sample": f"{n_cpu} calls of smatvec_cpu on the same W, x"}
        return rec

    def summary(self, warmup, steps):
        """The cold column of all 9 shapes in compact form, for the decode
        line (so every default bench run carries the matvec sweep)."""
        out = {"l2_read_gbs": self.l2_gbs, "launch_floor_us": self.floor_us,
               "peak": self.hbm, "peak_source": f"{self.src} hbm_gbs",
               "timing": "cold: one CUDA graph of back-to-back calls on copies of W >= 2x L2, CUDA events",
               "shapes": {}}
        for rows, cols in SWEEP_SHAPES:
            r = self.shape(rows, cols, warmup, steps, modes=("cold",), cpu_s=0.0)
            c = r["cold"]
            out["shapes"][r["shape"]] = {"GB/s": round(c["GB/s"], 1), "us_per_call": round(c["us_per_call"], 3),
                                         "frac_of_hbm": round(c["frac_of_hbm"], 3),
                                         "attainable_us": round(c["attainable_us"], 3),
                                         "frac_of_attainable": round(c["frac_of_attainable"], 3),
                                         "parity_rel_err": r["parity_rel_err"]}
        return out

    def close(self):
        self.L.ptc_timer_destroy(self.timer)
        self.L.ptc_destroy(self.pc)


def run_sweep(args):
    """One JSON line per shape of the isolated matvec sweep (MatvecSweep)."""
    sw = MatvecSweep(refs=not args.sweep_no_refs)
    shapes = SWEEP_SHAPES
    if args.sweep_shapes:
        shapes = [tuple(int(v) for v in s.split("x")) for s in args.sweep_shapes.split(",")]
    for rows, cols in shapes:
        r = sw.shape(rows, cols, args.warmup, args.steps)
        line = {"metric": "fp32 matvec GB/s", "shape": r["shape"], "unit": "GB/s", "n_gpus": 1,
                "value": r["cold"]["GB/s"], "higher_is_better": True, "dtype": "f32", "data": "synthetic",
                "bytes_per_call": r["bytes_per_call"], "cold": r["cold"], "hot": r["hot"],
                "cold_copies": r["cold_copies"],
                "l2_policy": f"cold: {r['cold_copies']} copies of W = "
                             f"{r['cold_copies'] * r['w_bytes'] / 2**20:.0f} MiB >= 2x L2",
                "peak": sw.hbm, "peak_source": f"{sw.src} hbm_gbs", "parity_rel_err": r["parity_rel_err"],
                "cpu_baseline": r["cpu_baseline"]}
        print(json.dumps(line), flush=True)
    sw.close()
    return 0


def train_flops(cfg, T):
    """Algorithmic FLOPs of one pt_train_step: forward 2*T*P_lin, backward dX
    and dW 2*(T-1)*P_lin each (P_lin = the linear layers' parameters: per
    layer 2*dim^2 + 2*kvd*dim + 3*hidden*dim, plus the V*dim classifier), plus
    attention forward and backward (~4x the forward score/value products)."""
    dim, hidden, L, nh, nkv, V, seq = cfg
    kvd = nkv * (dim // nh)
    p_lin = L * (2 * dim * dim + 2 * kvd * dim + 3 * hidden * dim) + V * dim
    attn_fwd = L * 2 * 2 * dim * T * (T + 1) / 2     # q.k and p.v over the causal triangle
    return 2 * T * p_lin + 2 * 2 * (T - 1) * p_lin + attn_fwd * 3


def run_train(args):
    """Training throughput: pt_train_step on the stories15M shape, T = 256
    seeded tokens, lr 1e-3 (the reference's training benchmark settings), timed with CUDA
    events around K whole steps (each returns its loss to the host)."""
    print(json.dumps(train_line(args.warmup, args.steps, not args.no_cpu_baseline)), flush=True)
    return 0


def train_line(warmup, steps, cpu):
    """The training measurement of run_train as a dict, with the GEMM
    launches of the timed steps by path (ptc_gemm_counters)."""
    import ctypes as C
    import oracle
    import pitorch_b200
    from pitorch_b200 import api
    L = pitorch_b200.lib()
    model, T, lr = "stories15M", 256, 1e-3
    cfg = synth.CONFIGS[model]
    blob = synth.make_blob(cfg)
    tokens = synth.make_tokens(cfg[5], T)
    ctx = api.Context(blob, max_T=T)
    pc = ctx.ptc_ctx()
    timer = L.ptc_timer_create(pc)
    losses = []
    for _ in range(warmup):
        losses.append(ctx.train_step(tokens, lr))
    L.ptc_sync(pc)
    cnt0, cnt1 = (C.c_longlong * 4)(), (C.c_longlong * 4)()
    L.ptc_gemm_counters(cnt0)
    with ClockSampler(0) as clk:
        L.ptc_timer_start(timer)
        for _ in range(steps):
            losses.append(ctx.train_step(tokens, lr))
        L.ptc_timer_stop(timer)
        ms = L.ptc_timer_ms(timer) / steps
    L.ptc_gemm_counters(cnt1)
    L.ptc_timer_destroy(timer)
    ctx.close()
    flops = train_flops(cfg, T)
    line = {
        "metric": "stories15M train step tokens/s (T=256)", "value": T / (ms / 1000.0), "unit": "tokens/s",
        "n_gpus": 1, "steps": steps, "warmup": warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,0.02) weights, seeded uniform tokens)",
        "config": {"workload": "pt_train_step: forward, cross-entropy, backward, SGD", "model": model,
                   "global_batch": 1, "seq_len": T, "lr": lr, "parallelism": "none"},
        "achieved_gflops": flops / (ms / 1000.0) / 1e9, "flops_per_step": flops,
        "losses_first": losses[:3], "clocks": clk.summary(),
    }
    per = [(cnt1[k] - cnt0[k]) / steps for k in range(4)]
    line["gemm_launches_per_step"] = {"tensor_core": per[0], "simt": per[1], "splitk_reduce": per[2],
                                      "simt_cluster_reduced": per[3]}
    if cpu:
        impl = "reference" if oracle.ref_available() else "port"
        m = oracle.Model(blob, max_T=T, impl=impl)
        t0 = time.perf_counter()
        ref_loss = m.train_step(tokens, lr)
        dt = time.perf_counter() - t0
        line["cpu_baseline"] = {"value": T / dt, "unit": "tokens/s", "cores": 1, "kind": impl,
                                "s_per_step": dt, "sample": "one pt_train_step at T=256 on the same weights"}
        line["loss_rel_err_step0"] = abs(losses[0] - ref_loss) / abs(ref_loss) if warmup else None
    return line


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="decode line only: skip the matvec sweep and training step it carries")
    ap.add_argument("--no-vocab-parallel", action="store_true",
                    help="N > 1: skip the second measurement with the classifier split over all ranks")
    ap.add_argument("--positions", type=int, default=0,
                    help="decode positions per step (default: the model's seq_len, 1024)")
    ap.add_argument("--sweep", action="store_true",
                    help="isolated fp32 matvec sweep (one JSON line per W shape) instead of the decode")
    ap.add_argument("--sweep-shapes", default="", help="e.g. 32000x768,2048x768 (default: the 9 shapes)")
    ap.add_argument("--sweep-no-refs", action="store_true",
                    help="skip the sweep's L2 and launch-floor references (for per-shape ncu captures)")
    ap.add_argument("--train", action="store_true", help="stories15M training step (T=256) instead of the decode")
    ap.add_argument("--timeline", action="store_true",
                    help="phase timeline of the decode kernels over 16 positions (ptc_decoder_trace)")
    ap.add_argument("--timeline-start", type=int, default=504, help="first traced position (multiple of 8)")
    args = ap.parse_args()
    if args.sweep:
        return run_sweep(args)
    if args.timeline:
        return run_timeline(args)
    if args.train and args.impl != "reference" and int(os.environ.get("WORLD_SIZE", "1")) == 1:
        return run_train(args)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if args.impl == "reference":
        return run_reference(args, rank)
    if world > 1:   # torchrun: one rank per GPU
        from pitorch_b200 import pipeline_bench
        return pipeline_bench.run(args, rank, world)
    return run_single(args)


if __name__ == "__main__":
    sys.exit(main())
