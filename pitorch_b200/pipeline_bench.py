"""bench.py at N > 1: the stories110M decode as a layer pipeline over N GPUs.

Launched by torchrun (one process per GPU, RANK / WORLD_SIZE / LOCAL_RANK /
MASTER_ADDR / MASTER_PORT in the environment). Each rank cuts its SHRD shard
out of the seeded synthetic model with the reference's layer assignment
(tools/shard_weights.py:49-66: the last rank holds embedding + classifier,
the others split the 12 layers), joins the ring (NCCL over NVLink) and runs

  value  pt_dist_generate_greedy: the whole 1024-position greedy decode
         enqueued on every rank with no host round trip per token; timed with
         CUDA events on each rank's stream, max over ranks.
  e2e    pt_dist_forward_step per position (host token in, host token out
         on the head rank), the reference's per-token API.

After those, the same two measurements with the vocab-parallel classifier
(pt_dist_vocab_parallel: every rank computes 1/N of the classifier rows and
the argmax is combined on the GPUs; a departure from the reference's ring
topology, reported separately under "vocab_parallel").

Batch-1 decode cannot overlap positions (each token depends on the previous
argmax), so the pipeline splits weights across GPUs without adding
throughput; every N runs the same full decode (fixed total work: "strong"
scaling), reported as measured against the serial roofline (each token's
bytes stream once, stage after stage).
"""
import json
import os
import sys
import time

import numpy as np


def run(args, rank, world):
    # NCCL's communicator set-up lines ("... nRanks N ...") show how many
    # ranks the run had; only the set-up subsystem, printed before the
    # bench's JSON line
    os.environ["NCCL_DEBUG"] = "INFO"
    os.environ["NCCL_DEBUG_SUBSYS"] = "INIT"
    os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")   # stdout carries only the JSON line
    import ctypes as C

    import pitorch_b200
    from pitorch_b200 import api, synth

    L = pitorch_b200.lib()
    local = int(os.environ.get("LOCAL_RANK", rank))
    model = "stories110M"
    cfg = synth.CONFIGS[model]
    seq = cfg[6] if not args.positions else min(args.positions, cfg[6])
    blob = synth.make_blob(cfg)
    prompt = synth.make_prompt(cfg[5], 8)
    import bench as _bench   # the single-GPU bench's clock sampler and byte model
    pipe = api.Pipeline(blob, rank, world, device=local)
    del blob
    # the communicator's own rank count, as NCCL reports it
    print(f"pitorch_b200: rank {rank}: NCCL communicator with {L.pt_dist_comm_size(C.byref(pipe.dist))} ranks, "
          f"hop transport {'NVLink peer stores' if L.pt_dist_transport(C.byref(pipe.dist)) == 1 else 'NCCL'}",
          file=sys.stderr, flush=True)
    pc = pipe.ctx.ptc_ctx()
    timer = L.ptc_timer_create(pc)

    def measure():
        """Device-loop decodes (timed, max over ranks), one host-driven decode
        (e2e), and the head's stream against the reference fixture."""
        for _ in range(args.warmup):
            pipe.generate_greedy(prompt, seq)
        ms = 0.0
        toks = None
        for _ in range(args.steps):
            L.ptc_sync(pc)
            L.ptc_timer_start(timer)
            toks = pipe.generate_greedy(prompt, seq)
            L.ptc_timer_stop(timer)
            ms += L.ptc_timer_ms(timer)
        ms_step = pipe.max_over_ranks(ms / args.steps)
        pipe.ctx.ctx.sync_logits = 0
        t0 = time.perf_counter()
        L.ptc_timer_start(timer)
        host_toks = pipe.decode_greedy(prompt, seq)
        L.ptc_timer_stop(timer)
        e2e_ms = pipe.max_over_ranks(L.ptc_timer_ms(timer))
        e2e_wall = pipe.max_over_ranks(1000 * (time.perf_counter() - t0))
        same = bool(np.array_equal(toks, host_toks)) if pipe.is_head else True
        same = pipe.max_over_ranks(0.0 if same else 1.0) == 0.0
        par = _bench.stream_parity(toks, seq) if pipe.is_head else {}
        matched = pipe.max_over_ranks(float(par.get("matched_positions", 0)))
        par_ok = pipe.max_over_ranks(1.0 if par.get("equal_up_to_first_near_tie") else 0.0) == 1.0
        return ms_step, e2e_ms, e2e_wall, same, matched, par_ok

    with _bench.ClockSampler(local) as clk:
        ms_step, e2e_ms, e2e_wall, same, matched, par_ok = measure()
    value = seq / (ms_step / 1000.0)

    dim, hidden, nl, nh, nkv, V, _ = cfg
    # kernels per position over all ranks: the layer kernels of every layer
    # (the same count per layer on every rank), the head rank's embedding and
    # classifier; NCCL's own send/recv kernels are not counted
    dec = pipe.ctx.ptc_decoder()
    n_local = int(pipe.ctx.cfg.n_layers)
    per_layer = (L.ptc_decoder_launches_per_step(dec) - (1 if pipe.is_head else 0)) // n_local if n_local else 0
    per_layer = int(pipe.max_over_ranks(float(per_layer)))
    p2p = L.pt_dist_transport(C.byref(pipe.dist)) == 1
    # per position: the layer kernels, the head's classifier and, with the
    # NVLink hops, one send kernel per layer rank (the receives and the next
    # embedding row are inside the decode kernels); with NCCL hops the head's
    # embedding kernel (NCCL's own kernels are not counted)
    launches = seq * (per_layer * nl + 1 + ((world - 1) if p2p else 1))
    hbm, src = _bench.peaks()
    mean_bytes = float(np.mean([_bench.decode_bytes_per_token(cfg, p) for p in range(seq)]))
    step_gbs = mean_bytes * seq / (ms_step / 1000.0) / 1e9
    line = None
    if rank == 0:
        line = {
            "metric": "batch-1 decode tokens/s (stories110M shape)", "value": value, "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded N(0,0.02) fp32 weights, seeded 8-token prompt)",
            "config": {"workload": f"{model} batch-1 greedy decode, {seq} positions per step, "
                                   f"layer pipeline over {world} GPUs",
                       "model": model, "global_batch": 1, "seq_len": seq,
                       "parallelism": f"pp{world} (last rank: embedding + classifier)",
                       "hop_transport": "peer stores over NVLink (CUDA IPC mailboxes)" if p2p
                                        else "NCCL send/recv",
                       "l2_policy": "weights > L2 per rank at N<=2; shards of ~57-113 MB at N>=4"},
            "e2e": {"value": seq / (e2e_ms / 1000.0), "unit": "tokens/s",
                    "api": "pt_dist_forward_step per position",
                    "h2d_bytes_per_step": 8 * seq, "d2h_bytes_per_step": 4 * seq,
                    "wall_ms_per_step": e2e_wall, "token_stream_equals_device_loop": same},
            "gpu_launches": args.steps * launches,
            # per-kernel rooflines are measured by the N = 1 line (the same
            # kernels); across stages the decode is one serial stream
            "roofline": {"kernel": "whole decode step, serial over the pipeline stages", "bound": "hbm",
                         "achieved": step_gbs, "peak": hbm, "unit": "GB/s", "frac": step_gbs / hbm,
                         "traffic": None, "peak_source": f"{src} hbm_gbs"},
            "step_roofline": {"bytes_per_token": mean_bytes, "achieved": step_gbs, "peak": hbm, "unit": "GB/s",
                              "frac": step_gbs / hbm, "peak_source": f"{src} hbm_gbs",
                              "basis": "serial: each token's weights and KV stream once, stage after stage"},
            "clocks": clk.summary(),
            "parity": {"fixture": "tests/golden/decode_stories110M_long.npz (reference host C)",
                       "compared": "the head rank's token stream of the last timed step",
                       "matched_positions": int(matched), "equal_up_to_first_near_tie": bool(par_ok)},
        }
    # the same decode with the classifier split over all ranks
    vp = None
    vp_ok = False
    if not getattr(args, "no_vocab_parallel", False):
        try:   # collective: every rank gets the same answer
            pipe.vocab_parallel()
            vp_ok = True
        except RuntimeError as e:
            vp = {"unavailable": str(e)}
    if vp_ok:
        try:   # a failed decode fails on every rank (its hops time out), before any collective
            with _bench.ClockSampler(local) as vclk:
                v_ms, v_e2e_ms, v_wall, v_same, v_matched, v_ok = measure()
        except RuntimeError as e:
            vp_ok, vp = False, {"error": str(e)}
    if vp_ok:
        v_gbs = mean_bytes * seq / (v_ms / 1000.0) / 1e9
        vp = {"value": seq / (v_ms / 1000.0), "unit": "tokens/s", "ms_per_step": v_ms,
              "parallelism": f"pp{world}, classifier rows split over all {world} ranks, argmax combined on the GPUs",
              "e2e": {"value": seq / (v_e2e_ms / 1000.0), "unit": "tokens/s",
                      "api": "pt_dist_forward_step per position", "wall_ms_per_step": v_wall,
                      "token_stream_equals_device_loop": v_same},
              "gpu_launches": args.steps * seq * (per_layer * nl + world + (world - 1)),
              "step_roofline": {"achieved": v_gbs, "peak": hbm, "unit": "GB/s", "frac": v_gbs / hbm},
              "clocks": vclk.summary(),
              "parity": {"fixture": "tests/golden/decode_stories110M_long.npz (reference host C)",
                         "matched_positions": int(v_matched), "equal_up_to_first_near_tie": bool(v_ok)}}
    if rank == 0:
        line["vocab_parallel"] = vp
        print(json.dumps(line), flush=True)
    L.ptc_timer_destroy(timer)
    pipe.close()
    return 0
