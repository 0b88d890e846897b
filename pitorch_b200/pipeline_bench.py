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

Batch-1 decode cannot overlap positions (each token depends on the previous
argmax), so the pipeline splits weights across GPUs without adding
throughput; the scaling is reported as measured ("weak": every N runs the
same full decode).
"""
import json
import os
import time

import numpy as np


def run(args, rank, world):
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
    pipe = api.Pipeline(blob, rank, world, device=local)
    del blob
    pc = pipe.ctx.ptc_ctx()
    timer = L.ptc_timer_create(pc)

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
    value = seq / (ms_step / 1000.0)

    pipe.ctx.ctx.sync_logits = 0
    t0 = time.perf_counter()
    L.ptc_timer_start(timer)
    host_toks = pipe.decode_greedy(prompt, seq)
    L.ptc_timer_stop(timer)
    e2e_ms = pipe.max_over_ranks(L.ptc_timer_ms(timer))
    e2e_wall = pipe.max_over_ranks(1000 * (time.perf_counter() - t0))
    same = True
    if pipe.is_head:
        same = bool(np.array_equal(toks, host_toks))
    same = pipe.max_over_ranks(0.0 if same else 1.0) == 0.0

    dim, hidden, nl, nh, nkv, V, _ = cfg
    n_layer_ranks = world - 1
    launches = seq * (5 * nl + 2 + 2 * n_layer_ranks)
    if rank == 0:
        line = {
            "metric": "batch-1 decode tokens/s (stories110M shape)", "value": value, "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded N(0,0.02) fp32 weights, seeded 8-token prompt)",
            "config": {"workload": f"{model} batch-1 greedy decode, {seq} positions per step, "
                                   f"layer pipeline over {world} GPUs",
                       "model": model, "global_batch": 1, "seq_len": seq,
                       "parallelism": f"pp{world} (last rank: embedding + classifier)",
                       "l2_policy": "weights > L2 per rank at N<=2; shards of ~57-113 MB at N>=4"},
            "e2e": {"value": seq / (e2e_ms / 1000.0), "unit": "tokens/s",
                    "api": "pt_dist_forward_step per position",
                    "h2d_bytes_per_step": 8 * seq, "d2h_bytes_per_step": 4 * seq,
                    "wall_ms_per_step": e2e_wall, "token_stream_equals_device_loop": same},
            "gpu_launches": args.steps * launches,
        }
        print(json.dumps(line), flush=True)
    L.ptc_timer_destroy(timer)
    pipe.close()
    return 0
