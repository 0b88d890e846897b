"""Host-side logic of the layer pipeline, on CPU only (no GPU calls).

* The shard cutter reproduces the reference's layer assignment
  (tools/shard_weights.py:49-66) and the SHRD layout that pt_shard.c reads
  (pitorch/model/pt_shard.c:15-130).
* The ring rendezvous that hands the NCCL id from rank 0 to the others works
  across two processes, and a rank whose peer never shows up gets -1 after
  its timeout instead of hanging (the reference's recv_raw contract,
  pitorch/dist/transport/pt_link_gpio.c:134-136).
"""
import ctypes as C
import multiprocessing as mp
import socket

import numpy as np
import pytest

from pitorch_b200 import api, synth


def reference_assignment(n_layers, world):
    # tools/shard_weights.py:49-66, restated
    if world == 1:
        return [(0, n_layers, 1, 1)]
    compute = world - 1
    base, extra = divmod(n_layers, compute)
    out, off = [], 0
    for r in range(compute):
        cnt = base + (1 if r < extra else 0)
        out.append((off, off + cnt, 0, 0))
        off += cnt
    out.append((n_layers, n_layers, 1, 1))
    return out


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_shard_layout_matches_reference(world):
    import pitorch_b200
    L = pitorch_b200.lib()
    cfg = synth.CONFIGS["tiny"] if world <= 3 else (64, 176, 7, 4, 4, 1024, 64)
    full = synth.make_blob(cfg)
    dim, hidden, nl, nh, nkv, V, seq = cfg
    kvd = nkv * (dim // nh)
    f = np.frombuffer(full, np.float32)
    # tensor offsets (in floats) in the full image, after the 7-int header
    sizes = [("emb", V * dim), ("rms_att", nl * dim), ("wq", nl * dim * dim), ("wk", nl * kvd * dim),
             ("wv", nl * kvd * dim), ("wo", nl * dim * dim), ("rms_ffn", nl * dim), ("w1", nl * hidden * dim),
             ("w2", nl * dim * hidden), ("w3", nl * hidden * dim), ("rms_final", dim)]
    off, full_t = 7, {}
    for name, n in sizes:
        full_t[name] = f[off:off + n]
        off += n
    per_layer = {"rms_att": dim, "wq": dim * dim, "wk": kvd * dim, "wv": kvd * dim, "wo": dim * dim,
                 "rms_ffn": dim, "w1": hidden * dim, "w2": dim * hidden, "w3": hidden * dim}
    for rank, (l0, l1, emb, head) in enumerate(reference_assignment(nl, world)):
        shard = api.make_shard(full, rank, world)
        buf = C.create_string_buffer(shard, len(shard))
        gcfg, info = api.pt_config_t(), api.pt_shard_info_t()
        L.pt_load_shard_header(C.byref(gcfg), C.byref(info), C.cast(buf, C.c_void_p))
        assert (info.l_start, info.l_end, info.has_embed, info.has_head) == (l0, l1, emb, head)
        assert (info.rank, info.world_size, info.n_local) == (rank, world, l1 - l0)
        assert L.pt_shard_file_size(C.cast(buf, C.c_void_p)) == len(shard)
        assert gcfg.n_layers == nl and gcfg.dim == dim
        s = np.frombuffer(shard, np.float32)
        p = 14   # 56-byte header
        if emb:
            assert np.array_equal(s[p:p + V * dim], full_t["emb"])
            p += V * dim
        for name in ("rms_att", "wq", "wk", "wv", "wo", "rms_ffn", "w1", "w2", "w3"):
            k = per_layer[name]
            want = full_t[name][l0 * k:l1 * k]
            assert np.array_equal(s[p:p + len(want)], want), (rank, name)
            p += len(want)
        if head:
            assert np.array_equal(s[p:p + dim], full_t["rms_final"])


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rdv_worker(rank, world, port, q):
    import pitorch_b200
    L = pitorch_b200.lib()
    blob = (C.c_ubyte * 128)()
    if rank == 0:
        for i in range(128):
            blob[i] = (i * 7 + 3) & 0xFF
    rc = L.pt_dist_rendezvous(rank, world, b"127.0.0.1", port, 20000, blob)
    q.put((rank, rc, bytes(blob)))


def test_rendezvous_two_processes():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_rdv_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    got = dict((r, (rc, b)) for r, rc, b in (q.get(timeout=60) for _ in range(2)))
    for p in ps:
        p.join(timeout=30)
    want = bytes(((i * 7 + 3) & 0xFF) for i in range(128))
    assert got[0][0] == 0 and got[1][0] == 0
    assert got[1][1] == want


def test_rendezvous_times_out_without_peer():
    import pitorch_b200
    L = pitorch_b200.lib()
    blob = (C.c_ubyte * 128)()
    # rank 1 of 2: nobody listens on this port -> -1 after the timeout
    assert L.pt_dist_rendezvous(1, 2, b"127.0.0.1", _free_port(), 500, blob) == -1
    # rank 0 of 2 whose peer never connects -> -1 after the timeout
    assert L.pt_dist_rendezvous(0, 2, b"127.0.0.1", _free_port(), 500, blob) == -1
