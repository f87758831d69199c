"""Tensor parallelism over moe_inter (cbmoe/tp.py) on 2 CPU ranks with gloo: every rank takes its slice of the
GGUF-format tables with the same `shard` the GPU path uses, computes the oracle's composition on it, and the
all-reduce sum of the partial outputs must equal the whole layer (the reference's own sharding,
engine/glm53/resident.py:36-43, and psum, model.py:855). No GPU; the expert kernels on each slice are the ones
tests/test_gpu_iq.py checks."""
import os
import socket

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import gen
from oracle import iq as oiq

E, H, I, K_TOP = 4, 512, 512, 2
QT = {"gate_q": "IQ2_S", "up_q": "IQ2_S", "down_q": "IQ3_S"}


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tables(rng):
    return {"gate_q": oiq.random_blocks(rng, E * I * (H // 256), QT["gate_q"]).reshape(-1),
            "up_q": oiq.random_blocks(rng, E * I * (H // 256), QT["up_q"]).reshape(-1),
            "down_q": oiq.random_blocks(rng, E * H * (I // 256), QT["down_q"]).reshape(-1)}


def _dense(raw, rows, K):
    tabs = oiq.tables()
    return {k: oiq.experts_dense(raw[k], QT[k], E, r, c, tabs) for k, (r, c) in rows_k(rows, K).items()}


def rows_k(I_, H_):
    return {"gate_q": (I_, H_), "up_q": (I_, H_), "down_q": (H_, I_)}


def _worker(rank, nranks, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=nranks)
    try:
        from cbmoe.tp import shard
        rng = np.random.default_rng(5)                           # the same tables and tokens on every rank
        raw = _tables(rng)
        x = gen.activations(rng, 6, H).astype(np.float32)
        idx, w = gen.routing(rng, 6, E, K_TOP)
        g, u, d, Ir = shard(raw["gate_q"], raw["up_q"], raw["down_q"], QT, E, H, I, rank, nranks)
        tg, tu, td, _ = shard(*(torch.from_numpy(raw[k]) for k in ("gate_q", "up_q", "down_q")), QT, E, H, I, rank,
                              nranks)
        assert np.array_equal(tg.numpy(), g) and np.array_equal(tu.numpy(), u) and np.array_equal(td.numpy(), d)
        W = _dense({"gate_q": g, "up_q": u, "down_q": d}, Ir, H)
        part = oiq.decode_apply(x, idx, w, W["gate_q"], W["up_q"], W["down_q"], gen.LIMIT)
        t = torch.from_numpy(part)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        if rank == 0:
            Wf = _dense(raw, I, H)
            want = oiq.decode_apply(x, idx, w, Wf["gate_q"], Wf["up_q"], Wf["down_q"], gen.LIMIT)
            q.put(float(np.abs(t.numpy() - want).max() / np.abs(want).max()))
    finally:
        dist.destroy_process_group()


def test_tp_sum_of_slices_is_the_layer():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert q.get(timeout=5) < 1e-10


def test_shard_rejects_partial_blocks():
    from cbmoe.tp import shard
    raw = _tables(np.random.default_rng(1))
    try:
        shard(raw["gate_q"], raw["up_q"], raw["down_q"], QT, E, H, I, 0, 4)   # 512 / 4 = 128: not a whole block
    except AssertionError:
        return
    raise AssertionError("a slice of partial 256-weight blocks was accepted")
