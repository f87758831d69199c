"""The expert-parallel protocol on 2 CPU ranks with gloo: dispatch rows to the ranks holding their experts, compute
there, return, combine; the result must equal the single-process layer. No GPU (the CUDA kernels run the same
bookkeeping; tests/test_gpu_ep.py runs them on 2 GPUs)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import ep, gen, moe

E, H, I, K_TOP = 8, 256, 256, 4


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _all_to_all(send, nranks, cap):
    """all-to-all by all_gather (gloo has no all_to_all): block p of every rank's buffer goes to rank p."""
    rank = dist.get_rank()
    t = torch.from_numpy(np.ascontiguousarray(send))
    bufs = [torch.zeros_like(t) for _ in range(nranks)]
    dist.all_gather(bufs, t)
    return torch.cat([b[rank * cap:(rank + 1) * cap] for b in bufs]).numpy()


def _worker(rank, nranks, port, cap, result_q, counts=None):
    """`counts`: tokens per rank (default: 12 split evenly); `cap` None = the capacity cbmoe.ep.agree_capacity
    agrees on (the largest N_local * k over the ranks), which is what the library's layer call uses."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=nranks)
    try:
        rng = np.random.default_rng(0)                       # same tables and tokens on every rank
        L = gen.moe_layer(rng, E, H, I)
        counts = counts or [12 // nranks] * nranks
        N_total = sum(counts)
        x = gen.activations(rng, N_total, H).astype(np.float32)
        idx, w = gen.routing(rng, N_total, E, K_TOP)
        per, a0 = counts[rank], sum(counts[:rank])
        xs, ids, ws = x[a0:a0 + per], idx[a0:a0 + per], w[a0:a0 + per]
        if cap is None:
            from cbmoe.ep import agree_capacity
            cap = agree_capacity(per, K_TOP)
            assert cap == max(counts) * K_TOP, (cap, counts)
        send_eid, slot_pos, dropped = ep.route(ids, E, nranks, cap)
        send_x = np.zeros((nranks * cap, H), np.float32)
        for s, pos in enumerate(slot_pos):
            if pos >= 0:
                send_x[pos] = xs[s // K_TOP]
        rx = _all_to_all(send_x, nranks, cap)
        re = _all_to_all(send_eid, nranks, cap)
        E_loc = E // nranks
        a = rank * E_loc
        local = {k_: (L[k_][0][a:a + E_loc], L[k_][1][a:a + E_loc]) for k_ in ("gate", "up", "down")}
        y = np.zeros((nranks * cap, H), np.float32)
        for r in range(nranks * cap):
            if re[r] >= 0:
                y[r] = moe.decode_apply(rx[r:r + 1], np.array([[re[r]]]), np.ones((1, 1), np.float32),
                                        local["gate"], local["up"], local["down"], gen.LIMIT)[0]
        yb = _all_to_all(y, nranks, cap)
        out = moe.shared_mlp(xs, *L["shared"], gen.LIMIT)
        for t in range(per):
            for j in range(K_TOP):
                pos = slot_pos[t * K_TOP + j]
                if pos >= 0:
                    out[t] += ws[t, j] * yb[pos]
        want = moe.moe_layer(xs, ids, ws, L["gate"], L["up"], L["down"], L["shared"], gen.LIMIT)
        result_q.put((rank, moe.max_rel_err(out, want), dropped))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("cap", [24, 5])
def test_ep_protocol_two_ranks(cap):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, cap, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
        assert p.exitcode == 0, "rank failed"
    res = [q.get(timeout=10) for _ in procs]
    for rank, err, dropped in res:
        if dropped == 0:
            assert err < 1e-6, (rank, err)
        else:                                           # a too-small capacity drops slots (flagged, not fatal)
            assert cap == 5 and err > 0


def test_ep_protocol_four_ranks():
    """The same protocol over 4 ranks (2 experts and 3 tokens per rank): the bookkeeping the 4- and 8-GPU runs use."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 4, port, 12, q)) for r in range(4)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
        assert p.exitcode == 0, "rank failed"
    res = [q.get(timeout=10) for _ in procs]
    assert sorted(r for r, _, _ in res) == [0, 1, 2, 3]
    for rank, err, dropped in res:
        assert dropped == 0 and err < 1e-6, (rank, err, dropped)


def test_ep_unequal_token_counts_agree_on_capacity():
    """Ranks holding different token counts (3 and 7): the default capacity is agreed by an all-reduce MAX
    (cbmoe.ep.agree_capacity), so both ranks address each other's receive rows alike and nothing drops."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, None, q, [3, 7])) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
        assert p.exitcode == 0, "rank failed"
    res = [q.get(timeout=10) for _ in procs]
    for rank, err, dropped in res:
        assert dropped == 0 and err < 1e-6, (rank, err, dropped)
