"""Tensor parallelism over the experts' intermediate dimension (moe_inter): the reference's own multi-chip scheme
(engine/glm53/resident.py:36-43 shards the GGUF tables this way; model.py:855 sums the partials with psum), here
for the GGUF-format tables (cbmoe.iq) with one process per GPU and an all-reduce over torch.distributed (NCCL).

Every rank holds all E experts but only its slice of the I intermediate rows: gate/up rows [r I/n, (r+1) I/n) and
the matching input blocks of down (I/n must be a multiple of the 256-weight block: GLM-5.3-Flash's I = 2048 splits
into one block per rank at n = 8). Every rank runs all tokens' slots on its slice, y_r = sum_k w * (Wd[:, I_r]
swiglu(Wg[I_r] x, Wu[I_r] x)); SwiGLU acts per intermediate index, so the all-reduce sum of the y_r is the full
layer's routed output. Expert parallelism (cbmoe.ep) moves token rows instead of partial outputs; this scheme moves
N x H fp32 per layer whatever the routing, which suits small batches.
"""
import torch
import torch.distributed as dist

from . import iq

QK_K = 256


def shard(gate, up, down, qtypes, E, H, I, rank, nranks):
    """Raw GGUF tables (uint8, [E][rows][K/256][block bytes] flattened; torch or numpy) -> this rank's slices
    (gate_r, up_r, down_r) and I_r = I / nranks: gate/up rows [rank I_r, (rank+1) I_r), down input blocks
    [rank I_r / 256, (rank+1) I_r / 256)."""
    assert I % nranks == 0 and (I // nranks) % QK_K == 0, ("moe_inter slices must be whole 256-weight blocks", I,
                                                          nranks)
    Ir = I // nranks
    bg, bu, bd = (iq.block_bytes(qtypes[k]) for k in ("gate_q", "up_q", "down_q"))

    def rows(t, bb):
        t = t.reshape(E, I, (H // QK_K) * bb)[:, rank * Ir:(rank + 1) * Ir]
        return t.contiguous().reshape(-1) if hasattr(t, "contiguous") else t.copy().reshape(-1)

    d = down.reshape(E, H, I // QK_K, bd)[:, :, rank * Ir // QK_K:(rank + 1) * Ir // QK_K]
    d = d.contiguous().reshape(-1) if hasattr(d, "contiguous") else d.copy().reshape(-1)
    return rows(gate, bg), rows(up, bu), d, Ir


class TensorParallel:
    """One process per GPU, after torch.distributed.init_process_group: pack_local keeps this rank's moe_inter
    slice of a layer's GGUF tables, layer() returns the full routed output on every rank."""

    def __init__(self, group=None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.nranks = dist.get_world_size(group)

    def pack_local(self, gate, up, down, qtypes, E, H, I):
        g, u, d, Ir = shard(gate, up, down, qtypes, E, H, I, self.rank, self.nranks)
        return iq.pack_layer(g, u, d, qtypes, E, H, Ir)

    def layer(self, p_local, x, idx, w, limit):
        """x bf16 [N, H] (the same on every rank), idx int32 [N, k], w fp32 [N, k] -> fp32 [N, H] routed output."""
        y = iq.apply(p_local, x.to(torch.bfloat16).contiguous(), idx.to(torch.int32).contiguous(),
                     w.to(torch.float32).contiguous(), limit)
        dist.all_reduce(y, op=dist.ReduceOp.SUM, group=self.group)
        return y
