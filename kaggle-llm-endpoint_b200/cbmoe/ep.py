"""Expert parallelism over the GPUs of one node (one process per GPU, torch.distributed for the plumbing).

    group = ExpertParallel()                                    # after torch.distributed.init_process_group
    local = group.pack_local(gate, up, down, shared)            # this rank's E/n experts (+ replicated shared)
    out = group.layer(local, x, idx, w, limit)                  # tokens of this rank -> bf16 [N_local, H]

The routed experts are sharded by id (rank r holds [r*E/n, (r+1)*E/n)); every rank keeps its tokens. One layer
call routes each (token, slot) to the rank holding its expert, exchanges rows with NCCL send/recv over NVLink,
runs the local experts on what it received, sends the outputs back and combines them with the shared expert
(include/cbmoe.h, cbmoe_ep_layer). The NCCL communicator is the library's own, bootstrapped through the
torch.distributed process group (rank 0's NCCL unique id is broadcast).
"""
import ctypes

import torch
import torch.distributed as dist

from ._lib import PATHS, Shared, check, lib, ptr, require_cuda, stream_handle
from .resident import _experts_struct


def agree_capacity(N_local, k, capacity=None, group=None):
    """Rows per peer that every rank of `group` uses: `capacity` when given (the caller keeps it equal on every
    rank), else the largest N_local * k over the ranks (all_reduce MAX). Ranks may hold different token counts; the
    peer transport addresses a peer's receive rows by the capacity, so it must be one value everywhere."""
    if capacity is not None:
        return max(1, int(capacity))
    dev = torch.device("cuda", torch.cuda.current_device()) if dist.get_backend(group) == "nccl" else torch.device("cpu")
    t = torch.tensor([N_local * k], dtype=torch.int64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return max(1, int(t.item()))


class ExpertParallel:
    """`transport`: "peer" (dispatch and return written straight into the other GPUs' memory over NVLink, CUDA IPC
    buffers set up on the first layer call, one process per GPU of one node, at most 8) or "nccl" (send/recv)."""

    def __init__(self, group=None, transport="peer"):
        self.group = group
        self.rank = dist.get_rank(group)
        self.nranks = dist.get_world_size(group)
        idbuf = torch.zeros(128, dtype=torch.uint8)
        if self.rank == 0:
            raw = (ctypes.c_uint8 * 128)()
            check(lib().cbmoe_ep_unique_id(raw), "cbmoe_ep_unique_id")
            idbuf.copy_(torch.tensor(list(raw), dtype=torch.uint8))
        dev = torch.device("cuda", torch.cuda.current_device())
        if dist.get_backend(group) == "nccl":
            t = idbuf.to(dev)
            dist.broadcast(t, src=0, group=group)
            idbuf = t.cpu()
        else:
            dist.broadcast(idbuf, src=0, group=group)
        raw = (ctypes.c_uint8 * 128)(*idbuf.tolist())
        comm = ctypes.c_void_p()
        check(lib().cbmoe_ep_comm_init(raw, self.nranks, self.rank, ctypes.byref(comm)), "cbmoe_ep_comm_init")
        self.comm = comm
        self._ws = None
        assert transport in ("peer", "nccl"), transport
        self.transport = transport if self.nranks <= 8 else "nccl"
        self._peer, self._peer_key = None, None

    def _peer_for(self, H, cap):
        """The peer-memory buffers for (H, cap); collective: every rank reaches it in the same layer call."""
        if self.transport != "peer":
            return None
        if self._peer_key != (H, cap):
            if self._peer is not None:
                torch.cuda.synchronize()
                check(lib().cbmoe_ep_peer_destroy(self._peer), "cbmoe_ep_peer_destroy")
                self._peer = None
            peer = ctypes.c_void_p()
            check(lib().cbmoe_ep_peer_init(self.comm, self.nranks, self.rank, H, cap, stream_handle(),
                                           ctypes.byref(peer)), "cbmoe_ep_peer_init")
            self._peer, self._peer_key = peer, (H, cap)
        return self._peer

    def close(self):
        if self._peer is not None:
            torch.cuda.synchronize()
            if dist.is_initialized():
                dist.barrier()   # every rank is past its last layer call before the buffers go
            check(lib().cbmoe_ep_peer_destroy(self._peer), "cbmoe_ep_peer_destroy")
            self._peer = None
        if self.comm:
            check(lib().cbmoe_ep_comm_destroy(self.comm), "cbmoe_ep_comm_destroy")
            self.comm = None

    def expert_range(self, E):
        assert E % self.nranks == 0, (E, self.nranks)
        n = E // self.nranks
        return self.rank * n, (self.rank + 1) * n

    def pack_local(self, gate, up, down, shared):
        """Full-layer CB3 tables (as for cbmoe.pack_layer) -> this rank's slice, packed; shared expert replicated."""
        from .resident import pack_layer
        E = gate[0].shape[0]
        a, b = self.expert_range(E)
        sl = lambda t: (t[0][a:b].contiguous(), t[1][a:b].contiguous())
        p = pack_layer(sl(gate), sl(up), sl(down), shared)
        p["E_total"] = E
        return p

    def layer(self, p, x, idx, w, limit, capacity=None, out=None, path="auto"):
        """x bf16 [N_local, H], idx int32 [N_local, k] (global expert ids), w fp32 [N_local, k] -> bf16 [N_local, H].
        `capacity` = rows per peer in each direction, the same on every rank (default: the largest N_local * k over
        the ranks, agreed by one small all-reduce per call; it never drops); `path` = kernels for the received rows
        ("auto", "decode", "grouped")."""
        require_cuda(x, idx, w)
        N, k = idx.shape
        cap = agree_capacity(N, k, capacity, self.group)
        ex = _experts_struct(p)
        s = p["shared"]
        sh = Shared(s["gate_up_q"].data_ptr(), s["gate_s"].data_ptr(), s["up_s"].data_ptr(), s["down_q"].data_ptr(),
                    s["down_s"].data_ptr(), s["scale_axis"])
        code = PATHS[path]
        nbytes = lib().cbmoe_ep_workspace_bytes(ex, N, k, self.nranks, cap, code)
        if self._ws is None or self._ws.numel() < nbytes:
            self._ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=x.device)
        if out is None:
            out = torch.empty((N, p["H"]), dtype=torch.bfloat16, device=x.device)
        xb = x.to(torch.bfloat16).contiguous()
        peer = self._peer_for(p["H"], cap)
        check(lib().cbmoe_ep_layer(self.comm, self.nranks, self.rank, ex, p["E_total"], sh, ptr(xb), N,
                                   ptr(idx.to(torch.int32).contiguous()), ptr(w.to(torch.float32).contiguous()), k,
                                   float(limit), cap, code, peer, ptr(out), ptr(self._ws), self._ws.numel(),
                                   stream_handle()),
              "cbmoe_ep_layer")
        return out
