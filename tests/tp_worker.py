"""One rank of the 2-GPU tensor-parallel parity check (launched by tests/test_gpu_tp.py through torchrun).

Every rank builds the same GGUF-format layer (IQ2_S gate/up, IQ3_S down) and tokens from one seed, keeps its
moe_inter slice (cbmoe.tp.TensorParallel), computes all slots on it and all-reduces the partial outputs; rank 0
compares the result with the CPU oracle's whole layer. Exit status 0 = parity holds on every rank."""
import datetime
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "kaggle-llm-endpoint_b200"), os.path.join(ROOT, "tests")):
    sys.path.insert(0, p)

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from oracle import gen  # noqa: E402
from oracle import iq as oiq  # noqa: E402

E, H, I, K_TOP = 4, 512, 512, 2
QT = {"gate_q": "IQ2_S", "up_q": "IQ2_S", "down_q": "IQ3_S"}
SHAPES = {"gate_q": (I, H), "up_q": (I, H), "down_q": (H, I)}


def main():
    rank = int(os.environ["RANK"])
    torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
    dev = torch.device("cuda", torch.cuda.current_device())
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    ok = True
    try:
        from cbmoe.tp import TensorParallel
        rng = np.random.default_rng(5)
        raw = {key: oiq.random_blocks(rng, E * rows * (K // 256), QT[key]).reshape(-1)
               for key, (rows, K) in SHAPES.items()}
        x = gen.activations(rng, 6, H)
        idx, w = gen.routing(rng, 6, E, K_TOP)
        tp = TensorParallel()
        p = tp.pack_local(*(torch.from_numpy(raw[key]).to(dev) for key in ("gate_q", "up_q", "down_q")), QT, E, H,
                          I)
        y = tp.layer(p, torch.from_numpy(x.view(np.uint16).copy()).to(dev).view(torch.bfloat16),
                     torch.from_numpy(idx).to(dev), torch.from_numpy(w).to(dev), gen.LIMIT)
        got = y.cpu().numpy()
        tabs = oiq.tables()
        W = {key: oiq.experts_dense(raw[key], QT[key], E, rows, K, tabs) for key, (rows, K) in SHAPES.items()}
        want = oiq.decode_apply(x.astype(np.float32), idx, w, W["gate_q"], W["up_q"], W["down_q"], gen.LIMIT)
        err = float(np.abs(got - want).max() / np.abs(want).max())
        print(f"rank {rank}: tensor-parallel layer max rel err {err:.2e}", flush=True)
        ok = err < 2e-3
    except Exception as e:  # report and fail this rank; the flag below fails all of them
        print(f"rank {rank}: {type(e).__name__}: {e}", flush=True)
        ok = False
    flag = torch.tensor([1 if ok else 0], device=dev)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    dist.destroy_process_group()
    sys.exit(0 if int(flag.item()) == 1 else 1)


if __name__ == "__main__":
    main()
