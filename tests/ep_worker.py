"""One rank of the 2-GPU expert-parallel parity check (launched by tests/test_gpu_ep.py through torchrun).

Every rank builds the same small layer and tokens from one seed, keeps its half of the experts and of the tokens,
runs cbmoe_ep_layer over both transports (peer memory over NVLink, NCCL send/recv) and both kernel paths for the
received rows, and rank 0 compares the gathered outputs with the CPU oracle's single-process layer. Exit status 0 =
parity holds."""
import datetime
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "kaggle-llm-endpoint_b200"), os.path.join(ROOT, "tests")):
    sys.path.insert(0, p)

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from helpers import shared_to_gpu, t_bf16, table_to_gpu  # noqa: E402
from oracle import gen, moe  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
    dev = torch.device("cuda", torch.cuda.current_device())
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    import cbmoe
    from cbmoe.ep import ExpertParallel
    ok = True
    groups = []
    cases = [(16, None, "auto"), (64, None, "auto"), (64, None, "grouped"), (6, 3, "auto")]
    try:
        E, H, I, k = 8, 512, 256, 4
        L = gen.moe_layer(np.random.default_rng(123), E, H, I)
        for transport in ("peer", "nccl"):
            group = ExpertParallel(transport=transport)
            groups.append(group)
            p = group.pack_local(table_to_gpu(L["gate"]), table_to_gpu(L["up"]), table_to_gpu(L["down"]),
                                 shared_to_gpu(L["shared"]))
            rng = np.random.default_rng(7)
            for case, (N_total, cap, path) in enumerate(cases):
                x = gen.activations(rng, N_total, H)
                idx, w = gen.routing(rng, N_total, E, k)
                per = N_total // world
                sl = slice(rank * per, (rank + 1) * per)
                out = group.layer(p, t_bf16(x[sl]), torch.from_numpy(idx[sl]).cuda(), torch.from_numpy(w[sl]).cuda(),
                                  gen.LIMIT, capacity=cap, path=path)
                torch.cuda.synchronize()
                errs = cbmoe.device_errors(clear=True)
                outs = [torch.empty_like(out) for _ in range(world)]
                dist.all_gather(outs, out)
                if rank == 0:
                    got = torch.cat(outs).float().cpu().numpy()
                    want = moe.moe_layer(x[:per * world].astype(np.float32), idx[:per * world], w[:per * world],
                                         L["gate"], L["up"], L["down"], L["shared"], gen.LIMIT)
                    err = moe.max_rel_err(got, want)
                    print(f"{transport} case {case}: N={N_total} cap={cap} path={path} max rel err {err:.2e} "
                          f"device errors {errs}", flush=True)
                    if cap is None:
                        ok = ok and err < 1e-2 and errs == 0
                    else:   # capacity below the slots: drops are flagged, never a fault
                        ok = ok and (bool(errs & 4) or err < 1e-2) and not (errs & 1)
    finally:
        for g in groups:
            g.close()
        flag = torch.tensor([1 if ok else 0], device=dev)
        dist.broadcast(flag, src=0)
        dist.destroy_process_group()
    sys.exit(0 if int(flag.item()) == 1 else 1)


if __name__ == "__main__":
    main()
