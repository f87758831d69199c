"""Expert-parallel protocol of cbmoe_ep_layer restated on the CPU (test infrastructure, see oracle/__init__.py).

The reference has no expert parallelism (it shards moe_inter and psums, launcher/glm53-flash/engine/glm53/
engine.py:129-176, model.py:855); what is pinned is that the EP layer equals the single-GPU layer
(model.py:840-856). This module restates the dispatch bookkeeping the CUDA route kernel performs, so a multi-rank
CPU test can run the whole protocol with gloo collectives:
  destination rank of slot (t, j) = idx[t, j] // (E / n); position = stable rank among this rank's slots for that
  destination (slot order t*k + j); slots past `capacity` are dropped; send row d*cap + pos carries token t.
"""
import numpy as np


def route(idx, E_total, nranks, cap):
    """idx int [N, k] -> (send_eid int32 [n*cap] local expert id or -1, slot_pos int32 [N*k] row or -1, dropped)."""
    E_loc = E_total // nranks
    flat = np.asarray(idx).reshape(-1)
    send_eid = np.full(nranks * cap, -1, np.int32)
    slot_pos = np.full(flat.size, -1, np.int32)
    fill = np.zeros(nranks, np.int64)
    dropped = 0
    for s, e in enumerate(flat):
        if e < 0:
            continue
        d = int(e) // E_loc
        if fill[d] < cap:
            pos = d * cap + fill[d]
            send_eid[pos] = int(e) - d * E_loc
            slot_pos[s] = pos
        else:
            dropped += 1
        fill[d] += 1
    return send_eid, slot_pos, dropped
