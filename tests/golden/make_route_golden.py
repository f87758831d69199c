"""Generate route.npz in this folder by EXECUTING the reference's router, moe_route (engine/glm53/model.py:798-808).

Run where the reference checkout (read-only) is available, naming its root in $CBMOE_REFERENCE:
    CBMOE_REFERENCE=<reference checkout> python tests/golden/make_route_golden.py
The function runs on make_golden.py's NumPy stand-in for jax, plus `lax.top_k` as a stable descending sort (the
largest values first, the lower index first among equal ones, as XLA's top_k orders them) and `jax.nn.sigmoid`.
Inputs: bf16-exact x [16, 256] and router weights [256, 160], a bias [160] (the e_score_correction_bias role),
k = 8, both settings of norm_topk, scaling 2.5; plus rows whose choice values tie, to pin the tie order.
"""
import os
import sys
import types

import numpy as np
import ml_dtypes

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import make_golden as mg  # noqa: E402


def top_k(a, k):
    a = np.asarray(a)
    order = np.argsort(-a, axis=-1, kind="stable")[..., :k]
    return mg.J(np.take_along_axis(a, order, -1)), mg.J(order.astype(np.int32))


def main():
    assert os.path.isdir(mg.ENGINE), f"reference engine not found at {mg.ENGINE}"
    lax = types.SimpleNamespace(top_k=top_k)
    jax = types.SimpleNamespace(nn=types.SimpleNamespace(
        one_hot=mg.jax.nn.one_hot,
        sigmoid=lambda x: mg.J((1.0 / (1.0 + np.exp(-np.asarray(x, np.float32)))).astype(np.float32))))
    moe_route = mg.ref_function("model.py", "moe_route", extra={"lax": lax, "jax": jax, "Cfg": object})
    rng = np.random.default_rng(31)
    N, D, E, k = 16, 256, 160, 8
    x = rng.standard_normal((N, D)).astype(ml_dtypes.bfloat16)
    W = (rng.standard_normal((D, E)) * 0.05).astype(ml_dtypes.bfloat16)
    b = (rng.standard_normal(E) * 0.1).astype(np.float32)
    x[3] = 0.0                                  # every logit 0: the choice is the bias alone
    b_tie = b.copy()
    b_tie[[7, 9, 40]] = 5.0                     # equal choices for every row of the tie case
    out = {"x": x.view(np.uint16), "W": W.view(np.uint16), "b": b, "b_tie": b_tie, "k": k, "scaling": 2.5}
    for norm in (True, False):
        for name, bias in (("", b), ("_tie", b_tie)):
            p = {"router_w": mg.J(W.astype(np.float32)), "router_bias": mg.J(bias)}
            cfg = types.SimpleNamespace(topk=k, norm_topk=norm, scaling=np.float32(2.5))
            idx, w = moe_route(p, mg.J(x.astype(np.float32)), cfg)
            out[f"idx{name}_{int(norm)}"] = np.asarray(idx)
            out[f"w{name}_{int(norm)}"] = np.asarray(w, np.float32)
    np.savez_compressed(os.path.join(HERE, "route.npz"), **out)
    print("route.npz written to", HERE)


if __name__ == "__main__":
    main()
