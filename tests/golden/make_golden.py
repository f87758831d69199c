"""Generate the golden fixtures in this folder by EXECUTING the reference's own functions.

Run where the reference checkout (read-only) is available, naming its root in $CBMOE_REFERENCE:
    CBMOE_REFERENCE=<reference checkout> python tests/golden/make_golden.py
Nothing at test time reads the reference; the tests only read the .npz written here.

JAX is not installed here, so the reference functions run on a NumPy-backed stand-in for the few `jax`,
`jax.numpy`, `lax` and `jax.nn` calls they make (argsort/cumsum/one_hot/.at[].set/where/take/einsum/...). The source
of each function is taken verbatim from the reference file with `ast` at generation time and executed in a
namespace whose `jnp`/`jax`/`lax` are that stand-in; no reference source is copied into this repository.

Executed reference functions (paths relative to launcher/glm53-flash/engine/glm53/):
  pallas_moe.py  ragged_plan                          -> plan_*.npz
  model.py       silu, swiglu_clamped                 -> swiglu.npz
  quant8.py      quantize_array, is_q8, dequant_tree  -> quant8.npz
  resident.py    ResidentFetch._apply_kernel          -> decode_compose.npz  (kernel calls stubbed, see below)
  resident.py    ResidentFetch._apply_ragged_kernel   -> ragged_compose_*.npz
  engine.py      Engine._logits_local (int8 columns) -> logits_q8.npz (the int8 lm_head: scale after the dot)
For the two compositions the Pallas kernels (`moe_matvec`, `moe_ragged_gateup/down`) and the GGUF plane helpers are
replaced by CB3 stand-ins (exact dequant + f32 contraction, bf16 rounding where the kernels round); what the fixture
pins is the reference's composition around them: slot repetition, swiglu, the weighted combine, the ragged plan,
the padded-row gather and the two combine modes.
"""
import ast
import os
import sys
import textwrap
import types

import numpy as np
import ml_dtypes

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
from oracle import cb3  # noqa: E402  (only for generating packed CB3 inputs)

REF = os.environ.get("CBMOE_REFERENCE", "")
ENGINE = os.path.join(REF, "launcher", "glm53-flash", "engine", "glm53")


# ------------------------------------------------------------------------------------------ NumPy stand-in for jax
class JArr(np.ndarray):
    """ndarray with jax's functional `.at[idx].set(v)` update."""

    @property
    def at(self):
        arr = self

        class _Idx:
            def __getitem__(self, key):
                class _Upd:
                    def set(self, v):
                        out = np.array(arr, copy=True).view(JArr)
                        out[key] = v
                        return out
                return _Upd()
        return _Idx()


def J(a):
    return np.asarray(a).view(JArr)


def _wrap(fn):
    def f(*a, **kw):
        r = fn(*a, **kw)
        return J(r) if isinstance(r, np.ndarray) else r
    return f


def _dot(a, b, preferred_element_type=None, precision=None):
    r = np.asarray(a, np.float32) @ np.asarray(b, np.float32)
    return J(r.astype(preferred_element_type or np.result_type(a, b)))


def _einsum(spec, *ops, precision=None, preferred_element_type=None):
    return J(np.einsum(spec, *[np.asarray(o, np.float32) for o in ops]))


jnp = types.SimpleNamespace(
    asarray=_wrap(np.asarray), array=_wrap(np.array), zeros=_wrap(np.zeros), full=_wrap(np.full),
    arange=_wrap(np.arange), argsort=_wrap(lambda a, axis=-1: np.argsort(a, axis=axis, kind="stable")),
    sum=_wrap(np.sum), cumsum=_wrap(np.cumsum), minimum=_wrap(np.minimum), maximum=_wrap(np.maximum),
    where=_wrap(np.where), take=_wrap(np.take), repeat=_wrap(np.repeat), clip=_wrap(np.clip), round=_wrap(np.round),
    abs=_wrap(np.abs), max=_wrap(np.max), concatenate=_wrap(np.concatenate), einsum=_einsum, dot=_dot,
    float32=np.float32, int32=np.int32, int8=np.int8, uint32=np.uint32, bfloat16=ml_dtypes.bfloat16)
jax = types.SimpleNamespace(nn=types.SimpleNamespace(
    one_hot=lambda x, n, dtype=np.float32: J((np.asarray(x)[..., None] == np.arange(n)).astype(dtype)),
    sigmoid=lambda x: J(1.0 / (1.0 + np.exp(-np.asarray(x))))))
lax = types.SimpleNamespace()


def ref_function(relpath, name, cls=None, extra=None):
    """Execute function `name` (optionally a method of class `cls`) from the reference file on the stand-in."""
    path = os.path.join(ENGINE, relpath)
    src = open(path).read()
    tree = ast.parse(src)
    body = tree.body
    if cls is not None:
        body = next(n for n in tree.body if isinstance(n, ast.ClassDef) and n.name == cls).body
    node = next(n for n in body if isinstance(n, ast.FunctionDef) and n.name == name)
    code = textwrap.dedent(ast.get_source_segment(src, node))
    ns = {"np": np, "jnp": jnp, "jax": jax, "lax": lax}
    ns.update(extra or {})
    exec(compile(code, f"{path}:{node.lineno}", "exec"), ns)
    return ns[name]


# ------------------------------------------------------------------------------------------------- fixtures
def gen_plans():
    ragged_plan = ref_function("pallas_moe.py", "ragged_plan")
    rng = np.random.default_rng(11)
    cases = [(20, 2, 6, 8), (24, 2, 6, 16), (37, 3, 10, 8), (64, 8, 16, 32), (1, 8, 12, 8), (50, 4, 40, 16)]
    for c, (T, k, E, tm) in enumerate(cases):
        hi = E if c % 2 == 0 else max(1, E // 2)          # odd cases leave the upper experts unused
        idx = np.stack([rng.choice(hi, size=k, replace=False) for _ in range(T)]).astype(np.int32)
        w = rng.uniform(0.01, 1.0, (T, k)).astype(np.float32)
        p = ragged_plan(J(idx), J(w), E, tm)
        np.savez(os.path.join(HERE, f"plan_{c}.npz"), idx=idx, w=w, E=E, tm=tm,
                 **{k_: np.asarray(v) for k_, v in p.items()})


def gen_swiglu():
    silu = ref_function("model.py", "silu")
    swiglu = ref_function("model.py", "swiglu_clamped", extra={"silu": silu})
    rng = np.random.default_rng(12)
    g = (rng.standard_normal((64, 96)) * 6).astype(np.float32)
    u = (rng.standard_normal((64, 96)) * 6).astype(np.float32)
    out = {f"out_{int(L)}": np.asarray(swiglu(J(g), J(u), np.float32(L))) for L in (10.0, 7.0)}
    np.savez(os.path.join(HERE, "swiglu.npz"), g=g, u=u, **out)


def gen_quant8():
    quantize_array = ref_function("quant8.py", "quantize_array")
    is_q8 = ref_function("quant8.py", "is_q8", extra={"Q8_KEYS": frozenset({"q", "s"})})
    dequant_tree = ref_function("quant8.py", "dequant_tree", extra={"is_q8": is_q8})
    rng = np.random.default_rng(13)
    w = (rng.standard_normal((96, 80)) * 0.02).astype(np.float32)
    w[3, :] = 0.0                                          # an all-zero row and column hit the 1e-12 floor
    w[:, 5] = 0.0
    out = {"w": w}
    for axis in (0, 1):
        qd = quantize_array(J(w), axis)
        out[f"q{axis}"] = np.asarray(qd["q"])
        out[f"s{axis}"] = np.asarray(qd["s"])
        deq = np.asarray(dequant_tree({"q": qd["q"], "s": qd["s"]}, ml_dtypes.bfloat16))
        out[f"deq{axis}"] = deq.view(np.uint16)
    np.savez(os.path.join(HERE, "quant8.npz"), **out)


def _tables(rng, E, H, I):
    t = {}
    for key, rows, K in (("gate", I, H), ("up", I, H), ("down", H, I)):
        t[key] = (cb3.pack(cb3.make_indices(rng, (E, rows, K))), cb3.make_codebooks(rng, (E, rows)))
    return t


def _fake_planes(tbl, E):
    return {"qs": np.zeros((1, E, 1), np.uint32), "cb3": tbl}


def gen_compositions():
    silu = ref_function("model.py", "silu")
    swiglu = ref_function("model.py", "swiglu_clamped", extra={"silu": silu})
    ragged_plan = ref_function("pallas_moe.py", "ragged_plan")
    rng = np.random.default_rng(14)
    E, H, I = 6, 256, 256        # kernel granularity: rows % 64 == 0, inputs % 256 == 0

    def deq(tbl):
        idx, cb = tbl
        return cb3.dequant(idx, cb, idx.shape[-1] * 32 // 3).astype(np.float32)

    def moe_matvec(planes, qt, nblk, flat, X, interpret=False):        # stand-in for pallas_moe.moe_matvec
        W = deq(planes["cb3"])
        x = np.asarray(X, np.float32)[:, :, 0]
        return J(np.einsum("nk,nrk->nr", x.astype(np.float64), W[np.asarray(flat)].astype(np.float64))
                 .astype(np.float32))

    def _grouped(planes_list, be, nb, xs, tm, fn):
        Ws = [deq(p["cb3"]) for p in planes_list]
        xs = np.asarray(xs)
        out = None
        for g in range(xs.shape[0] // tm):
            rows = slice(g * tm, (g + 1) * tm)
            if g < int(np.asarray(nb)[0]):
                e = int(np.asarray(be)[g])
                r = fn(xs[rows].astype(np.float32), [W[e].astype(ml_dtypes.bfloat16).astype(np.float32) for W in Ws])
                out = np.zeros((xs.shape[0], r.shape[1]), xs.dtype) if out is None else out
                out[rows] = r.astype(xs.dtype)
        return J(out)

    def moe_ragged_gateup(pg, pu, qt, nblk, be, nb, xs, limit, tm=32, interpret=False):
        return _grouped([pg, pu], be, nb, xs, tm,
                        lambda x, W: np.asarray(swiglu(J(x @ W[0].T), J(x @ W[1].T), limit), np.float32))

    def moe_ragged_down(pd, qt, nblk, be, nb, hs, tm=32, interpret=False):
        return _grouped([pd], be, nb, hs, tm, lambda x, W: x @ W[0].T)

    PL = types.SimpleNamespace(pm_x=lambda qt, x: J(np.asarray(x)[:, :, None]),
                               plane_rows=lambda qt, nblk: {"qs": 1})
    K = types.SimpleNamespace(moe_matvec=moe_matvec, ragged_plan=ragged_plan, pm_mxu=lambda qt, x: J(np.asarray(x)),
                              moe_ragged_gateup=moe_ragged_gateup, moe_ragged_down=moe_ragged_down)
    M = types.SimpleNamespace(swiglu_clamped=swiglu)
    extra = {"PL": PL, "K": K, "M": M}
    apply_kernel = ref_function("resident.py", "_apply_kernel", cls="ResidentFetch", extra=extra)
    apply_ragged = ref_function("resident.py", "_apply_ragged_kernel", cls="ResidentFetch", extra=extra)

    t = _tables(rng, E, H, I)
    planes = {k_: _fake_planes(v, E) for k_, v in t.items()}
    qtypes = {0: {"gate_q": "CB3", "up_q": "CB3", "down_q": "CB3"}}
    limit = np.float32(10.0)
    tabs = {f"{k_}_idx": v[0] for k_, v in t.items()}
    tabs.update({f"{k_}_cb": v[1].view(np.uint16) for k_, v in t.items()})

    # decode: N tokens x k slots (duplicate experts across tokens on purpose)
    N, k = 3, 3
    idx = np.array([[0, 4, 2], [4, 1, 5], [2, 0, 4]], np.int32)
    w = rng.uniform(0.05, 1.0, (N, k)).astype(np.float32)
    x = rng.standard_normal((N, H)).astype(np.float32)
    fake = types.SimpleNamespace(qtypes=qtypes, nblk={"gate_q": 1, "up_q": 1, "down_q": 1}, interpret=False)
    y = np.asarray(apply_kernel(fake, J(x), J(idx), J(w), 0, planes["gate"], planes["up"], planes["down"], limit))
    np.savez(os.path.join(HERE, "decode_compose.npz"), x=x, idx=idx, w=w, y=y, limit=limit, **tabs)

    # ragged prefill: both combine modes, bf16 activations (out_dtype bf16 as in the serve configuration)
    T, k = 10, 2
    idx = np.stack([rng.choice(4, size=k, replace=False) for _ in range(T)]).astype(np.int32)   # experts 4, 5 unused
    w = rng.uniform(0.05, 1.0, (T, k)).astype(np.float32)
    x = rng.standard_normal((T, H)).astype(np.float32)
    for combine in ("matmul", "gather"):
        fake = types.SimpleNamespace(qtypes=qtypes, nblk={"gate_q": 1, "up_q": 1, "down_q": 1}, interpret=False,
                                     tm=8, combine=combine, out_dtype=ml_dtypes.bfloat16)
        y = np.asarray(apply_ragged(fake, J(x), J(idx), J(w), 0, planes["gate"], planes["up"], planes["down"], limit),
                       np.float32)
        np.savez(os.path.join(HERE, f"ragged_compose_{combine}.npz"), x=x, idx=idx, w=w, y=y, limit=limit, tm=8,
                 **tabs)


def gen_logits():
    quantize_array = ref_function("quant8.py", "quantize_array")
    is_q8 = ref_function("quant8.py", "is_q8", extra={"Q8_KEYS": frozenset({"q", "s"})})
    q8mod = types.ModuleType("glm53.quant8")
    q8mod.is_q8 = is_q8
    pkg = types.ModuleType("glm53")
    pkg.quant8 = q8mod
    sys.modules.setdefault("glm53", pkg)
    sys.modules.setdefault("glm53.quant8", q8mod)
    logits_local = ref_function("engine.py", "_logits_local", cls="Engine")
    rng = np.random.default_rng(15)
    D, V, B = 512, 384, 5
    w = (rng.standard_normal((D, V)) * 0.02).astype(np.float32)
    w[:, 7] = 0.0                                          # a zero column: scale at the 1e-12 floor
    qd = quantize_array(J(w), 1)                           # per-column scales [1, V], as the lm_head leaf
    h = rng.standard_normal((B, D)).astype(np.float32)
    h[1] *= 30.0                                           # a token with a large range
    hb = h.astype(ml_dtypes.bfloat16)
    z = logits_local(None, {"q": qd["q"], "s": qd["s"]}, J(hb))
    np.savez(os.path.join(HERE, "logits_q8.npz"), h=hb.view(np.uint16), q=np.asarray(qd["q"]),
             s=np.asarray(qd["s"], np.float32), z=np.asarray(z).view(np.uint16))


if __name__ == "__main__":
    assert os.path.isdir(ENGINE), f"reference engine not found at {ENGINE!r}: set CBMOE_REFERENCE"
    gen_plans()
    gen_swiglu()
    gen_quant8()
    gen_compositions()
    gen_logits()
    print("golden fixtures written to", HERE)
