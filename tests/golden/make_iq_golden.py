"""Generate iq_samples.npz in this folder by EXECUTING the reference's IQ dequant (iqquant.py) on its own GGUF samples.

Run where the reference checkout (read-only) is available, naming its root in $CBMOE_REFERENCE, with gguf-py
installed:
    CBMOE_REFERENCE=<reference checkout> python tests/golden/make_iq_golden.py
Nothing at test time reads the reference; the tests read the .npz written here (and gguf-py, which is installed).

Executed reference functions (launcher/glm53-flash/engine/glm53/iqquant.py): dequant_iq2_s, dequant_iq3_s,
dequant_iq4_xs, dequant_q2_k, dequant_q3_k and the helpers they call (_f16, _u16, _bits8, _nibbles,
_signs_from_bits, _kv16, _f16_at, _kq_layout, q3k_scales, lookup with
LOOKUP_IMPL = "take", which the reference's tests hold equal to its select-tree lookup), on the NumPy stand-in
for jax of make_golden.py plus `jax.lax.bitcast_convert_type`. The grid tables come from the reference's own
iq_grids_data.py. Inputs:
  * the three real GGUF tensor slices of the reference's tests (engine/glm53/tests/data/*.bin, described by
    gguf_samples.json): IQ2_S 2 x 4096 (blk.3.ffn_gate_exps), IQ3_S 4 x 2048 (blk.3.ffn_down_exps), IQ4_XS 4 x 2048
    (blk.11.ffn_down_exps), stored here as raw bytes with the reference's output;
  * 16 random blocks per format (seeded; block scale d a positive f16 in [1e-3, 2e-2] as in the reference's
    test_random_blocks_match_gguf_py; Q2_K/Q3_K, which have no sample, only these).
Every output is also checked against gguf-py's dequantize (the reference's own oracle) before it is written.
"""
import importlib.util
import json
import os
import sys
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import make_golden as mg  # noqa: E402  (the NumPy stand-in for jax and ref_function)

BLOCK_BYTES = {"IQ2_S": 82, "IQ3_S": 110, "IQ4_XS": 136}
KQUANT_BYTES = {"Q2_K": 84, "Q3_K": 110}   # the MTP layer's formats: no GGUF sample in the reference, random blocks


def _bitcast(x, dtype):
    """jax.lax.bitcast_convert_type for a narrower -> wider type: the trailing axis (the size ratio) is consumed."""
    x = np.ascontiguousarray(np.asarray(x))
    out = x.view(dtype)
    if np.dtype(dtype).itemsize > x.dtype.itemsize:
        out = out.reshape(out.shape[:-1])
    return mg.J(out)


def stand_in():
    jnp = types.SimpleNamespace(**vars(mg.jnp))
    jnp.stack = mg._wrap(np.stack)
    jnp.uint8, jnp.uint16, jnp.float16 = np.uint8, np.uint16, np.float16
    lax = types.SimpleNamespace(bitcast_convert_type=_bitcast)
    jax = types.SimpleNamespace(lax=lax, nn=mg.jax.nn)
    return jnp, jax, lax


def reference_dequant():
    spec = importlib.util.spec_from_file_location("iq_grids_data", os.path.join(mg.ENGINE, "iq_grids_data.py"))
    gd = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(gd)
    g = gd.load()
    grids = {k: np.asarray(g[k]) for k in ("IQ2_S", "IQ3_S", "IQ2_XS", "IQ3_XXS")}
    jnp, jax, lax = stand_in()
    ns = {"jnp": jnp, "jax": jax, "lax": lax, "QK_K": 256, "GRIDS": grids, "LOOKUP_IMPL": "take",
          "KVALUES_IQ4NL": np.asarray(g["kvalues_iq4nl"]), "_TREES": {}}
    for name in ("_u16", "_u32", "_f16", "_bits8", "_nibbles", "_signs_from_bits", "_kv16", "lookup"):
        ns[name] = mg.ref_function("iqquant.py", name, extra=ns)
    ns["q3k_scales"] = mg.ref_function("iqquant.py", "q3k_scales", extra=ns)
    ns["_f16_at"] = mg.ref_function("iqquant.py", "_f16_at", extra=ns)
    ns["_kq_layout"] = mg.ref_function("iqquant.py", "_kq_layout", extra=ns)
    out = {qt: mg.ref_function("iqquant.py", f"dequant_{qt.lower()}", extra=ns) for qt in BLOCK_BYTES}
    out.update({qt: mg.ref_function("iqquant.py", f"dequant_{qt.lower()}", extra=ns) for qt in KQUANT_BYTES})
    return out


def gguf_dequant(raw, qt):
    import gguf.quants as gq
    from gguf import GGMLQuantizationType as T
    return gq.dequantize(np.ascontiguousarray(raw).reshape(-1), getattr(T, qt)).astype(np.float32)


def main():
    assert os.path.isdir(mg.ENGINE), f"reference engine not found at {mg.ENGINE}"
    deq = reference_dequant()
    samples = json.load(open(os.path.join(mg.ENGINE, "tests", "data", "gguf_samples.json")))
    out = {}
    rng = np.random.default_rng(21)
    for qt, bb in BLOCK_BYTES.items():
        s = samples[qt]
        raw = np.fromfile(os.path.join(mg.ENGINE, "tests", "data", os.path.basename(s["file"])), np.uint8)
        rows, ne0 = s["rows"], s["ne0"]
        blk = raw.reshape(rows, ne0 // 256, bb)
        ref = np.asarray(deq[qt](mg.J(blk)), np.float32).reshape(rows, ne0)
        np.testing.assert_array_equal(ref, gguf_dequant(raw, qt).reshape(rows, ne0))
        out.update({f"{qt}_raw": raw, f"{qt}_rows": rows, f"{qt}_ne0": ne0, f"{qt}_ref": ref,
                    f"{qt}_tensor": s["tensor"]})
        rb = rng.integers(0, 256, (16, bb), dtype=np.uint8)
        d = rng.uniform(1e-3, 2e-2, 16).astype(np.float16)
        rb[:, 0:2] = np.frombuffer(d.tobytes(), np.uint8).reshape(16, 2)
        rref = np.asarray(deq[qt](mg.J(rb)), np.float32).reshape(16, 256)
        np.testing.assert_array_equal(rref, gguf_dequant(rb, qt).reshape(16, 256))
        out.update({f"{qt}_rand_raw": rb, f"{qt}_rand_ref": rref})
    for qt, bb in KQUANT_BYTES.items():
        off = {"Q2_K": 80, "Q3_K": 108}[qt]
        rb = rng.integers(0, 256, (16, bb), dtype=np.uint8)
        rb[:, off:off + 2] = np.frombuffer(rng.uniform(1e-3, 2e-2, 16).astype(np.float16).tobytes(),
                                           np.uint8).reshape(16, 2)
        if qt == "Q2_K":
            rb[:, 82:84] = np.frombuffer(rng.uniform(1e-4, 2e-3, 16).astype(np.float16).tobytes(),
                                         np.uint8).reshape(16, 2)
        rref = np.asarray(deq[qt](mg.J(rb.reshape(16, 1, bb))), np.float32).reshape(16, 256)
        np.testing.assert_array_equal(rref, gguf_dequant(rb, qt).reshape(16, 256))
        out.update({f"{qt}_rand_raw": rb, f"{qt}_rand_ref": rref})
    np.savez_compressed(os.path.join(HERE, "iq_samples.npz"), **out)
    print("iq_samples.npz written to", HERE)


if __name__ == "__main__":
    main()
