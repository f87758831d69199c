"""GGUF -> table loader (cbmoe/gguf.py) on CPU: a small GGUF written by gguf-py (the writer the reference's own
reader test uses, engine/glm53/tests/test_gguf_reader.py) with a layer's three expert tensors in mixed IQ formats,
read whole and as a split mirror (1000-byte pieces + manifest.json)."""
import json

import numpy as np
import pytest

from oracle import iq as oiq

E, H, I, LAYER = 4, 512, 256, 3
QT = {"gate_q": "IQ2_S", "up_q": "IQ2_S", "down_q": "IQ3_S"}


def write_model(path, rng):
    from gguf import GGMLQuantizationType as T
    from gguf import GGUFWriter
    raw = {"gate_q": oiq.random_blocks(rng, E * I * (H // 256), QT["gate_q"]).reshape(E, I, -1),
           "up_q": oiq.random_blocks(rng, E * I * (H // 256), QT["up_q"]).reshape(E, I, -1),
           "down_q": oiq.random_blocks(rng, E * H * (I // 256), QT["down_q"]).reshape(E, H, -1)}
    w = GGUFWriter(str(path), "glm5next")
    w.add_uint32("glm5next.expert_count", E)
    for key, mat in (("gate_q", "gate"), ("up_q", "up"), ("down_q", "down")):
        w.add_tensor(f"blk.{LAYER}.ffn_{mat}_exps.weight", raw[key], raw_dtype=getattr(T, QT[key]))
    small = np.arange(64, dtype=np.float32).reshape(8, 8)
    w.add_tensor("blk.0.attn_norm.weight", small)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return raw, small


def split(path, d, piece=1000):
    d.mkdir()
    data = path.read_bytes()
    pieces = []
    for i, s in enumerate(range(0, len(data), piece)):
        (d / f"m.gguf.p{i:03d}").write_bytes(data[s:s + piece])
        pieces.append({"name": f"m.gguf.p{i:03d}", "start": s, "length": len(data[s:s + piece])})
    (d / "manifest.json").write_text(json.dumps({"files": {"m.gguf": {"size": len(data), "pieces": pieces}}}))


@pytest.fixture(scope="module")
def model_files(tmp_path_factory):
    tmp = tmp_path_factory.mktemp("gguf")
    raw, small = write_model(tmp / "m.gguf", np.random.default_rng(0))
    split(tmp / "m.gguf", tmp / "pieces")
    return tmp, raw, small


@pytest.mark.parametrize("where", ["file", "dir", "pieces"])
def test_reads_layer_tables(model_files, where):
    from cbmoe import gguf
    tmp, raw, small = model_files
    path = {"file": tmp / "m.gguf", "dir": tmp, "pieces": tmp / "pieces"}[where]
    m = gguf.GGUFModel([str(path)])
    assert m.kv["glm5next.expert_count"] == E
    shapes = gguf.layer_shapes(m, LAYER)
    assert shapes == {"gate_q": ("IQ2_S", E, I, H), "up_q": ("IQ2_S", E, I, H), "down_q": ("IQ3_S", E, H, I)}
    for threads, chunk in ((1, 1 << 20), (4, 999)):            # chunks that straddle the 1000-byte pieces
        got = gguf.read_layer(m, LAYER, threads=threads, chunk=chunk)
        for key in QT:
            assert np.array_equal(got[key], raw[key].reshape(-1)), key
    assert np.array_equal(m.read("blk.0.attn_norm.weight").view(np.float32).reshape(8, 8), small)
    m.close()


def test_reader_rejects_other_files(tmp_path):
    from cbmoe import gguf
    p = tmp_path / "x.gguf"
    p.write_bytes(b"NOPE" + bytes(64))
    with pytest.raises(ValueError):
        gguf.GGUFModel([str(p)])


@pytest.mark.gpu
def test_load_layer_runs_through_resident_fetch(model_files):
    """The loaded layer through ResidentFetch.apply against the oracle's composition of the same tables."""
    import torch
    import cbmoe
    from cbmoe import gguf
    from oracle import gen, moe
    tmp, raw, _ = model_files
    m = gguf.GGUFModel([str(tmp / "pieces")])
    p, qtypes = gguf.load_layer(m, LAYER)
    assert qtypes == QT
    rng = np.random.default_rng(1)
    x = gen.activations(rng, 5, H)
    idx, w = gen.routing(rng, 5, E, 2)
    y = cbmoe.ResidentFetch(qtypes={LAYER: qtypes}).apply(
        p, torch.from_numpy(x.view(np.uint16).copy()).cuda().view(torch.bfloat16), torch.from_numpy(idx).cuda(),
        torch.from_numpy(w).cuda(), LAYER, gen.LIMIT)
    tabs = oiq.tables()
    W = {k: oiq.experts_dense(raw[k].reshape(-1), QT[k], E, rows, K, tabs)
         for k, (rows, K) in {"gate_q": (I, H), "up_q": (I, H), "down_q": (H, I)}.items()}
    want = oiq.decode_apply(x.astype(np.float32), idx, w, W["gate_q"], W["up_q"], W["down_q"], gen.LIMIT)
    assert moe.max_rel_err(y.cpu().numpy(), want) < 2e-3
