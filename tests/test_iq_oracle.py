"""The GGUF-format oracle (oracle/iq.py: IQ2_S / IQ3_S / IQ4_XS, Q2_K / Q3_K) pinned against the reference (CPU
only).

The reference's own IQ dequant (iqquant.py, executed on its GGUF samples and on random blocks by
tests/golden/make_iq_golden.py) and gguf-py 0.19.0 (the reference's third-party oracle,
engine/glm53/tests/test_iqquant.py:11-32) must both agree with the restatement bit for bit in fp32.
"""
import os

import numpy as np
import pytest

from oracle import iq

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "iq_samples.npz")
QTYPES = list(iq.BLOCK_BYTES)
SAMPLED = ["IQ2_S", "IQ3_S", "IQ4_XS"]   # the formats with a real GGUF slice in the reference's tests


@pytest.fixture(scope="module")
def tabs():
    return iq.tables()


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


@pytest.mark.parametrize("qt", SAMPLED)
def test_reference_gguf_samples_bit_exact(qt, tabs, golden):
    """The real GLM-5.3-Flash tensor slices of the reference's tests, against the reference's own output."""
    got = iq.dequant_rows(golden[f"{qt}_raw"], qt, int(golden[f"{qt}_ne0"]), tabs)
    want = golden[f"{qt}_ref"]
    assert got.shape == want.shape == (int(golden[f"{qt}_rows"]), int(golden[f"{qt}_ne0"]))
    assert np.array_equal(got, want)
    assert np.abs(want).max() > 0


@pytest.mark.parametrize("qt", QTYPES)
def test_reference_random_blocks_bit_exact(qt, tabs, golden):
    assert np.array_equal(iq.DEQUANT[qt](golden[f"{qt}_rand_raw"], tabs[qt]), golden[f"{qt}_rand_ref"])


@pytest.mark.parametrize("qt", QTYPES)
def test_random_blocks_match_gguf_py(qt, tabs):
    import gguf.quants as gq
    from gguf import GGMLQuantizationType as T
    rng = np.random.default_rng(7)
    blk = iq.random_blocks(rng, 256, qt)
    off = iq.D_OFFSET[qt]
    blk[:3, off:off + 2] = np.frombuffer(np.array([0.0, -0.02, 6.0e-5], np.float16).tobytes(), np.uint8).reshape(3, 2)
    want = gq.dequantize(blk.reshape(-1), getattr(T, qt)).reshape(256, 256)
    assert np.array_equal(iq.DEQUANT[qt](blk, tabs[qt]), want)


def test_tables_shapes(tabs):
    assert tabs["IQ2_S"].shape == (1024, 8) and set(np.unique(tabs["IQ2_S"])) == {8.0, 25.0, 43.0}
    assert tabs["IQ3_S"].shape == (512, 4) and set(np.unique(tabs["IQ3_S"])) == set(range(1, 16, 2))
    assert tabs["IQ4_XS"].shape == (16,) and tabs["IQ4_XS"][0] == -127 and tabs["IQ4_XS"][-1] == 113
