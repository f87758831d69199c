"""The GPU kernels' per-lane GGUF dequant (csrc/iqlane.cuh), compiled for the host by tests/native/iqlane_host.cu,
against the oracle (oracle/iq.py, pinned to the reference): all five formats, the reference's GGUF samples and
random blocks with zero / negative / subnormal block scales, bit for bit. CPU only: it checks the kernels' index
and rounding logic where no GPU is available (test_gpu_iq.py runs the kernels themselves)."""
import ctypes
import os
import subprocess

import numpy as np
import pytest

from oracle import iq

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")


@pytest.fixture(scope="module")
def harness(tmp_path_factory):
    if not os.path.exists(NVCC):
        pytest.skip("nvcc not available")
    so = str(tmp_path_factory.mktemp("iqlane") / "libiqlane_host.so")
    cmd = [NVCC, "-std=c++17", "-O2", "-shared", "-Xcompiler", "-fPIC,-ffp-contract=off",
           "-I", os.path.join(ROOT, "include"), "-I", os.path.join(ROOT, "kaggle-llm-endpoint_b200", "csrc"),
           os.path.join(ROOT, "tests", "native", "iqlane_host.cu"), "-o", so]
    subprocess.run(cmd, check=True, capture_output=True)
    L = ctypes.CDLL(so)
    L.iqlane_host_dequant.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_long, ctypes.c_void_p, ctypes.c_void_p]
    L.iqlane_host_dequant.restype = ctypes.c_int
    return L


def host_dequant(L, qt, blk, table):
    blk = np.ascontiguousarray(blk, np.uint8)
    out = np.empty(blk.shape[0] * 256, np.float32)
    tab = None if table is None else np.ascontiguousarray(table, np.float32)
    rc = L.iqlane_host_dequant(iq.GGML_TYPE[qt], blk.ctypes.data, blk.shape[0],
                               None if tab is None else tab.ctypes.data, out.ctypes.data)
    assert rc == 0
    return out.reshape(blk.shape[0], 256)


@pytest.mark.parametrize("qt", list(iq.BLOCK_BYTES))
def test_lane_dequant_matches_oracle(harness, qt):
    tabs = iq.tables()
    rng = np.random.default_rng(17)
    blk = iq.random_blocks(rng, 300, qt)
    off = iq.D_OFFSET[qt]
    blk[:3, off:off + 2] = np.frombuffer(np.array([0.0, -0.02, 6.0e-5], np.float16).tobytes(), np.uint8).reshape(3, 2)
    want = iq.DEQUANT[qt](blk, tabs[qt])
    got = host_dequant(harness, qt, blk, tabs[qt])
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("qt", list(iq.BLOCK_BYTES))
def test_lane_dequant_matches_reference_fixtures(harness, qt):
    f = np.load(os.path.join(ROOT, "tests", "golden", "iq_samples.npz"))
    tabs = iq.tables()
    got = host_dequant(harness, qt, f[f"{qt}_rand_raw"], tabs[qt])
    assert np.array_equal(got.view(np.uint32), f[f"{qt}_rand_ref"].view(np.uint32))
    if f"{qt}_raw" in f:
        raw = f[f"{qt}_raw"].reshape(-1, iq.BLOCK_BYTES[qt])
        got = host_dequant(harness, qt, raw, tabs[qt]).reshape(f[f"{qt}_ref"].shape)
        assert np.array_equal(got.view(np.uint32), f[f"{qt}_ref"].view(np.uint32))
