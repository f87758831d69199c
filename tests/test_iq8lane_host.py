"""The int8 GGUF kernels' transcode and fragment arithmetic (csrc/iq8lane.cuh), compiled for the host by
tests/native/iq8lane_host.cu: every weight rebuilt from the lanes' words through the A fragments the kernels build
(and the input the MMA pairs it with) must equal the oracle's dequant of the raw block bit for bit, for IQ2_S and
IQ3_S, on the reference's GGUF samples and on random blocks. CPU only (test_gpu_iq.py runs the kernels)."""
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
    so = str(tmp_path_factory.mktemp("iq8lane") / "libiq8lane_host.so")
    cmd = [NVCC, "-std=c++17", "-O2", "-shared", "-Xcompiler", "-fPIC,-ffp-contract=off",
           "-I", os.path.join(ROOT, "include"), "-I", os.path.join(ROOT, "kaggle-llm-endpoint_b200", "csrc"),
           os.path.join(ROOT, "tests", "native", "iq8lane_host.cu"), "-o", so]
    subprocess.run(cmd, check=True, capture_output=True)
    L = ctypes.CDLL(so)
    L.iq8_host_reconstruct.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    L.iq8_host_reconstruct.restype = ctypes.c_int
    return L


def reconstruct(L, qt, blk16, table):
    blk16 = np.ascontiguousarray(blk16, np.uint8)
    out = np.empty((16, 256), np.float32)
    tab = np.ascontiguousarray(table, np.float32)
    rc = L.iq8_host_reconstruct(iq.GGML_TYPE[qt], blk16.ctypes.data, tab.ctypes.data, out.ctypes.data)
    assert rc == 0, rc
    return out


@pytest.mark.parametrize("qt", ["IQ2_S", "IQ3_S"])
def test_transcode_rebuilds_random_blocks(harness, qt):
    tabs = iq.tables()
    rng = np.random.default_rng(23)
    for _ in range(8):
        blk = iq.random_blocks(rng, 16, qt)
        blk[0, 0:2] = np.frombuffer(np.array([-0.02], np.float16).tobytes(), np.uint8)
        want = iq.DEQUANT[qt](blk, tabs[qt])
        got = reconstruct(harness, qt, blk, tabs[qt])
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("qt", ["IQ2_S", "IQ3_S"])
def test_transcode_rebuilds_reference_samples(harness, qt):
    f = np.load(os.path.join(ROOT, "tests", "golden", "iq_samples.npz"))
    tabs = iq.tables()
    raw, ref = f[f"{qt}_rand_raw"], f[f"{qt}_rand_ref"]
    n = raw.shape[0] // 16 * 16
    assert n >= 16
    for b0 in range(0, n, 16):
        got = reconstruct(harness, qt, raw[b0:b0 + 16], tabs[qt])
        assert np.array_equal(got.view(np.uint32), ref[b0:b0 + 16].reshape(16, 256).view(np.uint32))
