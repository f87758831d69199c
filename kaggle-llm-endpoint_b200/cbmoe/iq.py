"""llama.cpp IQ expert formats on the GPU: the counterpart of the reference's iqquant.dequant_rows
(engine/glm53/iqquant.py:230-235) over raw GGUF blocks (IQ2_S 82 B, IQ3_S 110 B, IQ4_XS 136 B per 256 weights),
through cbmoe_iq_dequant. Bit for bit the reference's fp32 values. The lookup tables are gguf-py's grids (the
reference loads the same ones, iq_grids_data.py), uploaded once per device.
"""
import ctypes

import numpy as np
import torch

from ._lib import check, lib, ptr, require_cuda, stream_handle

GGML_TYPE = {"IQ3_S": 21, "IQ2_S": 22, "IQ4_XS": 23}
QK_K = 256
_tables = {}


def block_bytes(qtype):
    return int(lib().cbmoe_iq_block_bytes(GGML_TYPE[qtype]))


def _host_table(qtype):
    import gguf.quants as gq
    if qtype == "IQ4_XS":
        return np.asarray(gq.IQ4_NL.kvalues, np.float32)
    cls = getattr(gq, qtype)
    cls.init_grid()
    return np.asarray(cls.grid, np.float32).reshape(cls.grid_shape)


def table(qtype, device):
    """The format's fp32 lookup table on `device` (gguf-py's grid / IQ4_NL levels), shape checked by the library."""
    key = (qtype, torch.device(device))
    t = _tables.get(key)
    if t is None:
        host = _host_table(qtype)
        entries, width = ctypes.c_int(), ctypes.c_int()
        check(lib().cbmoe_iq_table_shape(GGML_TYPE[qtype], ctypes.byref(entries), ctypes.byref(width)),
              "cbmoe_iq_table_shape")
        assert host.size == entries.value * width.value, (qtype, host.shape, entries.value, width.value)
        t = torch.from_numpy(host.reshape(-1).copy()).to(device)
        _tables[key] = t
    return t


def dequant_rows(raw, qtype, ne0):
    """raw uint8 [nbytes] (GPU) of a row-major GGUF tensor with ne0 weights per row -> fp32 [rows, ne0]."""
    require_cuda(raw)
    assert raw.dtype == torch.uint8 and raw.dim() == 1, (raw.dtype, raw.shape)
    bb = block_bytes(qtype)
    assert ne0 % QK_K == 0 and raw.numel() % (bb * (ne0 // QK_K)) == 0, (raw.numel(), bb, ne0)
    n_blocks = raw.numel() // bb
    raw = raw.contiguous()
    out = torch.empty((n_blocks * QK_K,), dtype=torch.float32, device=raw.device)
    check(lib().cbmoe_iq_dequant(GGML_TYPE[qtype], ptr(raw), n_blocks, ptr(table(qtype, raw.device)), ptr(out),
                                 stream_handle()), "cbmoe_iq_dequant")
    return out.view(-1, ne0)
