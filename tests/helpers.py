"""Conversions between the oracle's NumPy arrays and the CUDA library's torch tensors (tests only)."""
import numpy as np
import torch

from oracle import cb3


def t_u32(a, dev="cuda"):
    """uint32 NumPy -> int32 torch tensor with the same bits."""
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int32)).to(dev)


def t_bf16(a, dev="cuda"):
    """bf16 (ml_dtypes) or float NumPy -> torch bf16 with the same bits."""
    bits = np.ascontiguousarray(np.asarray(a, cb3.BF16)).view(np.int16)
    return torch.from_numpy(bits).to(dev).view(torch.bfloat16)


def bf16_bits_of(t):
    """torch bf16 -> NumPy uint16 bit patterns."""
    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def table_to_gpu(tbl, dev="cuda"):
    idx, cb = tbl
    return t_u32(idx, dev), t_bf16(cb, dev)


def shared_to_gpu(shared, dev="cuda"):
    return tuple((torch.from_numpy(q).to(dev), torch.from_numpy(np.asarray(s, np.float32)).to(dev)) for q, s in shared)
