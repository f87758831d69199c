"""ctypes binding of the C oracle (oracle/cbmoe_cpu.c): test infrastructure and the timed CPU baseline."""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
SO = os.path.join(HERE, "libcbmoe_cpu.so")
_lib = None


def build():
    """make -C oracle (gcc + OpenMP)."""
    src = os.path.join(HERE, "cbmoe_cpu.c")
    if not os.path.exists(SO) or os.path.getmtime(SO) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", HERE], check=True)
    return SO


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(SO):
            build()
        L = ctypes.CDLL(SO)
        P = ctypes.c_void_p
        L.cbmoe_cpu_cb3_matvec.argtypes = [P, P, ctypes.c_int, ctypes.c_int, P, ctypes.c_int, P, ctypes.c_int]
        L.cbmoe_cpu_moe_layer.argtypes = [ctypes.c_int] * 3 + [P] * 12 + [ctypes.c_int, P, ctypes.c_int, P, P,
                                                                          ctypes.c_int, ctypes.c_float, P, ctypes.c_int]
        L.cbmoe_cpu_moe_layer.restype = ctypes.c_int
        L.cbmoe_cpu_max_threads.restype = ctypes.c_int
        _lib = L
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def max_threads():
    return int(lib().cbmoe_cpu_max_threads())


def cb3_matvec(idx, cb, x, threads=0):
    """idx uint32 [rows, K*3/32], cb bf16 [rows, 8], x f32 [N, K] -> f32 [N, rows]."""
    idx = np.ascontiguousarray(idx, np.uint32)
    cb = np.ascontiguousarray(np.asarray(cb).view(np.uint16))
    x = np.ascontiguousarray(x, np.float32)
    rows, K = idx.shape[0], x.shape[1]
    y = np.zeros((x.shape[0], rows), np.float32)
    lib().cbmoe_cpu_cb3_matvec(_p(idx), _p(cb), rows, K, _p(x), x.shape[0], _p(y), threads)
    return y


def moe_layer(x, idx, w, gate, up, down, shared=None, limit=10.0, threads=0):
    """Routed CB3 experts (+ int8 shared expert) for tokens x f32 [N, H] -> f32 [N, H] (see cbmoe_cpu.c)."""
    (gi, gc), (ui, uc), (di, dc) = [(np.ascontiguousarray(a, np.uint32), np.ascontiguousarray(np.asarray(b).view(np.uint16)))
                                    for a, b in (gate, up, down)]
    E, I = gi.shape[:2]
    H = di.shape[1]
    x = np.ascontiguousarray(x, np.float32)
    idx = np.ascontiguousarray(idx, np.int32)
    w = np.ascontiguousarray(w, np.float32)
    N, k = idx.shape
    out = np.zeros((N, H), np.float32)
    if shared is not None:
        (gq, gs), (uq, us), (dq, ds) = shared
        axis = 1 if np.asarray(gs).shape[0] == 1 else 0
        sh = [np.ascontiguousarray(a) for a in (gq, np.asarray(gs, np.float32).reshape(-1), uq,
                                               np.asarray(us, np.float32).reshape(-1), dq,
                                               np.asarray(ds, np.float32).reshape(-1))]
    else:
        axis, sh = 1, [None] * 6
    rc = lib().cbmoe_cpu_moe_layer(E, H, I, _p(gi), _p(gc), _p(ui), _p(uc), _p(di), _p(dc), *[_p(a) for a in sh], axis,
                                   _p(x), N, _p(idx), _p(w), k, float(limit), _p(out), threads)
    assert rc == 0
    return out
