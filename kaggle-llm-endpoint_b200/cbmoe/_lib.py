"""ctypes binding of libcbmoe.so (include/cbmoe.h). The library is required: there is no CPU fallback, and every
function here raises if the library or a CUDA device is missing."""
import ctypes
import os

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libcbmoe.so")

c_int, c_float, c_size_t, c_void_p, c_int64 = ctypes.c_int, ctypes.c_float, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_int64

PATHS = {"auto": 0, "decode": 1, "grouped": 2}


class CbmoeError(RuntimeError):
    pass


class Experts(ctypes.Structure):
    _fields_ = [("E", c_int), ("H", c_int), ("I", c_int), ("gateup_idx", c_void_p), ("gateup_cb", c_void_p),
                ("down_idx", c_void_p), ("down_cb", c_void_p), ("gateup_cb8", c_void_p), ("down_cb8", c_void_p)]


class Shared(ctypes.Structure):
    _fields_ = [("gateup_q", c_void_p), ("gate_s", c_void_p), ("up_s", c_void_p), ("down_q", c_void_p),
                ("down_s", c_void_p), ("scale_axis", c_int)]


class IqExperts(ctypes.Structure):
    _fields_ = [("E", c_int), ("H", c_int), ("I", c_int), ("gate_type", c_int), ("up_type", c_int),
                ("down_type", c_int), ("gate", c_void_p), ("up", c_void_p), ("down", c_void_p),
                ("gate_table", c_void_p), ("up_table", c_void_p), ("down_table", c_void_p),
                ("gate8", c_void_p), ("up8", c_void_p), ("down8", c_void_p)]


# name: (restype, argtypes)
SIGNATURES = {
    "cbmoe_version": (c_int, []),
    "cbmoe_status_string": (ctypes.c_char_p, [c_int]),
    "cbmoe_last_cuda_error": (c_int, []),
    "cbmoe_device_errors": (c_int, [c_int, ctypes.POINTER(c_int)]),
    "cbmoe_num_sms": (c_int, []),
    "cbmoe_launch_count": (ctypes.c_longlong, []),
    "cbmoe_profile_enable": (c_int, [c_int]),
    "cbmoe_profile_read": (c_int, [c_int, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_longlong), c_int]),
    "cbmoe_selftest_wait_timeout": (c_int, [ctypes.c_longlong, c_void_p, c_void_p]),
    "cbmoe_cb3k_idx_bytes": (c_size_t, [c_int, c_int, c_int, c_int]),
    "cbmoe_cb3k_cb_bytes": (c_size_t, [c_int, c_int, c_int]),
    "cbmoe_cb3k_repack": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p,
                                  c_void_p, c_void_p]),
    "cbmoe_cb3k_dequant": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p]),
    "cbmoe_cb8_bytes": (c_size_t, [c_int, c_int, c_int]),
    "cbmoe_cb8_build": (c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_void_p]),
    "cbmoe_cb8_matvec_workspace_bytes": (c_size_t, [c_int, c_int]),
    "cbmoe_cb8_matvec": (c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p, c_int, c_void_p, c_void_p, c_size_t,
                                 c_void_p]),
    "cbmoe_w8k_bytes": (c_size_t, [c_int, c_int, c_int]),
    "cbmoe_w8k_repack": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_void_p, c_void_p]),
    "cbmoe_w8k_dequant": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p]),
    "cbmoe_plan_layout": (c_int, [c_int, c_int, c_int, c_int, c_int, ctypes.POINTER(c_int64)]),
    "cbmoe_route_plan": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_void_p, c_size_t,
                                 c_void_p]),
    "cbmoe_workspace_bytes": (c_size_t, [ctypes.POINTER(Experts), c_int, c_int, c_int]),
    "cbmoe_experts_apply": (c_int, [ctypes.POINTER(Experts), c_void_p, c_int, c_void_p, c_void_p, c_int, c_float,
                                    c_int, c_void_p, c_void_p, c_size_t, c_void_p]),
    "cbmoe_experts_apply_noalloc": (c_int, [ctypes.POINTER(Experts), c_void_p, c_int, c_void_p, c_void_p, c_int,
                                            c_float, c_void_p, c_void_p]),
    "cbmoe_moe_layer": (c_int, [ctypes.POINTER(Experts), ctypes.POINTER(Shared), c_void_p, c_int, c_void_p,
                                c_void_p, c_int, c_float, c_int, c_void_p, c_void_p, c_size_t, c_void_p]),
    "cbmoe_matvec_workspace_bytes": (c_size_t, [c_int]),
    "cbmoe_ep_unique_id": (c_int, [c_void_p]),
    "cbmoe_ep_comm_init": (c_int, [c_void_p, c_int, c_int, ctypes.POINTER(c_void_p)]),
    "cbmoe_ep_comm_destroy": (c_int, [c_void_p]),
    "cbmoe_ep_workspace_bytes": (c_size_t, [ctypes.POINTER(Experts), c_int, c_int, c_int, c_int, c_int]),
    "cbmoe_ep_layer": (c_int, [c_void_p, c_int, c_int, ctypes.POINTER(Experts), c_int, ctypes.POINTER(Shared),
                               c_void_p, c_int, c_void_p, c_void_p, c_int, c_float, c_int, c_int, c_void_p,
                               c_void_p, c_void_p, c_size_t, c_void_p]),
    "cbmoe_ep_peer_init": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_void_p, ctypes.POINTER(c_void_p)]),
    "cbmoe_ep_peer_destroy": (c_int, [c_void_p]),
    "cbmoe_cb3_matvec": (c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p, c_int, c_void_p, c_void_p, c_size_t,
                                 c_void_p]),
    "cbmoe_w8_linear": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_void_p, c_int, c_void_p, c_void_p,
                                c_size_t, c_void_p]),
    "cbmoe_w8_logits": (c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p, c_int, c_void_p, c_void_p, c_size_t,
                                c_void_p]),
    "cbmoe_route": (c_int, [c_void_p, c_int, c_int, c_void_p, c_void_p, c_int, c_int, c_int, c_float, c_void_p,
                            c_void_p, c_void_p]),
    "cbmoe_iq_block_bytes": (c_size_t, [c_int]),
    "cbmoe_iq_table_shape": (c_int, [c_int, ctypes.POINTER(c_int), ctypes.POINTER(c_int)]),
    "cbmoe_iq_dequant": (c_int, [c_int, c_void_p, ctypes.c_longlong, c_void_p, c_void_p, c_void_p]),
    "cbmoe_iq8_bytes": (c_size_t, [c_int, c_int, c_int, c_int]),
    "cbmoe_iq8_build": (c_int, [c_int, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p, c_void_p]),
    "cbmoe_iq_workspace_bytes": (c_size_t, [ctypes.POINTER(IqExperts), c_int, c_int]),
    "cbmoe_iq_experts_apply": (c_int, [ctypes.POINTER(IqExperts), c_void_p, c_int, c_void_p, c_void_p, c_int, c_float,
                                       c_void_p, c_void_p, c_size_t, c_void_p]),
}

_lib = None


def lib():
    """Load libcbmoe.so once (raises CbmoeError when it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise CbmoeError(f"{LIB_PATH} is missing: build it with kaggle-llm-endpoint_b200/build.py")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def check(rc, what=""):
    if rc != 0:
        L = lib()
        msg = L.cbmoe_status_string(rc).decode()
        if rc == -2:
            msg += f" (cudaError {L.cbmoe_last_cuda_error()})"
        raise CbmoeError(f"{what}: {msg} [{rc}]")


def ptr(t):
    return None if t is None else c_void_p(t.data_ptr())


def stream_handle(device=None):
    return c_void_p(torch.cuda.current_stream(device).cuda_stream)


def require_cuda(*tensors):
    if not torch.cuda.is_available():
        raise CbmoeError("cbmoe needs a CUDA device (no CPU fallback)")
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise CbmoeError("cbmoe tensors must live on the GPU")


def device_errors(clear=True):
    v = c_int(0)
    check(lib().cbmoe_device_errors(1 if clear else 0, ctypes.byref(v)), "cbmoe_device_errors")
    return v.value


PROFILE_KINDS = ("plan", "cb3_gateup", "cb3_down", "cb3_single", "w8_gateup", "w8_down", "w8_single",
                 "combine", "other", "grp_cb3_gateup", "grp_cb3_down", "grp_w8_gateup", "grp_w8_store", "exchange",
                 "iq_gateup", "iq_down")


def profile_enable(on=True):
    check(lib().cbmoe_profile_enable(1 if on else 0), "cbmoe_profile_enable")


def profile_read(reset=True):
    """{kernel kind: (launches, total ms)} of the launches timed since the last reset."""
    ms = (ctypes.c_double * 16)()
    cnt = (ctypes.c_longlong * 16)()
    check(lib().cbmoe_profile_read(1 if reset else 0, ms, cnt, 16), "cbmoe_profile_read")
    return {name: (int(cnt[i]), float(ms[i])) for i, name in enumerate(PROFILE_KINDS) if cnt[i]}


def launch_count():
    return int(lib().cbmoe_launch_count())
