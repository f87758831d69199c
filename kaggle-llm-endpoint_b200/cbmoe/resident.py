"""Host-side mirror of the reference's expert-fetch boundary (resident.py:68-210, `ResidentFetch`) and of
`moe_dense` below the router (model.py:840-856), on the CUDA library.

    tables = pack_layer(gate, up, down, shared)              # load time, like pack_layer_from_gguf + pack_chip_planes
    fetch = ResidentFetch(qtypes, D, ml)                     # engine-held object, same constructor knobs
    y = fetch.apply(p, x, idx, w, layer, limit)              # p = the layer's mlp params = tables
    out = moe_dense(p, x, idx, w, limit, fetch)              # routed + shared expert, bf16

`apply` keeps the reference's argument meaning: x [N, D] (bf16), idx int32 [N, k] into E, w fp32 [N, k] already
normalized and scaled, `layer` indexes `qtypes`, `limit` is the SwiGLU clamp; it returns the fp32 partial [N, D]
(the caller casts it, adds the shared expert and reduces across ranks). Shape problems raise like the reference's
asserts; there is no CPU fallback.
"""
import torch

from . import iq, ops
from ._lib import PATHS, Experts, Shared, check, lib, ptr, require_cuda, stream_handle

CB3 = "CB3"


def pack_layer(gate, up, down, shared=None, decode_tables="int8"):
    """Device tables of one layer from CB3 gate/up [E, I, H] and down [E, H, I] tables ((idx int32-packed uint32
    words, cb bf16) pairs on the GPU) and an optional int8 shared expert ((q [in, out] int8, s fp32) for gate, up,
    down; scales per output column [1, out] or per input row [in, 1] as quant8.quantize_array makes them).
    `decode_tables`: "int8" also builds the CB8 tables, so the decode path runs the int8-digit kernels (20 bytes per row
    more); "bf16" leaves them out (the bf16 decode kernels)."""
    (gi, gc), (ui, uc), (di, dc) = gate, up, down
    E, I, wpr = gi.shape
    H = wpr * 32 // 3
    assert di.shape[:2] == (E, H), (di.shape, E, H)
    assert decode_tables in ("int8", "bf16"), decode_tables
    gu_idx, gu_cb = ops.pack_cb3(gi, gc, ui, uc)
    dn_idx, dn_cb = ops.pack_cb3(di, dc)
    p = {"E": E, "H": H, "I": I, "gate_up_q": (gu_idx, gu_cb), "down_q": (dn_idx, dn_cb)}
    if decode_tables == "int8":
        p["gate_up_cb8"] = ops.build_cb8(gu_cb, 2, E, I)
        p["down_cb8"] = ops.build_cb8(dn_cb, 1, E, H)
    if shared is not None:
        (gq, gs), (uq, us), (dq, ds) = shared
        axis = 1 if gs.shape[0] == 1 else 0
        p["shared"] = {"gate_up_q": ops.pack_w8(gq, uq), "down_q": ops.pack_w8(dq),
                       "gate_s": gs.reshape(-1).float().contiguous(), "up_s": us.reshape(-1).float().contiguous(),
                       "down_s": ds.reshape(-1).float().contiguous(), "scale_axis": axis}
    return p


def _experts_struct(p):
    cb8 = (p["gate_up_cb8"].data_ptr(), p["down_cb8"].data_ptr()) if "gate_up_cb8" in p else (None, None)
    return Experts(p["E"], p["H"], p["I"], p["gate_up_q"][0].data_ptr(), p["gate_up_q"][1].data_ptr(),
                   p["down_q"][0].data_ptr(), p["down_q"][1].data_ptr(), *cb8)


def _shared_struct(s):
    return Shared(s["gate_up_q"].data_ptr(), s["gate_s"].data_ptr(), s["up_s"].data_ptr(), s["down_q"].data_ptr(),
                  s["down_s"].data_ptr(), s["scale_axis"])


class ResidentFetch:
    """Stored on the engine; `apply(p, x, idx, w, layer, limit)` as in resident.py:100-108.

    Constructor knobs keep the reference's names: `qtypes` {layer: {"gate_q", "up_q", "down_q"} -> format}
    ("CB3" only here), `D`, `ml` (this GPU's intermediate size), `out_dtype` of the returned partial,
    `gather_max_rows` (slots N*k at or below which the decode kernels run; above it the grouped path), and
    `path` to force "decode" or "grouped"."""

    def __init__(self, qtypes=None, D=None, ml=None, out_dtype=torch.float32, gather_max_rows=1024, path="auto"):
        self.qtypes = qtypes or {}
        self.D, self.ml = D, ml
        self.out_dtype = out_dtype
        self.gather_max_rows = gather_max_rows
        self.path = path
        self._ws = {}

    def _path_code(self, N, k):
        if self.path != "auto":
            return PATHS[self.path]
        return PATHS["decode"] if N * k <= self.gather_max_rows else PATHS["grouped"]

    def workspace(self, p, N, k, path, device):
        ex = _experts_struct(p)
        nbytes = lib().cbmoe_workspace_bytes(ex, N, k, path)
        key = (device, nbytes)
        ws = self._ws.get(key)
        if ws is None:
            ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=device)
            self._ws = {key: ws}
        return ex, ws

    def _check(self, p, x, idx, w, layer):
        require_cuda(x, idx, w)
        for key in ("gate_q", "up_q", "down_q"):
            have = p["qtypes"][key] if p.get("format") == "IQ" else CB3
            qt = self.qtypes.get(layer, {}).get(key, have)
            if qt != have:
                raise ValueError(f"layer {layer} {key}: qtypes says {qt}, the tables hold {have}")
        N, k = idx.shape
        assert x.shape == (N, p["H"]), (x.shape, N, p["H"])
        assert w.shape == (N, k), (w.shape, (N, k))
        if self.D is not None:
            assert self.D == p["H"], (self.D, p["H"])
        if self.ml is not None:
            assert self.ml == p["I"], (self.ml, p["I"])
        return N, k

    def apply(self, p, x, idx, w, layer, limit):
        """x [N, D]; idx [N, k] int32 into E; w [N, k] fp32 -> routed partial [N, D] in out_dtype."""
        N, k = self._check(p, x, idx, w, layer)
        if p.get("format") == "IQ":   # raw GGUF IQ tables (cbmoe.iq.pack_layer)
            y = iq.apply(p, x.to(torch.bfloat16).contiguous(), idx.to(torch.int32).contiguous(),
                         w.to(torch.float32).contiguous(), limit)
            return y if self.out_dtype == torch.float32 else y.to(self.out_dtype)
        xb = x.to(torch.bfloat16).contiguous()
        idx = idx.to(torch.int32).contiguous()
        w = w.to(torch.float32).contiguous()
        y = torch.empty((N, p["H"]), dtype=torch.float32, device=x.device)
        path = self._path_code(N, k)
        ex, ws = self.workspace(p, N, k, path, x.device)
        check(lib().cbmoe_experts_apply(ex, ptr(xb), N, ptr(idx), ptr(w), k, float(limit), path, ptr(y), ptr(ws),
                                        ws.numel(), stream_handle()), "cbmoe_experts_apply")
        return y if self.out_dtype == torch.float32 else y.to(self.out_dtype)

    def layer(self, p, x, idx, w, limit, out=None):
        """Routed experts + shared expert -> bf16 [N, D] (model.py:847-855 without the router and the reduce)."""
        N, k = self._check(p, x, idx, w, 0)
        if "shared" not in p:
            raise ValueError("layer tables have no shared expert")
        xb = x.to(torch.bfloat16).contiguous()
        idx = idx.to(torch.int32).contiguous()
        w = w.to(torch.float32).contiguous()
        if out is None:
            out = torch.empty((N, p["H"]), dtype=torch.bfloat16, device=x.device)
        path = self._path_code(N, k)
        ex, ws = self.workspace(p, N, k, path, x.device)
        sh = _shared_struct(p["shared"])
        check(lib().cbmoe_moe_layer(ex, sh, ptr(xb), N, ptr(idx), ptr(w), k, float(limit), path, ptr(out), ptr(ws),
                                    ws.numel(), stream_handle()), "cbmoe_moe_layer")
        return out


def moe_dense(p, x, idx, w, limit, fetch):
    """model.py:840-856 after `moe_route`: y = fetch.apply(...) + mlp_partial(shared), bf16 out (no TP reduce)."""
    return fetch.layer(p, x, idx, w, limit)


def moe_route(x, router_w, bias, k, norm_topk=True, scaling=1.0):
    """model.py:798-808 on the GPU (cbmoe_route): x [N, D] (bf16), router_w [D, E] (bf16), bias [E] ->
    (idx int32 [N, k], w fp32 [N, k]); sigmoid scores, top k of scores + bias, weights = the chosen scores,
    normalized when norm_topk, times scaling."""
    require_cuda(x, router_w, bias)
    N, D = x.shape
    assert router_w.shape[0] == D and bias.shape == (router_w.shape[1],), (x.shape, router_w.shape, bias.shape)
    E = router_w.shape[1]
    xb = x.to(torch.bfloat16).contiguous()
    wb = router_w.to(torch.bfloat16).contiguous()
    bf = bias.to(torch.float32).contiguous()
    idx = torch.empty((N, k), dtype=torch.int32, device=x.device)
    w = torch.empty((N, k), dtype=torch.float32, device=x.device)
    check(lib().cbmoe_route(ptr(xb), N, D, ptr(wb), ptr(bf), E, k, 1 if norm_topk else 0, float(scaling), ptr(idx),
                            ptr(w), stream_handle()), "cbmoe_route")
    return idx, w
