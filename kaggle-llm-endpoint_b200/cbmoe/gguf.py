"""GGUF -> device loader for the routed experts: the counterpart of the reference's gguf_reader (engine/glm53/
gguf_reader.py:78-163) and pack_layer_from_gguf (engine/glm53/resident.py:29-46).

The expert tensors blk.{L}.ffn_{gate,up,down}_exps.weight have GGUF dims [ne0 = inputs, ne1 = rows, ne2 = experts],
i.e. bytes ordered [expert][row][256-weight block][block bytes], which is exactly the table layout the IQ expert
kernels read (cbmoe_iq_experts_apply). So loading is a read into pinned host memory and one copy per matrix to
the GPU, no repack. Works on whole .gguf files and on the byte-range pieces of a split mirror (a manifest.json
{"files": {name: {"pieces": [{"name", "start", "length"}, ...]}}} next to them), like the reference's reader;
reads use os.pread from several threads (no mmap).
"""
import json
import os
import struct
from concurrent.futures import ThreadPoolExecutor

import numpy as np

# ggml_type -> (weights per block, bytes per block) for the types this loader sizes
GGML_BLOCK = {0: (1, 4), 1: (1, 2), 8: (32, 34), 10: (256, 84), 11: (256, 110), 12: (256, 144), 13: (256, 176),
              14: (256, 210), 16: (256, 66), 17: (256, 74), 18: (256, 98), 19: (256, 50), 20: (32, 18),
              21: (256, 110), 22: (256, 82), 23: (256, 136), 29: (256, 56), 30: (1, 2)}
GGML_NAME = {0: "F32", 1: "F16", 8: "Q8_0", 10: "Q2_K", 11: "Q3_K", 12: "Q4_K", 13: "Q5_K", 14: "Q6_K",
             16: "IQ2_XXS", 17: "IQ2_XS", 18: "IQ3_XXS", 19: "IQ1_S", 20: "IQ4_NL", 21: "IQ3_S", 22: "IQ2_S",
             23: "IQ4_XS", 29: "IQ1_M", 30: "BF16"}
EXPERT_MATS = (("gate_q", "gate"), ("up_q", "up"), ("down_q", "down"))


class ByteSource:
    """One logical file made of ordered (path, start, length) byte ranges (a whole file is one range)."""

    def __init__(self, ranges):
        self.ranges = sorted(ranges, key=lambda r: r[1])
        self.size = self.ranges[-1][1] + self.ranges[-1][2]
        self._fds = {}

    @classmethod
    def file(cls, path):
        return cls([(path, 0, os.path.getsize(path))])

    def _fd(self, path):
        fd = self._fds.get(path)
        if fd is None:
            fd = self._fds[path] = os.open(path, os.O_RDONLY)
        return fd

    def read_into(self, offset, out):
        """Fill the writable buffer `out` (bytes-like, len n) with bytes [offset, offset + n)."""
        mv = memoryview(out).cast("B")
        n, end = len(mv), offset + len(mv)
        got = 0
        for path, start, length in self.ranges:
            lo, hi = max(offset, start), min(end, start + length)
            if hi <= lo:
                continue
            fd, pos = self._fd(path), lo
            while pos < hi:
                k = os.preadv(fd, [mv[pos - offset:hi - offset]], pos - start)
                if k <= 0:
                    raise IOError(f"short read of {path} at {pos - start}")
                pos += k
            got += hi - lo
        if got != n:
            raise IOError(f"read {got} of {n} bytes at offset {offset}")

    def read(self, offset, n):
        out = bytearray(n)
        self.read_into(offset, out)
        return out

    def close(self):
        for fd in self._fds.values():
            os.close(fd)
        self._fds.clear()


def open_sources(paths):
    """.gguf files and/or directories (holding .gguf files or a mirror's manifest.json + pieces) -> {name: source}."""
    out = {}
    for p in paths:
        if os.path.isfile(p):
            out[os.path.basename(p)] = ByteSource.file(p)
            continue
        man = os.path.join(p, "manifest.json")
        if os.path.exists(man):
            for name, info in json.load(open(man))["files"].items():
                out[name] = ByteSource([(os.path.join(p, q["name"]), q["start"], q["length"]) for q in info["pieces"]])
        for fn in sorted(os.listdir(p)):
            if fn.endswith(".gguf"):
                out[fn] = ByteSource.file(os.path.join(p, fn))
    return out


class GGUFShard:
    """Header, key/values and tensor directory of one GGUF file (format version 2 or 3)."""

    _SCALAR = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<?", 10: "<Q", 11: "<q", 12: "<d"}

    def __init__(self, src, header_bytes=64 << 20):
        self.src = src
        buf = src.read(0, min(src.size, header_bytes))
        self._buf, self._pos = buf, 0
        if bytes(buf[:4]) != b"GGUF":
            raise ValueError("not a GGUF file")
        self._pos = 4
        self.version = self._u("<I")
        n_tensors, n_kv = self._u("<Q"), self._u("<Q")
        self.kv = {}
        for _ in range(n_kv):
            key = self._str()
            self.kv[key] = self._value(self._u("<I"))
        align = int(self.kv.get("general.alignment", 32))
        self.tensors = {}
        for _ in range(n_tensors):
            name = self._str()
            dims = [self._u("<Q") for _ in range(self._u("<I"))]
            ty, off = self._u("<I"), self._u("<Q")
            per, nb = GGML_BLOCK[ty]
            n = int(np.prod(dims)) if dims else 1
            self.tensors[name] = {"dims": dims, "type": GGML_NAME.get(ty, str(ty)), "ggml_type": ty, "offset": off,
                                  "nbytes": n // per * nb}
        self.data0 = (self._pos + align - 1) // align * align
        del self._buf

    def _u(self, fmt):
        v = struct.unpack_from(fmt, self._buf, self._pos)[0]
        self._pos += struct.calcsize(fmt)
        return v

    def _str(self):
        n = self._u("<Q")
        s = bytes(self._buf[self._pos:self._pos + n]).decode("utf-8", errors="replace")
        self._pos += n
        return s

    def _value(self, t):
        if t in self._SCALAR:
            return self._u(self._SCALAR[t])
        if t == 8:
            return self._str()
        if t == 9:
            et, n = self._u("<I"), self._u("<Q")
            return [self._value(et) for _ in range(n)]
        raise ValueError(f"GGUF value type {t}")

    def read_into(self, name, out, offset=0):
        t = self.tensors[name]
        self.src.read_into(self.data0 + t["offset"] + offset, out)


class GGUFModel:
    """All shards of a (split) GGUF model behind one tensor directory."""

    def __init__(self, paths):
        self.shards = {n: GGUFShard(s) for n, s in sorted(open_sources(paths).items())}
        self.kv, self.where = {}, {}
        for n, sh in self.shards.items():
            self.kv.update(sh.kv)
            for t in sh.tensors:
                self.where[t] = n

    def info(self, name):
        return self.shards[self.where[name]].tensors[name]

    def read_into(self, name, out, offset=0):
        self.shards[self.where[name]].read_into(name, out, offset)

    def read(self, name):
        out = np.empty(self.info(name)["nbytes"], np.uint8)
        self.read_into(name, out)
        return out

    def close(self):
        for sh in self.shards.values():
            sh.src.close()


def expert_tensor(layer, mat):
    return f"blk.{layer}.ffn_{mat}_exps.weight"


def layer_shapes(model, layer):
    """{key: (qtype, E, rows, K)} of a layer's three expert matrices; H and I from the gate's dims."""
    out = {}
    for key, mat in EXPERT_MATS:
        t = model.info(expert_tensor(layer, mat))
        K, rows, E = t["dims"]
        out[key] = (t["type"], E, rows, K)
    return out


def read_layer(model, layer, out=None, threads=8, chunk=64 << 20):
    """Bytes of one layer's expert tables into `out` ({key: writable uint8 buffer of the tensor's size}, e.g. pinned
    host tensors) or fresh numpy arrays, each tensor read in `chunk`-byte pieces on `threads` threads."""
    out = out or {key: np.empty(model.info(expert_tensor(layer, mat))["nbytes"], np.uint8) for key, mat in EXPERT_MATS}
    jobs = []
    for key, mat in EXPERT_MATS:
        name, buf = expert_tensor(layer, mat), memoryview(out[key]).cast("B")
        jobs += [(name, buf, o, min(chunk, len(buf) - o)) for o in range(0, len(buf), chunk)]
    with ThreadPoolExecutor(max(1, threads)) as pool:
        list(pool.map(lambda j: model.read_into(j[0], j[1][j[2]:j[2] + j[3]], j[2]), jobs))
    return out


def load_layer(model, layer, device="cuda", threads=8):
    """One layer's routed experts from the GGUF straight into GPU memory, as the table dict of cbmoe.iq.pack_layer
    (ResidentFetch.apply then runs them); returns (tables, qtypes) like the reference's pack_layer_from_gguf."""
    import torch
    from . import iq
    shapes = layer_shapes(model, layer)
    qtypes = {key: s[0] for key, s in shapes.items()}
    for key, qt in qtypes.items():
        if qt not in iq.GGML_TYPE:
            raise NotImplementedError(f"{expert_tensor(layer, dict(EXPERT_MATS)[key])}: format {qt} has no kernels here")
    E, I, H = shapes["gate_q"][1], shapes["gate_q"][2], shapes["gate_q"][3]
    assert shapes["up_q"][1:] == (E, I, H) and shapes["down_q"][1:] == (E, H, I), shapes
    host = {key: torch.empty(model.info(expert_tensor(layer, mat))["nbytes"], dtype=torch.uint8).pin_memory()
            for key, mat in EXPERT_MATS}
    read_layer(model, layer, {k: v.numpy() for k, v in host.items()}, threads=threads)
    dev = {k: v.to(device, non_blocking=True) for k, v in host.items()}
    torch.cuda.current_stream(device).synchronize()
    return iq.pack_layer(dev["gate_q"], dev["up_q"], dev["down_q"], qtypes, E, H, I), qtypes
