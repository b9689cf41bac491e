"""GGUF reader: the weights of a GGUF file (or a split GGUF) memory-mapped straight into the layouts the ops take.

The reference reads GGUFs with gguf-py (inspect_gguf.py:21-60) and its command programs view each parameter in place
(``command.parameter %weights, "name" : view<BYTESxi8>``, gen_llm.py:5366-5373): a quantised tensor is its raw block
bytes. This module parses the file format itself (no dependency on gguf-py) and hands out the same raw bytes:

* ``GGUFFile(path)`` -- metadata, tensor infos and a read-only ``numpy.memmap`` of every part. A split GGUF
  (``NAME-00001-of-0000N.gguf``, formats.split_parts, formats.py:41-49) opens all parts; the metadata comes from the
  first, the tensors from whichever part holds them.
* ``rows(name)`` -- a 2-D or 3-D weight as packed rows ``[rows][row_bytes]`` uint8 (ggml's ne0 is the row length k;
  the expert tensors ``blk.N.ffn_{gate,up,down}_exps.weight`` [E][n][k] become ``E * n`` stacked rows, the layout of
  lk_moe_* -- expert e's rows start at e * n), without a copy. ``to_device`` copies one into device memory.
* ``mxfp4_planes(name)`` -- ggml's 17-byte MXFP4 blocks repacked at load time into the split planes the MXFP4 x FP8
  GEMMs read (nibble plane [rows][k/2], E8M0 plane [rows][k/32]); the nibbles keep ggml's split16 order
  (LK_ORDER_SPLIT16).
* ``moe_config(layer)`` -- the routing options of an MoE layer (gating, norm, scale, biases, act), derived as the
  reference's inspect_gguf.py:284-320 does, including its per-architecture defaults for what llama.cpp does not
  store in the file.

File format (the ggml project's GGUF specification, versions 2 and 3, little endian): magic ``GGUF``, u32 version,
u64 tensor count, u64 metadata count; metadata as (string key, u32 value type, value); tensor infos as (string name,
u32 n_dims, u64 dims[n_dims] with ne0 first, u32 ggml type, u64 offset); the tensor data after the infos, aligned to
``general.alignment`` (32 by default), each tensor at its offset from there.
"""
import os
import re
import struct

import numpy as np

# ggml type id -> (values per block, bytes per block); the formats the reference decodes (formats.py:5-17)
GGML_BLOCKS = {0: (1, 4), 1: (1, 2), 30: (1, 2), 2: (32, 18), 6: (32, 22), 8: (32, 34), 11: (256, 110),
               12: (256, 144), 13: (256, 176), 14: (256, 210), 20: (32, 18), 21: (256, 110), 23: (256, 136), 39: (32, 17)}
GGML_NAMES = {0: "f32", 1: "f16", 30: "bf16", 2: "q4_0", 6: "q5_0", 8: "q8_0", 11: "q3_k", 12: "q4_k", 13: "q5_k",
              14: "q6_k", 20: "iq4_nl", 21: "iq3_s", 23: "iq4_xs", 39: "mxfp4"}

# metadata value types (GGUF specification)
_SCALAR = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<?", 10: "<Q", 11: "<q", 12: "<d"}
_STRING, _ARRAY = 8, 9


def split_parts(path):
    """The files of a split GGUF (llama.cpp gguf-split: NAME-00001-of-00003.gguf ...), given the first part, in order;
    [path] for a single-file GGUF (formats.py:41-49)."""
    m = re.search(r"-(\d{5})-of-(\d{5})\.gguf$", path)
    if not m:
        return [path]
    n = int(m.group(2))
    return [f"{path[:m.start()]}-{i:05d}-of-{n:05d}.gguf" for i in range(1, n + 1)]


class GGUFError(ValueError):
    pass


class _Cursor:
    def __init__(self, buf):
        self.buf, self.pos = buf, 0

    def take(self, fmt):
        v = struct.unpack_from(fmt, self.buf, self.pos)[0]
        self.pos += struct.calcsize(fmt)
        return v

    def string(self):
        n = self.take("<Q")
        s = bytes(self.buf[self.pos:self.pos + n]).decode("utf-8", errors="replace")
        self.pos += n
        return s

    def value(self, vtype):
        if vtype in _SCALAR:
            return self.take(_SCALAR[vtype])
        if vtype == _STRING:
            return self.string()
        if vtype == _ARRAY:
            etype, count = self.take("<I"), self.take("<Q")
            if etype in _SCALAR and etype != 7:
                dt = np.dtype(_SCALAR[etype])
                arr = np.frombuffer(self.buf, dt, count, self.pos).copy()
                self.pos += dt.itemsize * count
                return arr.tolist()
            return [self.value(etype) for _ in range(count)]
        raise GGUFError(f"unknown metadata value type {vtype}")


class TensorInfo:
    """One tensor of a GGUF: ggml dims (ne0 first), type, and where its bytes are."""

    def __init__(self, name, dims, ggml_type, part, offset):
        self.name, self.dims, self.type, self.part, self.offset = name, tuple(dims), ggml_type, part, offset
        if ggml_type not in GGML_BLOCKS:
            self.qk = self.block_bytes = None
            self.nbytes = None
            return
        self.qk, self.block_bytes = GGML_BLOCKS[ggml_type]
        n = int(np.prod(self.dims))
        if n % self.qk or self.dims[0] % self.qk:
            raise GGUFError(f"{name}: {self.dims} is not a whole number of {self.qk}-value blocks per row")
        self.nbytes = n // self.qk * self.block_bytes

    @property
    def format(self):
        return GGML_NAMES.get(self.type, f"ggml_type_{self.type}")

    @property
    def shape(self):
        """Row-major shape (the outermost dim first): [..., rows, k]."""
        return tuple(reversed(self.dims))

    @property
    def row_bytes(self):
        return self.dims[0] // self.qk * self.block_bytes

    def __repr__(self):
        return f"TensorInfo({self.name!r}, {self.format}, shape={self.shape})"


class GGUFFile:
    """A (possibly split) GGUF file opened read-only with its tensors memory-mapped."""

    def __init__(self, path):
        self.paths = split_parts(path)
        missing = [p for p in self.paths if not os.path.exists(p)]
        if missing:
            raise GGUFError(f"split GGUF: missing parts next to {path}: {[os.path.basename(p) for p in missing]}")
        self.maps, self.metadata, self.tensors, self.versions = [], {}, {}, []
        for part, p in enumerate(self.paths):
            mm = np.memmap(p, np.uint8, "r")
            self.maps.append(mm)
            self._parse(mm, part, first=part == 0)

    def _parse(self, mm, part, first):
        c = _Cursor(mm)
        if bytes(mm[:4]) != b"GGUF":
            raise GGUFError(f"{self.paths[part]}: not a GGUF file")
        c.pos = 4
        version = c.take("<I")
        if version not in (2, 3):
            raise GGUFError(f"{self.paths[part]}: GGUF version {version} (2 or 3 expected)")
        self.versions.append(version)
        n_tensors, n_kv = c.take("<Q"), c.take("<Q")
        meta = {}
        for _ in range(n_kv):
            key = c.string()
            meta[key] = c.value(c.take("<I"))
        if first:
            self.metadata = meta
        infos = []
        for _ in range(n_tensors):
            name = c.string()
            nd = c.take("<I")
            dims = [c.take("<Q") for _ in range(nd)]
            infos.append((name, dims, c.take("<I"), c.take("<Q")))
        align = int(meta.get("general.alignment", 32))
        data0 = (c.pos + align - 1) // align * align
        for name, dims, ty, off in infos:
            if name in self.tensors:
                raise GGUFError(f"tensor {name} appears twice")
            t = TensorInfo(name, dims, ty, part, data0 + off)
            if t.nbytes is not None and t.offset + t.nbytes > len(mm):
                raise GGUFError(f"{name}: data past the end of {self.paths[part]}")
            self.tensors[name] = t

    # ---------------------------------------------------------------------------------------------------------- data
    def raw(self, name):
        """The tensor's bytes as a flat read-only uint8 view of the mapped file."""
        t = self.tensors[name]
        if t.nbytes is None:
            raise GGUFError(f"{name}: ggml type {t.type} is not a format this library decodes")
        return self.maps[t.part][t.offset:t.offset + t.nbytes]

    def rows(self, name):
        """A weight as packed rows [rows][row_bytes] uint8 (every dim above ne0 folded into rows), no copy."""
        t = self.tensors[name]
        return self.raw(name).reshape(-1, t.row_bytes)

    def array(self, name):
        """A float tensor (f32 / f16 / bf16) as f32 of its row-major shape (a copy for f16 / bf16)."""
        t = self.tensors[name]
        raw = self.raw(name)
        if t.type == 0:
            return raw.view("<f4").reshape(t.shape)
        if t.type == 1:
            return raw.view("<f2").astype(np.float32).reshape(t.shape)
        if t.type == 30:
            return (raw.view("<u2").astype(np.uint32) << 16).view(np.float32).reshape(t.shape)
        raise GGUFError(f"{name} is {t.format}, not a float tensor")

    def to_device(self, name, device="cuda"):
        """rows(name) (or array(name) for float tensors) copied into a torch tensor on `device`."""
        import torch
        t = self.tensors[name]
        host = self.array(name) if t.type in (0, 1, 30) else self.rows(name)
        return torch.from_numpy(np.ascontiguousarray(host)).to(device)

    def mxfp4_planes(self, name):
        """ggml MXFP4 (17-byte blocks: E8M0 byte, 16 nibble bytes, element i low nibble / i + 16 high) repacked into
        (nibble plane [rows][k/2], E8M0 plane [rows][k/32]) for the MXFP4 x FP8 kernels, nibbles in split16 order."""
        t = self.tensors[name]
        if t.type != 39:
            raise GGUFError(f"{name} is {t.format}, not MXFP4")
        b = self.raw(name).reshape(-1, 17)
        rows = int(np.prod(t.shape[:-1]))
        return (np.ascontiguousarray(b[:, 1:]).reshape(rows, -1), np.ascontiguousarray(b[:, 0]).reshape(rows, -1))

    # ---------------------------------------------------------------------------------------------------------- config
    def field(self, key, default=None):
        return self.metadata.get(key, default)

    @property
    def arch(self):
        return self.field("general.architecture")

    def moe_config(self, layer=None):
        """The MoE routing of the model (inspect_gguf.py:284-320): experts, top-k (used), expert ffn width, gating
        (1 softmax, 2 sigmoid, 3 softmax of the picked biased logits), weight normalisation, expert_weights_scale,
        selection / router / expert biases, shared experts and their gate, fused gate/up, per-expert down scale.
        llama.cpp keeps some of these per architecture rather than in the file; those defaults are the reference's
        MOE_DEFAULTS table. None when the model has no experts."""
        arch = self.arch
        A = lambda k, d=None: self.field(f"{arch}.{k}", d)   # noqa: E731
        if not A("expert_count"):
            return None
        defaults = MOE_DEFAULTS.get(arch, {})
        ld = A("leading_dense_block_count", 0)
        li = ld if layer is None else layer
        has = lambda s: f"blk.{li}.{s}" in self.tensors   # noqa: E731
        cfg = {"experts": A("expert_count"), "used": A("expert_used_count"), "ffn": A("expert_feed_forward_length"),
               "leading_dense": ld, "gating": A("expert_gating_func", defaults.get("gating", 1)),
               "norm_weights": bool(A("expert_weights_norm", defaults.get("norm_weights", False))),
               "scale": A("expert_weights_scale", 1.0) or 1.0,
               "probs_bias": has("exp_probs_b.bias"), "router_bias": has("ffn_gate_inp.bias"),
               "expert_bias": all(has(f"ffn_{p}_exps.bias") for p in ("gate", "up", "down")),
               "gate_up_fused": has("ffn_gate_up_exps.weight"), "down_scale": has("ffn_down_exps.scale"),
               "shared_gate": has("ffn_gate_inp_shexp.weight")}
        cfg.update({k: v for k, v in defaults.items() if k in ("act", "swiglu_alpha", "swiglu_limit")})
        return cfg


# llama.cpp's per-architecture MoE routing (build_moe_ffn's norm_w and gating in src/models/<arch>.cpp), as the
# reference records it in inspect_gguf.py:287-291
MOE_DEFAULTS = {"qwen3moe": {"gating": 1, "norm_weights": True}, "qwen35moe": {"gating": 1, "norm_weights": True},
                "qwen3next": {"gating": 1, "norm_weights": True}, "qwen2moe": {"gating": 1, "norm_weights": False},
                "gemma4": {"gating": 1, "norm_weights": True}, "mellum": {"gating": 1, "norm_weights": True},
                "gpt-oss": {"gating": 3, "norm_weights": False, "act": "swiglu_oai", "swiglu_alpha": 1.702,
                            "swiglu_limit": 7.0}}
