"""On-disk weight formats: GGUF (metadata, tensor table, Q4_0 tensors) and the reference's
manifest.txt + weights.bin exports, loaded into device memory with mq_read_file_to_device.

- GGUF: the reader of lfm2/gguf_read.py:5-73 (header, typed metadata, tensor infos, data start at
  the file's alignment, bytes per tensor from the ggml type's block size). A Q4_0 tensor goes to the
  device as its raw blocks and through mq_q4_0_to_words into the GEMV's word layout
  (lfm2/convert.c:58-71).
- Manifests: llama/run.py:109-183 (header line, then `name offset nbytes`, 256-byte aligned) and
  qwen3moe/export.py:78-81,135 (`name offset nbytes dtype RxC`, 4096-byte aligned), read as
  qwen3moe/model.mojo:130-163 does: a device buffer per line, filled from the weights file.
"""
import ctypes
import os
import struct

import numpy as np
import torch

from ._lib import MQError, lib
from .pack import q4_0_to_words

__all__ = ["GGML_TYPES", "GGUF", "read_gguf", "Manifest", "read_file_to_device"]

# ggml tensor types: id -> (name, values per block, bytes per block), as the GGUF format defines them.
GGML_TYPES = {0: ("F32", 1, 4), 1: ("F16", 1, 2), 2: ("Q4_0", 32, 18), 3: ("Q4_1", 32, 20), 6: ("Q5_0", 32, 22),
              7: ("Q5_1", 32, 24), 8: ("Q8_0", 32, 34), 10: ("Q2_K", 256, 84), 11: ("Q3_K", 256, 110),
              12: ("Q4_K", 256, 144), 13: ("Q5_K", 256, 176), 14: ("Q6_K", 256, 210), 30: ("BF16", 1, 2)}

# GGUF metadata value types with a fixed-size little-endian encoding.
_SCALAR = {0: "B", 1: "b", 2: "H", 3: "h", 4: "I", 5: "i", 6: "f", 7: "?", 10: "Q", 11: "q", 12: "d"}
_NUMPY = {0: "<u1", 1: "<i1", 2: "<u2", 3: "<i2", 4: "<u4", 5: "<i4", 6: "<f4", 10: "<u8", 11: "<i8", 12: "<f8"}
_STRING, _ARRAY = 8, 9


def read_file_to_device(path, offset, nbytes, out=None, device=None):
    """nbytes at `offset` of the file into a device uint8 tensor (or into `out`, any dtype, exactly
    nbytes): M_driver_remote_file of qwen3moe/model.mojo:156-158."""
    if out is None:
        out = torch.empty(nbytes, dtype=torch.uint8, device=device or torch.device("cuda"))
    if not out.is_cuda or not out.is_contiguous() or out.numel() * out.element_size() != nbytes:
        raise MQError(-1, "out: must be a contiguous CUDA tensor of exactly nbytes bytes")
    lib.call("mq_read_file_to_device", ctypes.c_void_p(out.data_ptr()), nbytes, os.fsencode(path), offset,
             ctypes.c_void_p(torch.cuda.current_stream(out.device).cuda_stream))
    return out


class _Cursor:
    def __init__(self, buf):
        self.buf, self.pos = buf, 0

    def take(self, fmt):
        size = struct.calcsize("<" + fmt)
        if self.pos + size > len(self.buf):
            raise MQError(-1, "gguf: truncated file")
        (v,) = struct.unpack_from("<" + fmt, self.buf, self.pos)
        self.pos += size
        return v

    def string(self):
        n = self.take("Q")
        if self.pos + n > len(self.buf):
            raise MQError(-1, "gguf: truncated string")
        v = bytes(self.buf[self.pos:self.pos + n]).decode("utf-8", "replace")
        self.pos += n
        return v

    def value(self, vtype):
        if vtype in _SCALAR:
            return self.take(_SCALAR[vtype])
        if vtype == _STRING:
            return self.string()
        if vtype == _ARRAY:
            etype, count = self.take("I"), self.take("Q")
            if etype in _NUMPY:  # numeric arrays in one step (token tables run to 10^5 entries)
                a = np.frombuffer(self.buf, dtype=_NUMPY[etype], count=count, offset=self.pos)
                self.pos += a.nbytes
                return a.copy()
            return [self.value(etype) for _ in range(count)]
        raise MQError(-1, f"gguf: unknown metadata type {vtype}")


class GGUF:
    """A parsed GGUF file: version, metadata (dict), tensors (name -> info dict with dims, type,
    type_name, offset, nbytes, abs = absolute file offset), data_start."""

    def __init__(self, path, header_bytes=None):
        self.path = path
        with open(path, "rb") as f:
            buf = f.read() if header_bytes is None else f.read(header_bytes)
        c = _Cursor(buf)
        if bytes(buf[:4]) != b"GGUF":
            raise MQError(-1, f"{path}: not a GGUF file")
        c.pos = 4
        self.version = c.take("I")
        n_tensors, n_kv = c.take("Q"), c.take("Q")
        self.metadata = {}
        for _ in range(n_kv):
            key = c.string()
            self.metadata[key] = c.value(c.take("I"))
        self.tensors = {}
        for _ in range(n_tensors):
            name = c.string()
            dims = [c.take("Q") for _ in range(c.take("I"))]
            ttype, offset = c.take("I"), c.take("Q")
            self.tensors[name] = dict(name=name, dims=dims, type=ttype, offset=offset)
        align = int(self.metadata.get("general.alignment", 32))
        self.data_start = -(-c.pos // align) * align
        for t in self.tensors.values():
            if t["type"] not in GGML_TYPES:
                raise MQError(-1, f"gguf: tensor {t['name']} has unknown type {t['type']}")
            tname, per_block, block_bytes = GGML_TYPES[t["type"]]
            n = int(np.prod(t["dims"], dtype=np.int64)) if t["dims"] else 1
            t["type_name"] = tname
            t["nbytes"] = n // per_block * block_bytes
            t["abs"] = self.data_start + t["offset"]

    def to_device(self, name, device=None):
        """The tensor's raw bytes as a device uint8 tensor."""
        t = self.tensors[name]
        return read_file_to_device(self.path, t["abs"], t["nbytes"], device=device)

    def q4_0_words(self, name, device=None):
        """A Q4_0 matrix [rows, cols] (GGUF dims = [cols, rows]) as the GEMV's int4 words and fp16
        scales: (wq int32 [rows, cols / 8], ws fp16 [rows, cols / 32])."""
        t = self.tensors[name]
        if t["type_name"] != "Q4_0" or len(t["dims"]) != 2:
            raise MQError(-1, f"{name}: {t['type_name']} {t['dims']}, expected a 2-D Q4_0 tensor")
        cols, rows = t["dims"]
        wq, ws = q4_0_to_words(self.to_device(name, device))
        return wq.view(rows, cols // 8), ws.view(rows, cols // 32)


def read_gguf(path):
    return GGUF(path)


_TORCH = {"u32": torch.int32, "i32": torch.int32, "f16": torch.float16, "f32": torch.float32, "u8": torch.uint8}


class Manifest:
    """manifest.txt of a weights.bin export. entries: name -> dict(offset, nbytes, dtype, shape).

    Lines of three fields (llama/run.py:128-136,177-181) carry no dtype: `.q` tensors are int4 words,
    `.s` their fp16 scales, `rope.*` fp32 tables, everything else fp16 (the export's choices).
    Lines of five fields (qwen3moe/export.py:80) give the dtype and the shape."""

    def __init__(self, path):
        with open(path) as f:
            lines = f.read().splitlines()
        if not lines:
            raise MQError(-1, f"{path}: empty manifest")
        self.header = lines[0].split()
        self.entries = {}
        for ln in lines[1:]:
            f = ln.split()
            if not f:
                continue
            if len(f) < 3:
                raise MQError(-1, f"{path}: bad line {ln!r}")
            name, off, nbytes = f[0], int(f[1]), int(f[2])
            if len(f) >= 4:
                dtype = f[3]
                shape = [int(v) for v in f[4].split("x")] if len(f) >= 5 else None
            else:
                dtype = "u32" if name.endswith(".q") else "f32" if name.startswith("rope.") else "f16"
                shape = None
            if dtype not in _TORCH:
                raise MQError(-1, f"{path}: {name} has unknown dtype {dtype}")
            self.entries[name] = dict(offset=off, nbytes=nbytes, dtype=dtype, shape=shape)

    def load(self, weights_path, names=None, device=None):
        """The tensors (all, or `names`) on the device: one read of the file range they span into one
        buffer, each tensor a typed view of it (the exports align every tensor to 256 bytes or more)."""
        names = list(self.entries) if names is None else list(names)
        if not names:
            return {}
        sel = [self.entries[n] for n in names]
        lo = min(e["offset"] for e in sel)
        hi = max(e["offset"] + e["nbytes"] for e in sel)
        buf = read_file_to_device(weights_path, lo, hi - lo, device=device)
        out = {}
        for n, e in zip(names, sel):
            dt = _TORCH[e["dtype"]]
            size = torch.tensor([], dtype=dt).element_size()
            if (e["offset"] - lo) % size or e["nbytes"] % size:
                raise MQError(-1, f"{n}: offset or size is not a whole number of {e['dtype']} elements")
            t = buf[e["offset"] - lo:e["offset"] - lo + e["nbytes"]].view(dt)
            out[n] = t.view(*e["shape"]) if e["shape"] else t
        return out
