"""Writes tests/golden/small.gguf (a small seeded GGUF file, written here from the format's
definition) and tests/golden/gguf_small.json, the file as the reference's own reader
(lfm2/gguf_read.py parse, imported from the reference checkout) sees it: version, metadata, tensor
table (dims, type, offset, type name, bytes, absolute offset) and data start.

  python tests/golden/make_gguf.py [--ref <reference checkout>]

The file covers every metadata type (numeric arrays below and above 64 entries, string arrays),
a non-default alignment, and F32 / F16 / Q4_0 / BF16 / Q6_K tensors; the Q4_0 tensors hold seeded
random blocks with a fixed fp16 scale.
"""
import argparse
import json
import os
import struct
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ALIGN = 64


def _s(b):
    return struct.pack("<Q", len(b)) + b


def _value(t, v):
    scalar = {0: "B", 1: "b", 2: "H", 3: "h", 4: "I", 5: "i", 6: "f", 7: "?", 10: "Q", 11: "q", 12: "d"}
    if t in scalar:
        return struct.pack("<" + scalar[t], v)
    if t == 8:
        return _s(v.encode())
    et, items = v
    return struct.pack("<IQ", et, len(items)) + b"".join(_value(et, x) for x in items)


def write(path):
    rng = np.random.default_rng(42)
    meta = [("general.architecture", 8, "lfm2"), ("general.alignment", 4, ALIGN), ("t.u8", 0, 200), ("t.i8", 1, -7),
            ("t.u16", 2, 60000), ("t.i16", 3, -1234), ("t.u32", 4, 4000000000), ("t.i32", 5, -123456),
            ("t.f32", 6, 1.5), ("t.bool", 7, True), ("t.u64", 10, 2 ** 40 + 3), ("t.i64", 11, -(2 ** 40)),
            ("t.f64", 12, 0.1), ("t.small_u32", 9, (4, [1, 2, 3])), ("t.big_i32", 9, (5, list(range(-50, 50)))),
            ("t.big_f32", 9, (6, [float(x) for x in np.linspace(0, 1, 80, dtype=np.float32)])),
            ("t.strings", 9, (8, ["a", "bb", "é"])), ("t.u16s", 9, (2, [1, 65535]))]
    d = np.float16(0.03).tobytes()
    q4 = lambda nb: b"".join(d + rng.integers(0, 256, 16, dtype=np.uint8).tobytes() for _ in range(nb))  # noqa: E731
    tensors = [("w.f32", [4, 3], 0, rng.standard_normal(12).astype(np.float32).tobytes()),
               ("w.f16", [8], 1, rng.standard_normal(8).astype(np.float16).tobytes()),
               ("w.q4_0", [64, 3], 2, q4(2 * 3)),
               ("w.bf16", [16], 30, rng.integers(0, 65536, 16, dtype=np.uint16).tobytes()),
               ("w.q6_k", [256], 14, rng.integers(0, 256, 210, dtype=np.uint8).tobytes()),
               ("w.q4_0_big", [256, 40], 2, q4(8 * 40))]
    head = b"GGUF" + struct.pack("<IQQ", 3, len(tensors), len(meta))
    for k, t, v in meta:
        head += _s(k.encode()) + struct.pack("<I", t) + _value(t, v)
    data, offs = b"", []
    for _, _, _, raw in tensors:
        data += b"\0" * (-len(data) % ALIGN)
        offs.append(len(data))
        data += raw
    for (name, dims, t, _), off in zip(tensors, offs):
        head += _s(name.encode()) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", x) for x in dims)
        head += struct.pack("<IQ", t, off)
    head += b"\0" * (-len(head) % ALIGN)
    with open(path, "wb") as f:
        f.write(head + data)


def _plain(v):
    if isinstance(v, np.ndarray):
        return [x.item() for x in v]
    if isinstance(v, list):
        return [_plain(x) for x in v]
    return v


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("MQ_REFERENCE"),
                    help="the reference tree (default: $MQ_REFERENCE)")
    a = ap.parse_args()
    if not a.ref:
        ap.error("give the reference tree with --ref or MQ_REFERENCE")
    path = os.path.join(HERE, "small.gguf")
    write(path)
    sys.path.insert(0, os.path.join(a.ref, "lfm2"))
    import gguf_read  # the reference's reader

    with open(path, "rb") as f:
        ver, meta, tensors, data_start = gguf_read.parse(f.read())
    out = dict(version=ver, metadata={k: _plain(v) for k, v in meta.items()}, data_start=data_start,
               tensors=[dict(name=t["name"], dims=t["dims"], type=t["type"], offset=t["offset"], type_name=t["tname"],
                             nbytes=t["nbytes"], abs=t["abs"]) for t in tensors])
    with open(os.path.join(HERE, "gguf_small.json"), "w") as f:
        json.dump(out, f, indent=1)
    print(f"small.gguf: {os.path.getsize(path)} bytes, {len(tensors)} tensors")


if __name__ == "__main__":
    main()
