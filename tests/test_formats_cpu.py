"""On-disk formats on CPU: the GGUF reader against the reference's own reader's view of the same
file (tests/golden/gguf_small.json, made by make_gguf.py with lfm2/gguf_read.py), and the two
manifest formats (llama/run.py, qwen3moe/export.py)."""
import json
import os

import numpy as np
import pytest

from conftest import GOLDEN

from mq.formats import GGML_TYPES, GGUF, Manifest
from mq import MQError


def test_gguf_matches_reference_reader():
    ref = json.load(open(os.path.join(GOLDEN, "gguf_small.json")))
    g = GGUF(os.path.join(GOLDEN, "small.gguf"))
    assert g.version == ref["version"] and g.data_start == ref["data_start"]
    assert list(g.tensors) == [t["name"] for t in ref["tensors"]]
    for t in ref["tensors"]:
        mine = g.tensors[t["name"]]
        for key in ("dims", "type", "offset", "type_name", "nbytes", "abs"):
            assert mine[key] == t[key], (t["name"], key)
    assert list(g.metadata) == list(ref["metadata"])
    for key, want in ref["metadata"].items():
        got = g.metadata[key]
        got = [x.item() for x in got] if isinstance(got, np.ndarray) else got
        assert got == pytest.approx(want) if isinstance(want, (float, list)) else got == want, key


def test_gguf_q4_0_blocks_are_where_the_table_says():
    g = GGUF(os.path.join(GOLDEN, "small.gguf"))
    t = g.tensors["w.q4_0"]
    raw = open(os.path.join(GOLDEN, "small.gguf"), "rb").read()[t["abs"]:t["abs"] + t["nbytes"]]
    blocks = np.frombuffer(raw, np.uint8).reshape(-1, 18)
    assert blocks.shape[0] == 3 * 64 // 32
    assert (blocks[:, :2].copy().view(np.float16) == np.float16(0.03)).all()
    assert GGML_TYPES[t["type"]][0] == "Q4_0"


def test_gguf_rejects_other_files(tmp_path):
    p = tmp_path / "x.bin"
    p.write_bytes(b"GGML" + bytes(60))
    with pytest.raises(MQError, match="not a GGUF"):
        GGUF(str(p))
    raw = open(os.path.join(GOLDEN, "small.gguf"), "rb").read()
    p.write_bytes(raw[:100])
    with pytest.raises(MQError, match="truncated"):
        GGUF(str(p))


def test_manifest_llama_format(tmp_path):
    p = tmp_path / "manifest.txt"
    p.write_text("llama 2048 16 32 8 64 8192 128256 4096 8\nembed.0 0 512\nl0.wqkv.q 512 4096\n"
                 "l0.wqkv.s 4608 256\nrope.cos 4864 1024\n")
    m = Manifest(str(p))
    assert m.header[0] == "llama" and int(m.header[1]) == 2048
    assert m.entries["embed.0"] == dict(offset=0, nbytes=512, dtype="f16", shape=None)
    assert m.entries["l0.wqkv.q"]["dtype"] == "u32"
    assert m.entries["l0.wqkv.s"]["dtype"] == "f16"
    assert m.entries["rope.cos"]["dtype"] == "f32"


def test_manifest_qwen3moe_format(tmp_path):
    p = tmp_path / "manifest.txt"
    p.write_text("qwen3moe Qwen/Qwen3-30B-A3B@abcdef12 2048 48 32 4 128 128 8 768 151936\n"
                 "l0.experts.gu.q 0 3145728 u32 196608x16\nl0.experts.gu.s 3145728 98304 f16 196608x2\n"
                 "l0.router 3244032 1048576 f32 128x2048\n")
    m = Manifest(str(p))
    assert m.entries["l0.experts.gu.q"] == dict(offset=0, nbytes=3145728, dtype="u32", shape=[196608, 16])
    assert m.entries["l0.router"]["shape"] == [128, 2048]
    p.write_text("x\nbad 1 2 q7 3\n")
    with pytest.raises(MQError, match="unknown dtype"):
        Manifest(str(p))
