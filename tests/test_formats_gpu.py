"""Weight files into device memory (mq_read_file_to_device), GGUF Q4_0 tensors through
mq_q4_0_to_words into the GEMV, and manifest exports loaded as typed device views."""
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN, normwise
from oracle import q4

import mq

pytestmark = pytest.mark.gpu


def test_read_file_to_device_round_trip(cuda, tmp_path):
    rng = np.random.default_rng(1)
    raw = rng.integers(0, 256, 20 * (1 << 20) + 12345, dtype=np.uint8)  # three staging chunks, ragged end
    p = tmp_path / "w.bin"
    p.write_bytes(raw.tobytes())
    for off, n in [(0, raw.size), (7, raw.size - 7), (1 << 20, 9 * (1 << 20) + 3), (5, 1), (0, 0)]:
        t = mq.read_file_to_device(str(p), off, n, device=cuda)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(t.cpu().numpy(), raw[off:off + n])


def test_read_file_to_device_errors(cuda, tmp_path):
    p = tmp_path / "w.bin"
    p.write_bytes(bytes(100))
    with pytest.raises(mq.MQError, match="range ends"):
        mq.read_file_to_device(str(p), 50, 60, device=cuda)
    with pytest.raises(mq.MQError, match="open") as e:
        mq.read_file_to_device(str(tmp_path / "missing.bin"), 0, 4, device=cuda)
    assert e.value.code == -6


def test_gguf_q4_0_into_the_gemv(cuda):
    """A GGUF Q4_0 matrix read from the file, converted on the device, multiplied: the same numbers as
    ggml's dequantisation (lfm2/weights.py:61-68) times x."""
    g = mq.GGUF(os.path.join(GOLDEN, "small.gguf"))
    t = g.tensors["w.q4_0_big"]
    cols, rows = t["dims"]
    wq, ws = g.q4_0_words("w.q4_0_big", device=cuda)
    raw = np.fromfile(os.path.join(GOLDEN, "small.gguf"), np.uint8)[t["abs"]:t["abs"] + t["nbytes"]]
    rw, rd = q4.q4_0_to_words(raw)
    np.testing.assert_array_equal(wq.cpu().numpy().view(np.uint32).reshape(-1), rw.reshape(-1))
    np.testing.assert_array_equal(ws.cpu().numpy().view(np.uint16).reshape(-1), rd.view(np.uint16))
    x = np.random.default_rng(2).standard_normal((1, cols)).astype(np.float32)
    y = torch.empty(1, rows, device=cuda)
    mq.gemv_q4(wq, ws, torch.from_numpy(x).to(cuda), y, cols, group=32)
    ref = q4.dequant_q4_0(raw, rows, cols).astype(np.float64) @ x[0].astype(np.float64)
    assert normwise(y.cpu().numpy()[0], ref) <= 1e-4


def test_gguf_other_types_arrive_byte_exact(cuda):
    g = mq.GGUF(os.path.join(GOLDEN, "small.gguf"))
    raw = np.fromfile(os.path.join(GOLDEN, "small.gguf"), np.uint8)
    for name in ("w.f32", "w.f16", "w.bf16", "w.q6_k"):
        t = g.tensors[name]
        np.testing.assert_array_equal(g.to_device(name, device=cuda).cpu().numpy(), raw[t["abs"]:t["abs"] + t["nbytes"]])


def test_manifest_load_typed_views(cuda, tmp_path):
    """weights.bin + manifest.txt in both export formats: every tensor a typed device view of its bytes."""
    rng = np.random.default_rng(3)
    words = rng.integers(0, 1 << 32, (64, 16), dtype=np.uint32)
    scales = rng.standard_normal((64, 4)).astype(np.float16)
    table = rng.standard_normal((8, 32)).astype(np.float32)
    blob, lines5, lines3 = b"", [], []
    for name, a, dt in (("m.q", words, "u32"), ("m.s", scales, "f16"), ("rope.cos", table, "f32")):
        blob += b"\0" * (-len(blob) % 256)
        lines5.append(f"{name} {len(blob)} {a.nbytes} {dt} {'x'.join(map(str, a.shape))}")
        lines3.append(f"{name} {len(blob)} {a.nbytes}")
        blob += a.tobytes()
    (tmp_path / "weights.bin").write_bytes(blob)
    for lines, shaped in ((lines5, True), (lines3, False)):
        (tmp_path / "manifest.txt").write_text("test 1 2 3\n" + "\n".join(lines) + "\n")
        m = mq.Manifest(str(tmp_path / "manifest.txt"))
        w = m.load(str(tmp_path / "weights.bin"), device=cuda)
        torch.cuda.synchronize()
        assert w["m.q"].dtype == torch.int32 and w["m.s"].dtype == torch.float16 and w["rope.cos"].dtype == torch.float32
        np.testing.assert_array_equal(w["m.q"].cpu().numpy().view(np.uint32).reshape(words.shape), words)
        np.testing.assert_array_equal(w["m.s"].cpu().numpy().reshape(scales.shape), scales)
        np.testing.assert_array_equal(w["rope.cos"].cpu().numpy().reshape(table.shape), table)
        if shaped:
            assert tuple(w["m.q"].shape) == words.shape
    part = m.load(str(tmp_path / "weights.bin"), names=["m.s"], device=cuda)
    np.testing.assert_array_equal(part["m.s"].cpu().numpy().reshape(scales.shape), scales)
