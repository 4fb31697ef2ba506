"""Writes the golden fixtures under tests/golden/ from the reference itself, run in this container.

  python tests/golden/make_golden.py [--ref <reference checkout>]

Sources (nothing here is restated; every output comes from the reference's own code):
  * llama/run.py quantize4                    -> quantize4.npz        (int4 packer, G=64, max/7)
  * qwen3moe/reference.py Weights.int4        -> int4_dequant_g*.npz  (word-layout dequantiser)
  * lfm2/weights.py dequant_q4_0              -> q4_0_dequant.npz     (GGUF Q4_0 dequantiser)
  * llama/st2bin.c (oracle/_ref/st2bin)       -> st2bin_q4.npz        (C packer, bf16 -> int4 G=64)
  * qwen3moe/convert.c (oracle/_ref/...)      -> qwen3moe_q4_g*.npz   (searched-scale packer)
  * lfm2/convert.c (oracle/_ref/lfm2_convert) -> lfm2_q4.npz          (GGUF Q4_0 -> words)
  * qwen3/convert.cpp addPacked (oracle/_ref/qwen3_pack) -> qwen3_pack.npz (ternary transpose)
  * transformers' Qwen3MoeSparseMoeBlock (the module qwen3moe/reference.py runs as its reference,
    :94-147), on int4 experts dequantised as Weights.int4 does -> moe_block.npz
Inputs are small seeded arrays with edge cases (all-zero groups, tiny and large magnitudes,
exact ties). The binaries are built by `make -C oracle`.
"""
import argparse
import os
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
BIN = os.path.join(REPO, "oracle", "_ref")


def _import(ref, sub, mod):
    sys.path.insert(0, os.path.join(ref, sub))
    try:
        return __import__(mod)
    finally:
        sys.path.pop(0)


def bf16_bits(a):
    """fp32 -> bf16 bit patterns (round to nearest even) and the bf16 values as fp32."""
    u = np.asarray(a, np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return r, (r.astype(np.uint32) << 16).view(np.float32)


def weights_with_edges(rng, rows, cols, group, std=0.02):
    w = rng.normal(0, std, size=(rows, cols)).astype(np.float32)
    w[0, :group] = 0.0                                   # an all-zero group
    w[1, :group] = rng.normal(0, 1e-6, size=group)       # tiny values (scale near fp16 subnormal)
    w[2, :group] = rng.normal(0, 30.0, size=group)       # large values
    w[3, :group] = np.tile([0.5, -0.5, 0.25, -0.25], group // 4)  # many exact ties
    w[4, group:2 * group] = 7.0                          # constant group (max = every element)
    w[5, 5] = -1.0                                       # lone outlier
    return w


def run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    return r.returncode, r.stdout + r.stderr


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("MQ_REFERENCE"),
                    help="the reference tree (default: $MQ_REFERENCE)")
    a = ap.parse_args()
    if not a.ref:
        ap.error("give the reference tree with --ref or MQ_REFERENCE")
    ref = a.ref
    rng = np.random.default_rng(1234)
    os.environ.setdefault("PYTHONDONTWRITEBYTECODE", "1")

    # --- llama/run.py quantize4 -------------------------------------------------------------
    import torch
    llama_run = _import(ref, "llama", "run")
    w16 = weights_with_edges(rng, 12, 256, 64).astype(np.float16)
    packed, s16, deq = llama_run.quantize4(torch.from_numpy(w16))
    np.savez(os.path.join(HERE, "quantize4.npz"), w16=w16, packed=packed, s16=s16, deq=deq, group=64)

    # --- qwen3moe/reference.py Weights.int4 ---------------------------------------------------
    qref = _import(ref, "qwen3moe", "reference")
    for g in (32, 64, 128):
        rows, cols = 24, 512
        wq = rng.integers(0, 1 << 32, size=(rows, cols // 8), dtype=np.uint32)
        ws = np.abs(rng.normal(0, 0.02, size=(rows, cols // g))).astype(np.float16)
        ws[0, 0] = 0.0
        ws[1, 0] = np.float16(6e-8)  # fp16 subnormal scale
        blob = wq.tobytes() + ws.tobytes()
        obj = qref.Weights.__new__(qref.Weights)
        obj.bf16 = False
        obj.bin = np.frombuffer(blob, np.uint8)
        obj.man = {"m.q": (0, wq.nbytes, "u32", [rows, cols // 8]),
                   "m.s": (wq.nbytes, ws.nbytes, "f16", [rows, cols // g])}
        deq = obj.int4("m").numpy()
        deq_part = obj.int4("m", 3, 5).numpy()
        np.savez(os.path.join(HERE, f"int4_dequant_g{g}.npz"), wq=wq, ws=ws, deq=deq, deq_rows_3_8=deq_part, group=g)

    # --- lfm2/weights.py dequant_q4_0 ----------------------------------------------------------
    lw = _import(ref, "lfm2", "weights")
    rows, cols = 6, 128
    d = np.abs(rng.normal(0, 0.02, size=rows * cols // 32)).astype(np.float16)
    d[0] = 0
    qs = rng.integers(0, 256, size=(rows * cols // 32, 16), dtype=np.uint8)
    blocks = np.concatenate([d.view(np.uint8).reshape(-1, 2), qs], axis=1)
    deq = lw.dequant_q4_0(blocks.tobytes(), rows, cols)
    np.savez(os.path.join(HERE, "q4_0_dequant.npz"), blocks=blocks, deq=deq, rows=rows, cols=cols)

    with tempfile.TemporaryDirectory() as tmp:
        # --- llama/st2bin.c: bf16 -> int4, G=64 ------------------------------------------------
        rows, cols = 10, 256
        bits, vals = bf16_bits(weights_with_edges(rng, rows, cols, 64))
        src = os.path.join(tmp, "model.safetensors")
        bits.tofile(src)
        qbytes, sbytes = rows * cols // 2, rows * cols // 64 * 2
        recipe = os.path.join(tmp, "recipe")
        with open(recipe, "w") as f:
            f.write(f"size {qbytes + sbytes}\nq4 0 {qbytes} 0 {rows} {cols}\n")
        out = os.path.join(tmp, "w.bin")
        rc, msg = run([os.path.join(BIN, "st2bin"), src, recipe, tmp, out])
        assert rc == 0, msg
        raw = np.fromfile(out, np.uint8)
        np.savez(os.path.join(HERE, "st2bin_q4.npz"), bf16=bits, words=raw[:qbytes].view(np.uint32).reshape(rows, cols // 8),
                 scales=raw[qbytes:].view(np.float16).reshape(rows, cols // 64), group=64)

        # --- qwen3moe/convert.c: searched scale, G = 32 / 64 / 128 ------------------------------
        for g in (32, 64, 128):
            rows, cols = 8, 512
            bits, vals = bf16_bits(weights_with_edges(rng, rows, cols, g))
            shard = os.path.join(tmp, "shard.bin")
            bits.tofile(shard)
            qbytes, sbytes = rows * cols // 2, rows * cols // g * 2
            with open(recipe, "w") as f:
                f.write(f"size {qbytes + sbytes}\nsrc shard.bin\nq4 0 {qbytes} 0 {rows} {cols} {g}\n")
            out = os.path.join(tmp, "moe.bin")
            rc, msg = run([os.path.join(BIN, "qwen3moe_convert"), tmp, recipe, out])
            assert rc == 0, msg
            raw = np.fromfile(out, np.uint8)
            np.savez(os.path.join(HERE, f"qwen3moe_q4_g{g}.npz"), bf16=bits,
                     words=raw[:qbytes].view(np.uint32).reshape(rows, cols // 8),
                     scales=raw[qbytes:].view(np.float16).reshape(rows, cols // g), group=g)

        # --- lfm2/convert.c: GGUF Q4_0 blocks -> words + d ---------------------------------------
        rows, cols = 6, 256
        d = np.abs(rng.normal(0, 0.02, size=rows * cols // 32)).astype(np.float16)
        qs = rng.integers(0, 256, size=(rows * cols // 32, 16), dtype=np.uint8)
        blocks = np.concatenate([d.view(np.uint8).reshape(-1, 2), qs], axis=1)
        gguf = os.path.join(tmp, "m.gguf")
        blocks.tofile(gguf)
        qbytes, sbytes = rows * cols // 2, rows * cols // 32 * 2
        with open(recipe, "w") as f:
            f.write(f"size {qbytes + sbytes}\nq4 0 {rows} {cols} 0 {qbytes}\n")
        out = os.path.join(tmp, "lfm2.bin")
        rc, msg = run([os.path.join(BIN, "lfm2_convert"), gguf, recipe, out])
        assert rc == 0, msg
        raw = np.fromfile(out, np.uint8)
        np.savez(os.path.join(HERE, "lfm2_q4.npz"), blocks=blocks, words=raw[:qbytes].view(np.uint32).reshape(rows, cols // 8),
                 scales=raw[qbytes:qbytes + sbytes].view(np.float16).reshape(rows, cols // 32))

        # --- qwen3/convert.cpp addPacked: MLX 2-bit rows -> transposed words + scales ------------
        n, k = 40, 512
        r = rng.integers(0, 1 << 32, size=(n, k // 16), dtype=np.uint32)
        codes = (r & np.uint32(0x55555555)) + ((r >> np.uint32(1)) & np.uint32(0x55555555))
        scales = np.abs(rng.normal(0, 0.05, size=(n, k // 128))).astype(np.float16)
        biases = (-scales.astype(np.float32)).astype(np.float16)
        paths = [os.path.join(tmp, p) for p in ("c.u32", "s.f16", "b.f16")]
        for p, arr in zip(paths, (codes, scales, biases)):
            arr.tofile(p)
        rc, msg = run([os.path.join(BIN, "qwen3_pack"), *paths, str(n), str(k), tmp])
        assert rc == 0, msg
        raw = np.fromfile(os.path.join(tmp, "weights.bin"), np.uint8)
        wb = n * k // 16 * 4
        bad = biases.copy()
        bad[3, 1] = np.float16(0.5)
        bad.tofile(paths[2])
        rc_bad, msg_bad = run([os.path.join(BIN, "qwen3_pack"), *paths, str(n), str(k), tmp])
        np.savez(os.path.join(HERE, "qwen3_pack.npz"), codes=codes, scales=scales, biases=biases,
                 w=raw[:wb].view(np.uint32).reshape(k // 16, n), s=raw[wb:].view(np.float16).reshape(k // 128, n),
                 bad_biases=bad, bad_rc=rc_bad, bad_msg=msg_bad.strip())
    # --- the MoE block of transformers on dequantised int4 experts -------------------------------
    from transformers import Qwen3MoeConfig
    from transformers.models.qwen3_moe import modeling_qwen3_moe as qm
    d, fe, experts, topk, tokens, g = 256, 256, 8, 2, 24, 32
    cfg = Qwen3MoeConfig(hidden_size=d, num_experts=experts, num_experts_per_tok=topk, moe_intermediate_size=fe,
                         norm_topk_prob=True, intermediate_size=4 * d, num_attention_heads=4, num_key_value_heads=2,
                         head_dim=64)
    block = qm.Qwen3MoeSparseMoeBlock(cfg).eval()
    gu_wq = rng.integers(0, 1 << 32, size=(experts * 2 * fe, d // 8), dtype=np.uint32)
    gu_ws = np.abs(rng.normal(0, 0.02, size=(experts * 2 * fe, d // g))).astype(np.float16)
    dn_wq = rng.integers(0, 1 << 32, size=(experts * d, fe // 8), dtype=np.uint32)
    dn_ws = np.abs(rng.normal(0, 0.02, size=(experts * d, fe // g))).astype(np.float16)
    router = rng.normal(0, 0.1, size=(experts, d)).astype(np.float32)
    x = rng.standard_normal((tokens, d)).astype(np.float32)

    def deq(wq, ws, rows, cols):  # Weights.int4 of qwen3moe/reference.py:53-65 on the same words
        obj = qref.Weights.__new__(qref.Weights)
        obj.bin = np.frombuffer(wq.tobytes() + ws.tobytes(), np.uint8)
        obj.man = {"m.q": (0, wq.nbytes, "u32", [rows, cols // 8]), "m.s": (wq.nbytes, ws.nbytes, "f16", [rows, cols // g])}
        return obj.int4("m")

    with torch.no_grad():
        block.experts.gate_up_proj.copy_(deq(gu_wq, gu_ws, experts * 2 * fe, d).reshape(experts, 2 * fe, d))
        block.experts.down_proj.copy_(deq(dn_wq, dn_ws, experts * d, fe).reshape(experts, d, fe))
        block.gate.weight.copy_(torch.from_numpy(router))
        xt = torch.from_numpy(x)
        _, w_sel, ids_sel = block.gate(xt)
        y = block(xt[None])[0]
    np.savez(os.path.join(HERE, "moe_block.npz"), x=x, router=router, logits=x @ router.T, gu_wq=gu_wq, gu_ws=gu_ws,
             dn_wq=dn_wq, dn_ws=dn_ws, ids=ids_sel.numpy().astype(np.int32), weights=w_sel.numpy().astype(np.float32),
             y=y.numpy(), d=d, fe=fe, experts=experts, topk=topk, group=g)
    print("fixtures written to", HERE)


if __name__ == "__main__":
    main()
