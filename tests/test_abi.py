"""The C ABI without a GPU: libmq.so loads, exports every entry point include/mq.h declares, and
rejects bad arguments with a status and a message before touching a device."""
import ctypes
import os
import re

import pytest

from conftest import REPO

HEADER = os.path.join(REPO, "include", "mq.h")


def declared():
    text = open(HEADER).read()
    return re.findall(r"MQ_API\s+[\w\s\*]*?\b(mq_\w+)\s*\(", text)


def test_header_and_signatures_agree():
    from mq._lib import SIGNATURES

    names = declared()
    assert names, "no MQ_API declarations found"
    assert sorted(names) == sorted(SIGNATURES), "mq/_lib.py SIGNATURES must list exactly include/mq.h's entry points"


def test_library_exports_every_declared_symbol():
    from mq._lib import lib, library_path

    assert os.path.exists(library_path), "build libmq.so first (python mojo-adreno_b200/build.py)"
    dll = ctypes.CDLL(library_path)
    missing = [n for n in declared() if not hasattr(dll, n)]
    assert not missing, f"not exported: {missing}"
    assert lib.mq_version() >= 100


def _status(name, *args):
    from mq._lib import lib

    rc = getattr(lib, name)(*args)
    return rc, lib.mq_last_error().decode()


def test_gemv_rejects_bad_arguments_before_launch():
    P = ctypes.c_void_p
    ok = P(1 << 20)  # never dereferenced: validation fails first
    rc, msg = _status("mq_gemv_q4", None, ok, ok, 0, ok, 16, 256, 32, 1, 0, None)
    assert rc == -1 and "null" in msg
    rc, msg = _status("mq_gemv_q4", ok, ok, ok, 0, ok, 16, 256, 48, 1, 0, None)
    assert rc == -1 and "group" in msg
    rc, msg = _status("mq_gemv_q4", ok, ok, ok, 0, ok, 16, 200, 32, 1, 0, None)
    assert rc == -1 and "multiple" in msg
    rc, msg = _status("mq_gemv_q4", ok, ok, ok, 0, ok, 16, 256, 32, 0, 0, None)
    assert rc == -1 and "batch" in msg
    rc, msg = _status("mq_gemv_q4", P((1 << 20) + 4), ok, ok, 0, ok, 16, 256, 32, 1, 0, None)
    assert rc == -2 and "aligned" in msg


def test_tgemv_rejects_bad_arguments_before_launch():
    P = ctypes.c_void_p
    ok = P(1 << 20)
    rc, msg = _status("mq_tgemv", ok, ok, ok, ok, 64, 200, 1, None)
    assert rc == -1 and "128" in msg
    rc, msg = _status("mq_tgemv", ok, ok, ok, ok, 0, 256, 1, None)
    assert rc == -1 and "shape" in msg
    rc, msg = _status("mq_tgemv", P((1 << 20) + 4), ok, ok, ok, 66, 256, 1, None)
    assert rc == -2 and "aligned" in msg
    rc, msg = _status("mq_tgemv", ok, ok, ok, ok, 64, 256, 5, None)
    assert rc == -1 and "batch" in msg


def test_fused_epilogues_reject_bad_arguments_before_launch():
    P = ctypes.c_void_p
    ok = P(1 << 20)
    rc, msg = _status("mq_gate_up_q4", ok, ok, ok, 0, ok, 40, 256, 32, 1, None)
    assert rc == -1 and "multiple of 16" in msg
    rc, msg = _status("mq_gate_up_q4", ok, ok, ok, 0, ok, 48, 256, 32, 5, None)
    assert rc == -1 and "batch" in msg
    rc, msg = _status("mq_moe_gate_up_q4", ok, ok, 96, ok, ok, ok, 2, 40, 256, 32, None)
    assert rc == -1 and "fe" in msg
    rc, msg = _status("mq_tgemv_head", ok, ok, ok, ok, None, 64, 256, 1, None)
    assert rc == -1 and "candidates" in msg
    rc, msg = _status("mq_head_argmax", ok, 0, 1, ok, None)
    assert rc == -1 and "ncand" in msg


def test_packers_and_ep_plan_reject_bad_arguments_before_launch():
    P = ctypes.c_void_p
    ok = P(1 << 20)
    rc, msg = _status("mq_quantize_q4", ok, 0, 4, 256, 48, 0, ok, ok, None)
    assert rc == -1 and "group" in msg
    rc, msg = _status("mq_quantize_q4", ok, 5, 4, 256, 32, 0, ok, ok, None)
    assert rc == -1 and "w_dtype" in msg
    rc, msg = _status("mq_quantize_q4", ok, 0, 4, 256, 32, 2, ok, ok, None)
    assert rc == -1 and "method" in msg
    rc, msg = _status("mq_q4_0_to_words", P((1 << 20) + 1), 4, ok, ok, None)
    assert rc == -2 and "aligned" in msg
    rc, msg = _status("mq_pack_ternary", ok, ok, None, 4, 200, ok, ok, None)
    assert rc == -1 and "128" in msg
    rc, msg = _status("mq_pack_half", ok, ok, 7, None)
    assert rc == -1 and "even" in msg
    rc, msg = _status("mq_ep_plan", ok, 4, 8, 128, 3, 0, ok, ok, ok, ok, ok, None)
    assert rc == -1 and "multiple of world" in msg


def test_python_ops_refuse_cpu_tensors():
    import torch

    import mq

    wq = torch.zeros(16, 32, dtype=torch.int32)
    ws = torch.zeros(16, 8, dtype=torch.float16)
    x = torch.zeros(1, 256)
    y = torch.zeros(1, 16)
    with pytest.raises(mq.MQError, match="CUDA"):
        mq.gemv_q4(wq, ws, x, y, 256, group=32)


def test_router_chain_and_layer_reject_bad_arguments_before_launch():
    P = ctypes.c_void_p
    ok = P(1 << 20)
    # mq_moe_route_group(w, x, logits, ids, weights, tokens, experts, topk, d, tile, counts, offsets, order,
    #                    slot_of, tiles, ntiles, stream)
    rc, msg = _status("mq_moe_route_group", None, ok, None, ok, ok, 4, 128, 8, 2048, 64, None, None, None, None, None,
                      None, None)
    assert rc == -1 and "null" in msg
    rc, msg = _status("mq_moe_route_group", ok, ok, None, ok, ok, 4, 300, 8, 2048, 64, None, None, None, None, None,
                      None, None)
    assert rc == -1 and "experts" in msg
    rc, msg = _status("mq_moe_route_group", ok, ok, None, ok, ok, 4, 128, 8, 2050, 64, None, None, None, None, None,
                      None, None)
    assert rc == -1 and "multiple of 4" in msg
    rc, msg = _status("mq_moe_route_group", ok, ok, None, ok, ok, 4, 128, 8, 2048, 64, ok, None, None, None, None,
                      None, None)
    assert rc == -1 and "grouping outputs" in msg
    rc, msg = _status("mq_moe_route_group", P((1 << 20) + 4), ok, None, ok, ok, 4, 128, 8, 2048, 64, None, None, None,
                      None, None, None, None)
    assert rc == -2 and "aligned" in msg
    # mq_moe_layer(x, router_w, gu_wq, gu_ws, dn_wq, dn_ws, y, ids, weights, logits, tokens, experts, topk, d, fe,
    #              group, add, workspace, bytes, stream)
    rc, msg = _status("mq_moe_layer", ok, ok, ok, ok, ok, ok, ok, ok, ok, None, 4, 128, 8, 2048, 700, 32, 0, ok, 1 << 30,
                      None)
    assert rc == -1 and "multiples of 256" in msg
    rc, msg = _status("mq_moe_layer", ok, ok, ok, ok, ok, ok, ok, ok, ok, None, 4, 128, 8, 2048, 768, 32, 0, ok, 16,
                      None)
    assert rc == -1 and "workspace" in msg
