"""tcgen05 int4 GEMM parity on the GPU through the C ABI: the kernel against the oracle (float64 on
the reference's dequantised weights and the same x). The product rounds x and q*scale to fp16 once
each and accumulates in fp32, so the bar is the north star's normwise 1e-3 and ~1e-4 is expected."""
import numpy as np
import pytest
import torch

from conftest import normwise
from oracle import q4

import mq
from mq import synth

pytestmark = pytest.mark.gpu
TOL = 1e-3


def run(cuda, wq, ws, x, group, add_to=None):
    n, k = wq.shape[0], wq.shape[1] * 8
    m = x.shape[0]
    twq = torch.from_numpy(wq.view(np.int32)).to(cuda)
    tws = torch.from_numpy(ws).to(cuda)
    tx = torch.from_numpy(x).to(cuda)
    ty = torch.full((m, n), float("nan"), device=cuda) if add_to is None else torch.from_numpy(add_to).to(cuda)
    mq.p_gemm_q4(twq, tws, tx, ty, n, k, m, group=group, add=add_to is not None)
    torch.cuda.synchronize()
    assert mq.device_status() == 0
    return ty.cpu().numpy()


def ref(wq, ws, x, group):
    return q4.gemv(wq, ws, x.astype(np.float32), group)


@pytest.mark.parametrize("n,k,m", [(128, 256, 16), (128, 256, 1), (256, 512, 40), (130, 256, 17), (384, 768, 300)])
@pytest.mark.parametrize("group", [32, 64, 128])
def test_gemm_small(cuda, n, k, m, group):
    rng = np.random.default_rng(n + k + m + group)
    x = rng.standard_normal((m, k)).astype(np.float16)
    wq, ws = synth.q4_matrix(rng, n, k, group)
    y = run(cuda, wq, ws, x, group)
    assert np.isfinite(y).all()
    assert normwise(y, ref(wq, ws, x, group)) <= TOL


def test_gemm_extra_token_tile(cuda):
    """512 tokens over 12288 rows: three token tiles of 176 (288 CTAs in two full waves) instead of two
    of 256 (192 CTAs, a wave and a third)."""
    rng = np.random.default_rng(512)
    x = rng.standard_normal((512, 512)).astype(np.float16)
    wq, ws = synth.q4_matrix(rng, 12288, 512, 32)
    y = run(cuda, wq, ws, x, 32)
    assert normwise(y, ref(wq, ws, x, 32)) <= TOL


@pytest.mark.parametrize("name", ["gate_up", "down", "qkv"])
def test_gemm_prefill_config(cuda, name):
    """Llama-3.2-1B prefill shapes, 431 tokens, Q4_0 G=32, fp16 X."""
    x, wq, ws = synth.prefill(seed=0)[name]
    y = run(cuda, wq, ws, x, 32)
    err = normwise(y, ref(wq, ws, x, 32))
    assert err <= TOL, err


def test_gemm_fp32_x_workspace_and_add(cuda):
    rng = np.random.default_rng(3)
    n, k, m = 1024, 2048, 96
    x = rng.standard_normal((m, k)).astype(np.float32)
    wq, ws = synth.q4_matrix(rng, n, k, 32)
    r = rng.standard_normal((m, n)).astype(np.float32)
    y = run(cuda, wq, ws, x, 32, add_to=r.copy())
    assert normwise(y, r + ref(wq, ws, x, 32)) <= TOL


def test_gemm_split_k(cuda):
    """Few output tiles and a long K: the launcher splits K across CTAs (red.add into zeroed y)."""
    rng = np.random.default_rng(4)
    n, k, m = 256, 8192, 64
    x = rng.standard_normal((m, k)).astype(np.float16)
    wq, ws = synth.q4_matrix(rng, n, k, 32)
    y = run(cuda, wq, ws, x, 32)
    assert normwise(y, ref(wq, ws, x, 32)) <= TOL


@pytest.mark.parametrize("dtype", [np.float16, np.float32])
def test_gemv_batch64_routes_to_gemm(cuda, dtype):
    """BASELINE configs[1] batch 64: mq.gemv_q4 with batch > 4 runs the tensor-core GEMM."""
    rng = np.random.default_rng(5)
    n, k = 2048, 2048
    x = rng.standard_normal((64, k)).astype(dtype)
    wq, ws = synth.q4_matrix(rng, n, k, 32)
    ty = torch.full((64, n), float("nan"), device=cuda)
    mq.gemv_q4(torch.from_numpy(wq.view(np.int32)).to(cuda), torch.from_numpy(ws).to(cuda), torch.from_numpy(x).to(cuda),
               ty, k, group=32)
    torch.cuda.synchronize()
    assert normwise(ty.cpu().numpy(), ref(wq, ws, x, 32)) <= TOL
