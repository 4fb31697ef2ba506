"""Ternary prefill GEMM (p_gemm_t2) on the tcgen05 tensor cores against the float64 oracle on the
exact ternary matrix: normwise <= 1e-3 (x is rounded to fp16; the weights are exact in fp16)."""
import numpy as np
import pytest
import torch

from conftest import normwise
from oracle import ternary

import mq
from mq import synth

pytestmark = pytest.mark.gpu
TOL = 1e-3


def dense(w, s, n, k):
    c = ternary.codes(w, n, k).astype(np.float64) - 1.0
    return c * np.repeat(s.T.astype(np.float64), 128, axis=1)


@pytest.mark.parametrize("rows,n,k,xdt", [(128, 4096, 4096, np.float32), (37, 1000, 512, np.float32),
                                          (431, 2048, 1024, np.float16), (5, 132, 256, np.float32),
                                          (512, 12288, 512, np.float16)])  # 3 token tiles of 176 (wave fill)
def test_gemm_t2_matches_oracle(cuda, rows, n, k, xdt):
    rng = np.random.default_rng(rows + n + k)
    w, s = synth.ternary_matrix(rng, n, k)
    x = rng.standard_normal((rows, k)).astype(xdt)
    y = torch.full((rows, n), float("nan"), device=cuda)
    mq.p_gemm_t2(torch.from_numpy(x).to(cuda), torch.from_numpy(w.view(np.int32)).to(cuda), torch.from_numpy(s).to(cuda),
                 y, n, k)
    torch.cuda.synchronize()
    assert mq.device_status() == 0
    ref = x.astype(np.float64) @ dense(w, s, n, k).T
    assert normwise(y.cpu().numpy(), ref) <= TOL


def test_gemm_t2_add_and_fp16_x_exactness(cuda):
    """add accumulates into y; with fp16-representable x the only error is fp32 accumulation."""
    rng = np.random.default_rng(3)
    n, k, rows = 512, 1024, 64
    w, s = synth.ternary_matrix(rng, n, k)
    x = rng.standard_normal((rows, k)).astype(np.float16).astype(np.float32)
    base = rng.standard_normal((rows, n)).astype(np.float32)
    y = torch.from_numpy(base.copy()).to(cuda)
    mq.p_gemm_t2(torch.from_numpy(x).to(cuda), torch.from_numpy(w.view(np.int32)).to(cuda), torch.from_numpy(s).to(cuda),
                 y, n, k, add=True)
    torch.cuda.synchronize()
    ref = base + x.astype(np.float64) @ dense(w, s, n, k).T
    assert normwise(y.cpu().numpy(), ref) <= 1e-5
