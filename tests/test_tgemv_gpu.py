"""Ternary GEMV parity on the GPU: the kernel against the exact oracle (float64), normwise
<= 1e-3 as the bar; the kernel's products and group sums are exact integers on x carried as 15-bit
fixed point per 128-k group, so its error is far below the bar."""
import numpy as np
import pytest
import torch

from conftest import normwise
from oracle import ternary

import mq
from mq import synth

pytestmark = pytest.mark.gpu
TOL = 1e-3
TIGHT = 1e-4  # x step: 1/65024 of its 128-k group's largest |x|


def run(cuda, x, w, s, n, k):
    ty = torch.full((x.shape[0], n), float("nan"), device=cuda)
    mq.project(torch.from_numpy(x).to(cuda), torch.from_numpy(w.view(np.int32)).to(cuda), torch.from_numpy(s).to(cuda),
               ty, n, k)
    torch.cuda.synchronize()
    return ty.cpu().numpy()


@pytest.mark.parametrize("n,k", [(12288, 4096), (4096, 12288), (1024, 128), (36, 256), (4, 512), (5000, 1024)])
@pytest.mark.parametrize("batch", [1, 2, 4])
def test_tgemv_matches_oracle(cuda, n, k, batch):
    rng = np.random.default_rng(n + k + batch)
    x = rng.standard_normal((batch, k)).astype(np.float16)
    w, s = synth.ternary_matrix(rng, n, k)
    y = run(cuda, x, w, s, n, k)
    ref = ternary.tgemv(x, w, s, n, k)
    assert np.isfinite(y).all()
    assert normwise(y, ref) <= TIGHT


def test_tgemv_head_rows(cuda):
    """The Qwen3 head shape's layout at full width (151936 outputs), on a K slice for oracle speed."""
    rng = np.random.default_rng(11)
    n, k = 151936, 256
    x = rng.standard_normal((1, k)).astype(np.float16)
    w, s = synth.ternary_matrix(rng, n, k)
    y = run(cuda, x, w, s, n, k)
    assert normwise(y, ternary.tgemv(x, w, s, n, k)) <= TIGHT


def test_tgemv_fp16_pairs_buffer(cuda):
    """The reference passes x as fp16 pairs in uint32 words (qwen3/kernels/qwen3k.mojo:17-20)."""
    rng = np.random.default_rng(12)
    n, k = 256, 1024
    x = rng.standard_normal((1, k)).astype(np.float16)
    w, s = synth.ternary_matrix(rng, n, k)
    ty = torch.zeros(1, n, device=cuda)
    mq.project(torch.from_numpy(x.view(np.int32)).to(cuda), torch.from_numpy(w.view(np.int32)).to(cuda),
               torch.from_numpy(s).to(cuda), ty, n, k)
    torch.cuda.synchronize()
    assert normwise(ty.cpu().numpy(), ternary.tgemv(x, w, s, n, k)) <= TIGHT


def test_tgemv_all_codes(cuda):
    """Codes all 0, all 1, all 2 and code 3 never produced: exact -sum x, 0, +sum x per group."""
    n, k = 32, 512
    x = np.random.default_rng(13).standard_normal((1, k)).astype(np.float16)
    w = np.zeros((k // 16, n), np.uint32)
    w[:, 8:16] = 0x55555555
    w[:, 16:24] = 0xAAAAAAAA
    s = np.full((k // 128, n), 0.5, np.float16)
    y = run(cuda, x, w, s, n, k)
    ref = ternary.tgemv(x, w, s, n, k)
    assert normwise(y, ref) <= TIGHT
    # code 1 is weight 0: the integer group sums cancel exactly
    assert np.abs(y[0, 8:16]).max() == 0.0
