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


def run_head(cuda, x, w, s, n, k):
    b = x.shape[0]
    ty = torch.full((b, n), float("nan"), device=cuda)
    tc = torch.full((b, -(-n // 512), 3), float("nan"), device=cuda)
    mq.packed_head(torch.from_numpy(x).to(cuda), torch.from_numpy(w.view(np.int32)).to(cuda), torch.from_numpy(s).to(cuda),
                   ty, tc, n, k)
    idx = mq.head_argmax(tc)
    torch.cuda.synchronize()
    return ty.cpu().numpy(), tc.cpu().numpy(), idx.cpu().numpy()


def check_candidates(y, cand):
    """The kernel's candidates equal the oracle's selection over the kernel's own logits, bit for bit
    (value and index where the block is not flagged)."""
    ref = ternary.head_candidates(y)
    np.testing.assert_array_equal(cand[..., 2], ref[..., 2])
    ok = ref[..., 2] == 0
    np.testing.assert_array_equal(cand[..., 0][ok], ref[..., 0][ok])
    np.testing.assert_array_equal(cand[..., 1][ok], ref[..., 1][ok])


@pytest.mark.parametrize("n,k,batch", [(151936, 256, 1), (75968, 512, 2), (12288, 1024, 4), (1000, 128, 1), (4, 256, 3)])
def test_packed_head_candidates(cuda, n, k, batch):
    """packed_head with select (bonsai/kernels/kernels.mojo:451-517): logits as mq_tgemv, candidates per
    512 logits, and the device greedy index (best_of, lfm2/kernels/dsk.mojo:442-465) against the oracle."""
    rng = np.random.default_rng(n + k + batch)
    x = rng.standard_normal((batch, k)).astype(np.float16)
    w, s = synth.ternary_matrix(rng, n, k)
    y, cand, idx = run_head(cuda, x, w, s, n, k)
    ref = ternary.tgemv(x, w, s, n, k)
    assert normwise(y, ref) <= TIGHT
    check_candidates(y, cand)
    np.testing.assert_array_equal(idx, ternary.greedy(cand))
    np.testing.assert_array_equal(idx, y.argmax(axis=1))  # numpy's argmax also takes the first maximum
    for b in range(batch):  # the exact argmax too, where the top two are apart by more than the error
        top2 = np.sort(ref[b])[-2:]
        if top2[1] - top2[0] > 4 * TIGHT * np.abs(ref[b]).max():
            assert idx[b] == ref[b].argmax()
    if n >= 151936:  # large heads run the same K-unsplit kernel as mq_tgemv: identical logits
        np.testing.assert_array_equal(y, run(cuda, x, w, s, n, k))


def test_packed_head_ties_take_the_lowest_index(cuda):
    """Equal logits (identical columns give bit-identical sums): within a block and across blocks the
    lowest index wins, as greedy() and the subgroup reduction of packed_head order them."""
    rng = np.random.default_rng(21)
    n, k = 4096, 256
    x = rng.standard_normal((1, k)).astype(np.float16)
    w, s = synth.ternary_matrix(rng, n, k)
    y0 = ternary.tgemv(x, w, s, n, k)[0]
    top = int(y0.argmax())
    for dst in (5, 700, 3000, 4095):  # copies of the best column, in and out of its block
        w[:, dst] = w[:, top]
        s[:, dst] = s[:, top]
    y, cand, idx = run_head(cuda, x, w, s, n, k)
    check_candidates(y, cand)
    assert idx[0] == min(5, top)
    assert cand[0, 0, 1] == min(5, top) or top >= 512


def test_packed_head_flags_non_finite(cuda):
    """A non-finite logit flags its block, and the greedy index is -1 (greedy() stops there)."""
    rng = np.random.default_rng(22)
    n, k = 2048, 256
    x = rng.standard_normal((1, k)).astype(np.float16)
    w, s = synth.ternary_matrix(rng, n, k)
    s[0, 1300] = np.float16(np.inf)
    y, cand, idx = run_head(cuda, x, w, s, n, k)
    assert not np.isfinite(y[0, 1300])
    np.testing.assert_array_equal(cand[0, :, 2], [0, 0, 1, 0])
    check_candidates(y, cand)
    assert idx[0] == -1


def test_packed_head_all_negative_tail_stays_in_range(cuda):
    """A last block that is partly past n and whose logits are all negative still names a real index."""
    rng = np.random.default_rng(23)
    n, k = 1000, 128
    x = np.abs(rng.standard_normal((1, k))).astype(np.float16)
    w = np.zeros((k // 16, n), np.uint32)  # every code 0: logit = -scale * sum x < 0
    s = np.abs(rng.standard_normal((k // 128, n))).astype(np.float16) + np.float16(0.1)
    y, cand, idx = run_head(cuda, x, w, s, n, k)
    assert (y < 0).all()
    check_candidates(y, cand)
    assert 512 <= cand[0, 1, 1] < n and 0 <= idx[0] < n


@pytest.mark.parametrize("n,k,batch", [(75893, 4096, 1), (1003, 1024, 3), (33, 256, 2), (6, 128, 1), (5, 512, 4),
                                       (1, 128, 1)])
def test_tgemv_ragged_width(cuda, n, k, batch):
    """Any width n, as the reference's per-output tail handles it (bonsai/kernels/kernels.mojo:477-487):
    n % 4 != 0 (a row stride no tensor map can describe) streams with cp.async; 75893 is the second
    half of the Qwen3 head (qwen3/model.mojo:176-181, qwen3/convert.cpp:16,122-123) at full K."""
    rng = np.random.default_rng(n + k + batch)
    x = rng.standard_normal((batch, k)).astype(np.float16)
    w, s = synth.ternary_matrix(rng, n, k)
    y = run(cuda, x, w, s, n, k)
    assert np.isfinite(y).all()
    assert normwise(y, ternary.tgemv(x, w, s, n, k)) <= TIGHT
    assert mq.device_status() == 0


@pytest.mark.parametrize("n", [151936, 75776, 75893])
def test_packed_head_full_size(cuda, n):
    """The head at full size against the oracle: BASELINE configs[4]'s [151936, 4096] and the two halves
    the reference's converter writes, head0 = 74 * 1024 rows and head1 = 151669 - 74 * 1024 = 75893 rows
    (qwen3/convert.cpp:16,122-123), with candidates and the device greedy."""
    rng = np.random.default_rng(n)
    k = 4096
    x = rng.standard_normal((1, k)).astype(np.float16)
    w, s = synth.ternary_matrix(rng, n, k)
    y, cand, idx = run_head(cuda, x, w, s, n, k)
    ref = ternary.tgemv(x, w, s, n, k)
    assert normwise(y, ref) <= TIGHT
    check_candidates(y, cand)
    np.testing.assert_array_equal(idx, ternary.greedy(cand))
    np.testing.assert_array_equal(idx, y.argmax(axis=1))
    top2 = np.sort(ref[0])[-2:]
    if top2[1] - top2[0] > 4 * TIGHT * np.abs(ref[0]).max():
        assert idx[0] == ref[0].argmax()


@pytest.mark.parametrize("n", [4096, 1003])
def test_tgemv_non_finite_x(cuda, n):
    """A NaN or an infinity in x makes the outputs non-finite where the reference's fp32 sums are
    (every output: x * w is infinite, or NaN for w = 0), and the greedy index -1 (bonsai/bonsai_vk.c:506-515
    stops on non-finite logits); a finite token in the same batch is unaffected."""
    rng = np.random.default_rng(31 + n)
    k = 1024
    x = rng.standard_normal((3, k)).astype(np.float16)
    x[0, 517] = np.float16(np.nan)
    x[1, 3] = np.float16(-np.inf)
    w, s = synth.ternary_matrix(rng, n, k)
    ref = ternary.tgemv(x, w, s, n, k)
    assert not np.isfinite(ref[:2]).any()
    y = run(cuda, x, w, s, n, k)
    np.testing.assert_array_equal(np.isfinite(y), np.isfinite(ref))
    assert normwise(y[2:], ref[2:]) <= TIGHT
    yh, cand, idx = run_head(cuda, x, w, s, n, k)
    np.testing.assert_array_equal(np.isfinite(yh), np.isfinite(ref))
    assert (cand[:2, :, 2] == 1).all() and (cand[2, :, 2] == 0).all()
    np.testing.assert_array_equal(idx, [-1, -1, ternary.greedy(cand[2:])[0]])
