"""mq_gemm_q4_noalloc (fp32 x, scratch in libmq's own device memory) against mq_gemm_q4 with a caller
workspace, through the C ABI. Collected last so that it also runs after every other test in the
same process; it passes on its own in a fresh process too."""
import ctypes

import numpy as np
import pytest
import torch

from conftest import normwise
from oracle import q4 as oq4

from mq import MQ_F32, synth
from mq._lib import MQError, lib

TOL = 1e-3
MAX_ACTIVATIONS = (4 << 20) // 2  # m * k limit of the fixed scratch


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _t(a, dev):
    a = np.ascontiguousarray(a)
    return torch.from_numpy(a.view(np.int32) if a.dtype == np.uint32 else a).to(dev)


def test_noalloc_rejects_oversized_activations():
    """Sizes beyond the fixed scratch fail with EINVAL before anything reaches a device."""
    fake = ctypes.c_void_p(1 << 20)
    with pytest.raises(MQError, match="scratch") as e:
        lib.call("mq_gemm_q4_noalloc", fake, fake, fake, fake, 256, 8192, MAX_ACTIVATIONS // 8192 + 1, 32, 0, None)
    assert e.value.code == -1


@pytest.mark.gpu
@pytest.mark.parametrize("m,n,k,group,add", [(37, 1000, 2048, 32, False), (256, 2048, 8192, 64, True),
                                             (5, 384, 768, 128, False)])
def test_noalloc_matches_workspace_entry(cuda, m, n, k, group, add):
    rng = np.random.default_rng(m * 7 + n)
    wq, ws = synth.q4_matrix(rng, n, k, group)
    dwq, dws = _t(wq, cuda), _t(ws, cuda)
    nbytes = lib.mq_gemm_q4_workspace_size(m, k, MQ_F32)
    work = torch.empty(nbytes, dtype=torch.uint8, device=cuda)
    w64 = oq4.dequant(wq, ws, group).astype(np.float64)
    for call in range(2):  # two calls in a row, new activations each time
        x = rng.standard_normal((m, k)).astype(np.float32)
        y0 = rng.standard_normal((m, n)).astype(np.float32)
        dx = _t(x, cuda)
        y_ref = _t(y0, cuda)
        y = _t(y0, cuda)
        lib.call("mq_gemm_q4", _p(dwq), _p(dws), _p(dx), MQ_F32, _p(y_ref), n, k, m, group, int(add), _p(work), nbytes,
                 _stream())
        lib.call("mq_gemm_q4_noalloc", _p(dwq), _p(dws), _p(dx), _p(y), n, k, m, group, int(add), _stream())
        torch.cuda.synchronize()
        assert lib.mq_device_status(1, None) == 0
        got, want = y.cpu().numpy(), y_ref.cpu().numpy()
        assert normwise(got, want) <= TOL, f"call {call}"
        exact = x.astype(np.float64) @ w64.T + (y0 if add else 0.0)
        assert normwise(got, exact) <= TOL, f"call {call}"
