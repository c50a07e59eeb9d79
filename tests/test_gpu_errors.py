"""GPU tests of the error path of the asynchronous kernel entry points.

A bounded wait inside a kernel that gives up must be reported for the call that made it
(mmfree_cuda_kernel_status returns MMFREE_E_TIMEOUT once, then clears it), must not poison
the next, unrelated call, and must leave the GPU usable. The failure is made without any
fault: the diagnostic switch mmfree_cuda_set_wait_limit(0) makes the BitLinear prologue's
row-staging wait give up at once (it still drains the copy it issued before returning).
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import bits_equal
from matmulfreellmcpu_b200 import _lib, api

pytestmark = pytest.mark.gpu


def _inputs(M, K, N, seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((M, K)).astype(np.float32)
    wq = rng.choice(np.array([-1, 0, 1], np.int8), size=(N, K), p=[0.3, 0.4, 0.3])
    return x, np.ones(K, np.float32), wq


def _dev(a, cuda):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(cuda)


class _GiveUp:
    """Every staged row wait gives up while the block runs (limit restored on exit)."""

    def __enter__(self):
        api.set_wait_limit(0)

    def __exit__(self, *exc):
        api.set_wait_limit(-1)


@pytest.mark.parametrize("M", [4, 64])  # dp4a path, tensor-core path
def test_bitlinear_timeout_is_reported_then_cleared(cuda, orc, M):
    K, N = 2048, 512
    x, nw, wq = _inputs(M, K, N, seed=M)
    xd, nwd = _dev(x, cuda), _dev(nw, cuda)
    wp = api.repack_ternary(_dev(wq, cuda))
    api.kernel_status()  # nothing pending from earlier tests
    with _GiveUp():
        # queued: the failure happens on the device (asking for the accumulators keeps a
        # few-row call on the prologue + matmul kernels, whose row wait this gives up)
        api.bitlinear(xd, nwd, wp, 20.0, N, want_acc=True)
    with pytest.raises(_lib.MmfreeError) as e:
        api.kernel_status()
    assert e.value.code == _lib.E_TIMEOUT
    api.kernel_status()  # reported once, then cleared
    # the next calls, of this entry point and of an unrelated synchronous one, succeed
    api.repack_ternary(_dev(wq, cuda))
    out, acc, _ = api.bitlinear(xd, nwd, wp, 20.0, N, want_acc=True)
    api.kernel_status()
    r_out, r_acc, _ = orc.bitlinear(x, nw, wq, 20.0, act_quant=1)
    assert np.array_equal(acc.cpu().numpy(), r_acc)
    assert bits_equal(out.cpu().numpy(), r_out)


def test_cluster_timeout_is_reported(cuda):
    M, K, N = 20, 1024, 256
    x, nw, wq = _inputs(M, K, N, seed=5)
    xd, nwd = _dev(x, cuda), _dev(nw, cuda)
    wp = api.repack_ternary(_dev(wq, cuda))
    api.kernel_status()
    with _GiveUp():
        api.bitlinear_cluster(xd, [nwd] * 3, [wp] * 3, [20.0] * 3, N)
    with pytest.raises(_lib.MmfreeError) as e:
        api.kernel_status()
    assert e.value.code == _lib.E_TIMEOUT
    outs, _ = api.bitlinear_cluster(xd, [nwd] * 3, [wp] * 3, [20.0] * 3, N)
    api.kernel_status()
    ref, _, _ = api.bitlinear(xd, nwd, wp, 20.0, N)
    for o in outs:
        assert bits_equal(o.cpu().numpy(), ref.cpu().numpy())
