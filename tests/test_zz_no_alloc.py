"""GPU test of mmfree_cuda_bitlinear_noalloc, the BitLinear entry point that allocates no
device memory (for callers such as plugins inside a process whose allocator owns the GPU,
decode loops that must not block on an allocation, or work issued during stream capture,
where cudaMalloc is not allowed). It must return what mmfree_cuda_bitlinear returns for the
same inputs, call after call, although every call shares one static scratch array.

This file sorts last so that a run stopping at the first failure has run everything else.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import bits_equal
from matmulfreellmcpu_b200 import _lib, api

pytestmark = pytest.mark.gpu

FLOAT_TOL = 1e-4  # same tolerance as tests/test_gpu_kernels.py for Float-mode outputs


def _dev(a, cuda):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(cuda)


def _inputs(M, K, N, seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((M, K)).astype(np.float32)
    x[rng.random((M, K)) < 0.01] *= np.float32(20.0)
    wq = rng.choice(np.array([-1, 0, 1], np.int8), size=(N, K), p=[0.3, 0.4, 0.3])
    nw = (0.5 + rng.random(K)).astype(np.float32)
    return x, nw, wq


def _noalloc(cuda, x, nw, wp, scale, N, mode):
    """One call of the new entry point through the C ABI; returns (out, acc, norm) on host."""
    import torch
    M, K = x.shape
    out = torch.empty(M, N, dtype=torch.float32, device=cuda)
    norm = torch.empty(M, K, dtype=torch.float32, device=cuda)
    acc = torch.empty(M, N, dtype=torch.int32, device=cuda)
    aq = _lib.ACT_FIXED_Q510 if mode == "fixed" else _lib.ACT_FLOAT
    rc = _lib.lib().mmfree_cuda_bitlinear_noalloc(
        out.data_ptr(), x.data_ptr(), nw.data_ptr(), wp.data_ptr(), scale, M, K, N, 1e-6,
        norm.data_ptr(), aq, 10, acc.data_ptr(), torch.cuda.current_stream().cuda_stream)
    _lib.check(rc)
    torch.cuda.synchronize()
    return out.cpu().numpy(), (acc.cpu().numpy() if mode == "fixed" else None), norm.cpu().numpy()


@pytest.mark.parametrize("mode", ["fixed", "float"])
def test_noalloc_matches_bitlinear_on_consecutive_calls(cuda, mode):
    # consecutive calls with different shapes: the shared scratch keeps the previous call's
    # bytes, which must not leak into the next result
    for i, (M, K, N) in enumerate([(16, 2048, 2048), (5, 1003, 77), (1, 5632, 2048),
                                   (64, 2560, 512)]):
        x, nw, wq = _inputs(M, K, N, seed=100 + i)
        xd, nwd = _dev(x, cuda), _dev(nw, cuda)
        wp = api.repack_ternary(_dev(wq, cuda))
        ref_out, ref_acc, ref_norm = api.bitlinear(xd, nwd, wp, 20.0, N, act_quant=mode,
                                                   want_norm=True, want_acc=(mode == "fixed"))
        ref_out, ref_norm = ref_out.cpu().numpy(), ref_norm.cpu().numpy()
        for _ in range(2):  # two calls in a row on the same inputs
            out, acc, norm = _noalloc(cuda, xd, nwd, wp, 20.0, N, mode)
            assert bits_equal(norm, ref_norm)
            if mode == "fixed":
                assert np.array_equal(acc, ref_acc.cpu().numpy())
                assert bits_equal(out, ref_out)
            else:
                assert np.abs(out - ref_out).max() <= FLOAT_TOL * max(1.0, float(np.abs(ref_out).max()))


@pytest.mark.parametrize("M", [3, 40])  # dp4a and tensor-core kernels
def test_noalloc_matches_oracle(cuda, orc, M):
    # pinned to the CPU oracle directly, not only through mmfree_cuda_bitlinear
    K, N = 2048, 2048
    x, nw, wq = _inputs(M, K, N, seed=7 + M)
    xd, nwd = _dev(x, cuda), _dev(nw, cuda)
    wp = api.repack_ternary(_dev(wq, cuda))
    r_out, r_acc, r_norm = orc.bitlinear(x, nw, wq, 20.0, act_quant=1, want_norm=True)
    for _ in range(2):
        out, acc, norm = _noalloc(cuda, xd, nwd, wp, 20.0, N, "fixed")
        assert np.array_equal(acc, r_acc)
        assert bits_equal(out, r_out)
        assert bits_equal(norm, r_norm)


def test_noalloc_timeout_is_reported_then_cleared(cuda):
    # a kernel that gives up a bounded wait records it in the array's own error word; the
    # status call reports it once, and the next call is correct again
    M, K, N = 4, 1024, 256
    x, nw, wq = _inputs(M, K, N, seed=11)
    xd, nwd = _dev(x, cuda), _dev(nw, cuda)
    wp = api.repack_ternary(_dev(wq, cuda))
    ref_out, _, _ = api.bitlinear(xd, nwd, wp, 20.0, N)
    api.kernel_status()
    api.set_wait_limit(0)
    try:
        _noalloc(cuda, xd, nwd, wp, 20.0, N, "fixed")
    finally:
        api.set_wait_limit(-1)
    with pytest.raises(_lib.MmfreeError) as e:
        api.kernel_status()
    assert e.value.code == _lib.E_TIMEOUT
    api.kernel_status()
    out, _, _ = _noalloc(cuda, xd, nwd, wp, 20.0, N, "fixed")
    api.kernel_status()
    assert bits_equal(out, ref_out.cpu().numpy())


def test_noalloc_rejects_oversize_calls(cuda):
    import torch
    M, K, N = 4096, 2560, 64  # 2 * 4096 * 2560 bytes of planes > 4 MiB
    x = torch.zeros(M, K, device=cuda)
    nw = torch.ones(K, device=cuda)
    wp = api.repack_ternary(torch.zeros(N, K, dtype=torch.int8, device=cuda))
    out = torch.empty(M, N, device=cuda)
    rc = _lib.lib().mmfree_cuda_bitlinear_noalloc(
        out.data_ptr(), x.data_ptr(), nw.data_ptr(), wp.data_ptr(), 1.0, M, K, N, 1e-6, None,
        _lib.ACT_FIXED_Q510, 10, None, None)
    assert rc == _lib.E_INVALID
    assert b"MMFREE_CUDA_NOALLOC_SCRATCH_BYTES" in _lib.lib().mmfree_cuda_last_error()
