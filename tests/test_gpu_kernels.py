"""GPU parity of the kernel entry points against the CPU oracle and the golden fixtures.

FixedQ510: bit-exact (int32 accumulators, outputs, norm_out). Float: the ternary sum is
re-associated on the GPU, so outputs agree to |d| <= 1e-4 * max(1, max|ref|); every other
op (norm, quant, sigmoid/silu/swiglu, scan) is bit-exact in both modes.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import bits_equal, golden
from matmulfreellmcpu_b200 import _lib, api

pytestmark = pytest.mark.gpu

SWEEP_KN = [(1024, 1024), (1024, 5632), (2048, 2048), (2048, 11264), (5632, 2048),
            (2560, 13824), (6912, 2560)]
FLOAT_TOL = 1e-4


def sweep_inputs(M, K, N, seed):
    """Config-1 inputs: N(0,1) activations, 1% outliers x20, ternary p=(.3,.4,.3)."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((M, K)).astype(np.float32)
    x[rng.random((M, K)) < 0.01] *= np.float32(20.0)
    wq = rng.choice(np.array([-1, 0, 1], np.int8), size=(N, K), p=[0.3, 0.4, 0.3])
    return x, np.ones(K, np.float32), wq


def to_dev(a, cuda):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(cuda)


def run_gpu(cuda, x, nw, wq, scale, mode):
    wp = api.repack_ternary(to_dev(wq, cuda))
    out, acc, norm = api.bitlinear(to_dev(x, cuda), to_dev(nw, cuda), wp, scale, wq.shape[0],
                                   act_quant=mode, want_norm=True, want_acc=(mode == "fixed"))
    return (out.cpu().numpy(), None if acc is None else acc.cpu().numpy(), norm.cpu().numpy())


def assert_float_close(got, ref):
    tol = FLOAT_TOL * max(1.0, float(np.abs(ref).max()))
    assert np.abs(got - ref).max() <= tol


def test_repack_matches_host_pack(cuda):
    rng = np.random.default_rng(3)
    for n, k in [(37, 100), (2048, 1024), (96, 1003)]:
        wq = rng.choice(np.array([-1, 0, 1], np.int8), size=(n, k))
        dev = api.repack_ternary(to_dev(wq, cuda)).cpu().numpy()
        assert np.array_equal(dev, api.pack_ternary_host(wq))


def test_repack_rejects_non_ternary(cuda):
    wq = np.zeros((32, 64), np.int8)
    wq[5, 7] = -3
    with pytest.raises(_lib.MmfreeError) as e:
        api.repack_ternary(to_dev(wq, cuda))
    assert e.value.code == _lib.E_RANGE


@pytest.mark.parametrize("idx", range(5))
@pytest.mark.parametrize("mode", ["fixed", "float"])
def test_bitlinear_golden_fixtures(cuda, idx, mode):
    g = golden("ops.npz")
    out, acc, norm = run_gpu(cuda, g[f"bl{idx}_x"], g[f"bl{idx}_nw"], g[f"bl{idx}_wq"], 20.0, mode)
    assert bits_equal(norm, g[f"bl{idx}_norm"])
    if mode == "fixed":
        assert np.array_equal(acc, g[f"bl{idx}_fixed_acc"])
        assert bits_equal(out, g[f"bl{idx}_fixed_out"])
    else:
        assert_float_close(out, g[f"bl{idx}_float_out"])


@pytest.mark.parametrize("K,N", SWEEP_KN)
@pytest.mark.parametrize("M", [1, 16, 64])
def test_bitlinear_sweep_fixed_exact(cuda, orc, M, K, N):
    x, nw, wq = sweep_inputs(M, K, N, seed=M * 7 + K + N)
    out, acc, norm = run_gpu(cuda, x, nw, wq, 20.0, "fixed")
    r_out, r_acc, r_norm = orc.bitlinear(x, nw, wq, 20.0, act_quant=1, want_norm=True)
    assert np.array_equal(acc, r_acc)
    assert bits_equal(out, r_out)
    assert bits_equal(norm, r_norm)


@pytest.mark.parametrize("K,N", SWEEP_KN)
@pytest.mark.parametrize("M", [1, 16, 64])
def test_bitlinear_sweep_float(cuda, orc, M, K, N):
    """Float on every sweep shape: the few-row fused kernel (M = 1) and the bf16 tensor-core
    path (M >= 16); norms bit for bit, outputs within the Float tolerance."""
    x, nw, wq = sweep_inputs(M, K, N, seed=K + N + M)
    out, _, norm = run_gpu(cuda, x, nw, wq, 20.0, "float")
    r_out, _, r_norm = orc.bitlinear(x, nw, wq, 20.0, act_quant=0, want_norm=True)
    assert bits_equal(norm, r_norm)
    assert_float_close(out, r_out)
    if M == 1:  # without norm_out the C ABI takes the single fused launch
        o1, _, _ = api.bitlinear(to_dev(x, cuda), to_dev(nw, cuda), api.repack_ternary(to_dev(wq, cuda)),
                                 20.0, N, act_quant="float")
        assert_float_close(o1.cpu().numpy(), r_out)


@pytest.mark.parametrize("K,N", [(2560, 13824), (2048, 11264), (6912, 2560)])
@pytest.mark.parametrize("M", [512, 4096])
def test_bitlinear_large_m_rows(cuda, orc, M, K, N):
    """Full sweep sizes: rows are independent, so sampled rows must match the oracle run on
    those rows alone (bit-exact in FixedQ510, within tolerance in Float) -- a size-independent
    check of the large-M path."""
    x, nw, wq = sweep_inputs(M, K, N, seed=M + K)
    rows = np.random.default_rng(M).choice(M, 6, replace=False)
    out, acc, _ = run_gpu(cuda, x, nw, wq, 20.0, "fixed")
    r_out, r_acc, _ = orc.bitlinear(x[rows], nw, wq, 20.0, act_quant=1)
    assert np.array_equal(acc[rows], r_acc)
    assert bits_equal(out[rows], r_out)
    fo, _, _ = run_gpu(cuda, x, nw, wq, 20.0, "float")
    f_out, _, _ = orc.bitlinear(x[rows], nw, wq, 20.0, act_quant=0)
    assert_float_close(fo[rows], f_out)


@pytest.mark.parametrize("M,K,N", [(1100, 1000, 700), (1030, 1003, 96), (1024, 5632, 64)])
def test_bitlinear_many_rows_all_match(cuda, orc, M, K, N):
    """M >= 1024: the many-rows prep (up to 8 rows per CTA, their 8-lane exact chains side by
    side; a ragged last CTA; K % 4 != 0 rows staged without the bulk copy) and the tensor-core
    matmul without a k-split; ragged M, K and N, a K % 8 scalar tail, saturating outliers;
    every row's accumulators, outputs and norm bit for bit."""
    x, nw, wq = sweep_inputs(M, K, N, seed=11 + K)
    x[::7, :4] = np.float32(600.0)  # y * 1024 past the int16 range on some rows
    out, acc, norm = run_gpu(cuda, x, nw, wq, 20.0, "fixed")
    r_out, r_acc, r_norm = orc.bitlinear(x, nw, wq, 20.0, act_quant=1, want_norm=True)
    assert np.array_equal(acc, r_acc)
    assert bits_equal(out, r_out)
    assert bits_equal(norm, r_norm)
    fo, _, fn = run_gpu(cuda, x, nw, wq, 20.0, "float")
    f_out, _, f_norm = orc.bitlinear(x, nw, wq, 20.0, act_quant=0, want_norm=True)
    assert bits_equal(fn, f_norm)
    assert_float_close(fo, f_out)


@pytest.mark.parametrize("M,K,N", [(64, 2048, 101), (40, 2048, 200), (20, 1000, 66), (64, 5632, 256),
                                   (64, 2048, 6144), (64, 2048, 11264), (48, 1536, 5632)])
def test_bitlinear_split_k_tile_edges(cuda, orc, M, K, N):
    """Few output tiles, so the reduction is split over a cluster: partial row quads
    (N % 4 != 0, no 16-byte stores), tokens past M in a tile, cluster sizes 8, 4 and 2."""
    x, nw, wq = sweep_inputs(M, K, N, seed=M + K + N)
    out, acc, _ = run_gpu(cuda, x, nw, wq, 20.0, "fixed")
    r_out, r_acc, _ = orc.bitlinear(x, nw, wq, 20.0, act_quant=1)
    assert np.array_equal(acc, r_acc)
    assert bits_equal(out, r_out)


def test_bitlinear_saturation_and_ragged(cuda, orc):
    """Q5.10 saturation (|y*1024| > 32767), K%8 tails, K%64 and N%32 padding, frac_bits."""
    rng = np.random.default_rng(11)
    for M, K, N, frac in [(3, 13, 5, 10), (4, 999, 33, 10), (2, 520, 70, 8), (1, 8, 1, 12)]:
        x = rng.standard_normal((M, K)).astype(np.float32)
        x[:, :3] *= 400.0
        nw = (0.5 + rng.random(K)).astype(np.float32)
        wq = rng.choice(np.array([-1, 0, 1], np.int8), size=(N, K))
        import torch
        wp = api.repack_ternary(to_dev(wq, cuda))
        out, acc, _ = api.bitlinear(to_dev(x, cuda), to_dev(nw, cuda), wp, 3.5, N,
                                    frac_bits=frac, want_acc=True)
        r_out, r_acc, _ = orc.bitlinear(x, nw, wq, 3.5, act_quant=1, frac_bits=frac)
        assert np.array_equal(acc.cpu().numpy(), r_acc)
        assert bits_equal(out.cpu().numpy(), r_out)
        del torch


@pytest.mark.parametrize("M,K,N", [(2100, 960, 5000), (1500, 2048, 13000)])
def test_bitlinear_rows_kernel_ragged(cuda, orc, M, K, N):
    """Enough output tiles for the persistent large-M kernel (two or more per SM): ragged
    tokens (2100 = 32 x 64 + 52), an odd chunk count (K = 960: the last 128-k block holds one
    chunk), partial last weight tiles (5000 and 13000 rows: 136 and 200 rows in the last
    256-row tile, a partial 32-row group), saturating outliers; every accumulator, output and
    norm bit for bit. The same shapes in Float (bf16 planes on the one-tile-per-CTA kernel):
    norms bit for bit, outputs within the Float tolerance."""
    x, nw, wq = sweep_inputs(M, K, N, seed=23 + K)
    x[::9, :4] = np.float32(600.0)
    out, acc, norm = run_gpu(cuda, x, nw, wq, 20.0, "fixed")
    r_out, r_acc, r_norm = orc.bitlinear(x, nw, wq, 20.0, act_quant=1, want_norm=True)
    assert np.array_equal(acc, r_acc)
    assert bits_equal(out, r_out)
    assert bits_equal(norm, r_norm)
    fo, _, fn = run_gpu(cuda, x, nw, wq, 20.0, "float")
    f_out, _, f_norm = orc.bitlinear(x, nw, wq, 20.0, act_quant=0, want_norm=True)
    assert bits_equal(fn, f_norm)
    assert_float_close(fo, f_out)


@pytest.mark.parametrize("M", [3, 20, 1100])
@pytest.mark.parametrize("K,nan_row", [(203, False), (200, True)])
def test_bitlinear_quant_extremes(cuda, orc, M, K, nan_row):
    """Q5.10 codes at the edges of cvtps2dq: y*1024 >= 2^31 (INT32_MIN, clamped to -32768),
    <= -2^31, +-inf, in the SIMD body and in the K % 8 tail, and a NaN row (every code
    -32768) at K % 8 == 0; through the dp4a path (3 rows), the per-row prep (20) and the
    many-rows prep (1100). A NaN row with a K % 8 tail is not compared: the reference's
    scalar-tail cast gives INT32_MIN there, which its int32 dot product multiplies by the
    weight, a value the 16-bit code planes cannot hold."""
    rng = np.random.default_rng(17 + M)
    N = 40
    x = rng.standard_normal((M, K)).astype(np.float32)
    if nan_row:
        x[1, 10] = np.float32(np.nan)
    nw = (0.5 + rng.random(K)).astype(np.float32)
    nw[5], nw[6], nw[7], nw[8] = 1e7, -1e7, np.inf, 3e38
    nw[K - 3], nw[K - 2], nw[K - 1] = 1e7, -np.inf, 3e38
    wq = rng.choice(np.array([-1, 0, 1], np.int8), size=(N, K))
    out, acc, norm = run_gpu(cuda, x, nw, wq, 20.0, "fixed")
    r_out, r_acc, r_norm = orc.bitlinear(x, nw, wq, 20.0, act_quant=1, want_norm=True)
    assert np.array_equal(acc, r_acc)
    assert bits_equal(out, r_out)
    assert bits_equal(norm, r_norm)


def test_bitlinear_cluster(cuda, orc):
    rng = np.random.default_rng(5)
    M, K, N = 4, 2048, 2048
    x = rng.standard_normal((M, K)).astype(np.float32)
    nws = [(0.5 + rng.random(K)).astype(np.float32) for _ in range(3)]
    wqs = [rng.choice(np.array([-1, 0, 1], np.int8), size=(N, K)) for _ in range(3)]
    scales = [61.5, 62.25, 63.0]
    outs, acc = api.bitlinear_cluster(to_dev(x, cuda), [to_dev(n, cuda) for n in nws],
                                      [api.repack_ternary(to_dev(w, cuda)) for w in wqs],
                                      scales, N, want_acc=True)
    for j in range(3):
        r_out, r_acc, _ = orc.bitlinear(x, nws[j], wqs[j], scales[j], act_quant=1)
        assert np.array_equal(acc[j].cpu().numpy(), r_acc)
        assert bits_equal(outs[j].cpu().numpy(), r_out)


def test_ternary_matmul_seam(cuda):
    import torch
    rng = np.random.default_rng(9)
    b, n, m = 5, 1000, 77
    codes = rng.integers(-32768, 32768, size=(b, n)).astype(np.int32)
    wq = rng.choice(np.array([-1, 0, 1], np.int8), size=(m, n))
    acc = api.ternary_matmul(to_dev(codes, cuda), api.repack_ternary(to_dev(wq, cuda)), m)
    ref = (codes.astype(np.int64) @ wq.T.astype(np.int64)).astype(np.int32)
    assert np.array_equal(acc.cpu().numpy(), ref)
    codes[1, 4] = 40000
    with pytest.raises(_lib.MmfreeError) as e:
        api.ternary_matmul(to_dev(codes, cuda), api.repack_ternary(to_dev(wq, cuda)), m)
    assert e.value.code == _lib.E_RANGE
    del torch


@pytest.mark.parametrize("shape", [(1, 64), (5, 37), (16, 256)])
def test_row_ops_golden(cuda, shape):
    g = golden("ops.npz")
    p = f"sc{shape[0]}x{shape[1]}"
    i, f, gg, w = (to_dev(g[f"{p}_{k}"], cuda) for k in ("i", "f", "g", "w"))
    st = to_dev(g[f"{p}_s0"], cuda)
    out = api.hgrn_scan(i, f, st)
    assert bits_equal(out.cpu().numpy(), g[f"{p}_out"])
    assert bits_equal(st.cpu().numpy(), g[f"{p}_state"])
    assert bits_equal(api.rmsnorm_swishgate(gg, i, w).cpu().numpy(), g[f"{p}_swishgate"])
    assert bits_equal(api.rmsnorm(gg, w).cpu().numpy(), g[f"{p}_rmsnorm"])


@pytest.mark.parametrize("n", [8, 29, 1000, 1003])
def test_swiglu_golden(cuda, n):
    g = golden("ops.npz")
    out = api.swiglu(to_dev(g[f"ew{n}_x"], cuda), to_dev(g[f"ew{n}_b"], cuda))
    assert bits_equal(out.cpu().numpy(), g[f"ew{n}_swiglu"])


def test_swiglu_wide_range_matches_oracle(cuda, orc):
    """The exact exp and the branch-free correctly rounded division over a wide range:
    magnitudes 2^-40..2^40 of both signs, values around the exp clamp, zeros, subnormals,
    infinities and NaN, with a SIMD tail; b = 1 on even elements, so those outputs are the
    quotients themselves. Bit-exact against the reference restatement."""
    rng = np.random.default_rng(5)
    n = 1 << 22
    a = (np.exp2(rng.uniform(-40, 40, n)) * rng.choice([-1.0, 1.0], n)).astype(np.float32)
    a[: n // 4] = rng.uniform(-100.0, 100.0, n // 4).astype(np.float32)
    specials = np.array([0.0, -0.0, 1e-45, -1e-45, 1e-38, -1e-38, 88.3762626647949,
                         -88.3762626647949, 89.0, -89.0, 1e30, -1e30, np.inf, -np.inf, np.nan,
                         1.0, -1.0, 2.0, 0.5, 27.7, -27.7, 41.6, -41.6], np.float32)
    a[: specials.size] = specials
    a = np.concatenate([a, specials[:5]])  # length % 8 == 5: a scalar tail
    b = np.ones_like(a)
    b[1::2] = rng.standard_normal(b[1::2].size).astype(np.float32)
    out = api.swiglu(to_dev(a, cuda), to_dev(b, cuda)).cpu().numpy()
    assert bits_equal(out, orc.swiglu(a, b))


def test_bitlinear_rejects_bad_shapes(cuda):
    import torch
    x = torch.zeros(2, 8, device=cuda)
    nw = torch.ones(8, device=cuda)
    wp = api.repack_ternary(torch.zeros(4, 8, dtype=torch.int8, device=cuda))
    lib = _lib.lib()
    s = torch.cuda.current_stream().cuda_stream
    rc = lib.mmfree_cuda_bitlinear(x.data_ptr(), x.data_ptr(), nw.data_ptr(), wp.data_ptr(), 1.0,
                                   2, _lib.MAX_IN_DIM + 1, 4, 1e-6, None, 1, 10, None, s)
    assert rc == _lib.E_INVALID
    rc = lib.mmfree_cuda_bitlinear(x.data_ptr(), x.data_ptr(), nw.data_ptr(), wp.data_ptr(), 1.0,
                                   0, 8, 4, 1e-6, None, 1, 10, None, s)
    assert rc == _lib.OK  # zero rows is a no-op
