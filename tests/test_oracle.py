"""Pins the CPU oracle (oracle/mmfree_oracle.c) to the reference engine.

The reference ships no golden vectors on its main branch, so the pins are outputs of the
reference's own code (tests/golden/*.npz, written by tests/golden/make_golden.py from
oracle/_ref, the reference compiled from its sources). Where the compiled reference is
present, the oracle is also compared with it live on fresh inputs.
"""
from __future__ import annotations

import hashlib
import os

import numpy as np
import pytest

from conftest import bits_equal, golden
from matmulfreellmcpu_b200 import blob as B

OPS = golden("ops.npz")
OP_SHAPES = [(1, 64, 32), (3, 100, 37), (4, 256, 96), (2, 1024, 64), (5, 1003, 77)]


def _ref():
    import oracle
    if not os.path.exists(oracle.REF_SO):
        pytest.skip("compiled reference absent (oracle/_ref is built only where the "
                    "reference tree exists)")
    return oracle.Reference()


@pytest.mark.parametrize("idx", range(len(OP_SHAPES)))
@pytest.mark.parametrize("mode", ["fixed", "float"])
def test_bitlinear_golden(orc, idx, mode):
    x, nw, wq = OPS[f"bl{idx}_x"], OPS[f"bl{idx}_nw"], OPS[f"bl{idx}_wq"]
    out, acc, norm = orc.bitlinear(x, nw, wq, 20.0, act_quant=int(mode == "fixed"),
                                   want_norm=True)
    assert bits_equal(out, OPS[f"bl{idx}_{mode}_out"])
    assert bits_equal(norm, OPS[f"bl{idx}_norm"])
    if mode == "fixed":
        assert np.array_equal(acc, OPS[f"bl{idx}_fixed_acc"])


@pytest.mark.parametrize("n", [8, 29, 1000, 1003])
def test_elementwise_golden(orc, n):
    v, b = OPS[f"ew{n}_x"], OPS[f"ew{n}_b"]
    assert bits_equal(orc.sigmoid(v), OPS[f"ew{n}_sigmoid"])
    assert bits_equal(orc.silu(v), OPS[f"ew{n}_silu"])
    assert bits_equal(orc.swiglu(v, b), OPS[f"ew{n}_swiglu"])
    assert np.array_equal(orc.quant_q510(v), OPS[f"ew{n}_quant"])
    assert bits_equal(orc.sumsq(v[np.isfinite(v)]), OPS[f"ew{n}_sumsq"][0])


@pytest.mark.parametrize("shape", [(1, 64), (5, 37), (16, 256)])
def test_scan_swishgate_golden(orc, shape):
    p = f"sc{shape[0]}x{shape[1]}"
    out, st = orc.hgrn_scan(OPS[f"{p}_i"], OPS[f"{p}_f"], OPS[f"{p}_s0"])
    assert bits_equal(out, OPS[f"{p}_out"]) and bits_equal(st, OPS[f"{p}_state"])
    assert bits_equal(orc.rmsnorm_swishgate(OPS[f"{p}_g"], OPS[f"{p}_i"], OPS[f"{p}_w"]),
                      OPS[f"{p}_swishgate"])
    assert bits_equal(orc.rmsnorm(OPS[f"{p}_g"], OPS[f"{p}_w"]), OPS[f"{p}_rmsnorm"])


def _sha(path):
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 22), b""):
            h.update(chunk)
    return h.digest()


@pytest.mark.parametrize("name", ["tiny", "ragged", "small"])
def test_model_golden(orc, blob_cache, name):
    g = golden(f"model_{name}.npz")
    path = B.cached_blob(name, 0, blob_cache)
    assert _sha(path) == g["blob_sha256"].tobytes(), "seeded blob writer changed"
    m = orc.model(B.Blob.open(path))
    prompts = [g[f"serve_prompt{k}"] for k in range(3)]
    for aq, mode in ((1, "fixed"), (0, "float")):
        stream, _ = m.generate(g["prompt"], 9, act_quant=aq)
        assert np.array_equal(stream, g[f"{mode}_stream"])
        assert bits_equal(m.forward(stream, act_quant=aq)[-1], g[f"{mode}_logits"])
        assert bits_equal(m.forward(g["prompt"], act_quant=aq), g[f"{mode}_prefix_logits"])
        for k, s in enumerate(m.generate_serve(prompts, 6, act_quant=aq)):
            assert np.array_equal(s, g[f"{mode}_serve{k}"])


def test_config0_370m_golden(orc, blob_cache):
    """Benchmark configuration 0: 370M blob seed 0, 16 ids seed 0, 32 greedy tokens."""
    g = golden("config_370M.npz")
    path = B.cached_blob("370M", 0, blob_cache)
    assert _sha(path) == g["blob_sha256"].tobytes()
    m = orc.model(B.Blob.open(path))
    stream, _ = m.generate(g["prompt"], 32, act_quant=1)
    assert np.array_equal(stream, g["fixed_stream"])
    assert bits_equal(m.forward(stream, act_quant=1)[-1], g["fixed_logits"])


def test_oracle_matches_live_reference(orc):
    """Fresh random inputs (not in any fixture) through both checkers."""
    R = _ref()
    rng = np.random.default_rng(1234)
    for M, K, N in [(2, 72, 40), (3, 2048, 128), (1, 13, 9)]:
        x = (rng.standard_normal((M, K)) * rng.choice([0.1, 1, 40], (M, K))).astype(np.float32)
        wq = rng.choice(np.array([-1, 0, 1], np.int8), size=(N, K))
        nw = rng.random(K).astype(np.float32) + 0.5
        for aq in (1, 0):
            a = orc.bitlinear(x, nw, wq, 7.5, act_quant=aq, want_norm=True)
            b = R.bitlinear(x, nw, wq, 7.5, act_quant=aq, want_norm=True)
            assert bits_equal(a[0], b[0]) and bits_equal(a[2], b[2])
            if aq:
                assert np.array_equal(a[1], b[1])
    for n in (5, 8, 77, 4096):
        v = (rng.standard_normal(n) * 6).astype(np.float32)
        w = rng.standard_normal(n).astype(np.float32)
        assert bits_equal(orc.sigmoid(v), R.sigmoid(v))
        assert bits_equal(orc.swiglu(v, w), R.swiglu(v, w))
        assert bits_equal(orc.sumsq(v), R.sumsq(v))


def test_oracle_catches_a_planted_mistake(orc):
    """The pins are sharp: an oracle variant with an unfused recurrence step is caught."""
    g = golden("ops.npz")
    i, f, s0 = g["sc16x256_i"], g["sc16x256_f"], g["sc16x256_s0"]
    st = s0.copy()
    out = np.empty_like(i)
    for t in range(i.shape[0]):  # mul-then-add: the mistake the reference build does not make
        st = (f[t] * st).astype(np.float32) + i[t]
        out[t] = st
    assert not bits_equal(out, g["sc16x256_out"])
    assert bits_equal(orc.hgrn_scan(i, f, s0)[0], g["sc16x256_out"])
