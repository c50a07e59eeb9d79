"""GPU parity of the model path (generate / forward / generate_serve / serving session)
against the reference's own outputs (golden fixtures) and the CPU oracle.

FixedQ510 must match bit for bit (ids and logits). Float must match the logits within
max|d| <= 1e-3 * (max - min) of the reference logits.
"""
from __future__ import annotations

import os

import numpy as np
import pytest

from conftest import bits_equal, golden
from matmulfreellmcpu_b200 import _lib, api
from matmulfreellmcpu_b200 import blob as B

pytestmark = pytest.mark.gpu


def float_close(got, ref, rel=1e-3):
    span = float(ref.max() - ref.min())
    return float(np.abs(got - ref).max()) <= rel * span


@pytest.fixture(scope="module")
def models(cuda, blob_cache):
    cache = {}

    def get(name, mode):
        key = (name, mode)
        if key not in cache:
            cache[key] = api.Model(B.cached_blob(name, 0, blob_cache), mode)
        return cache[key]
    yield get
    for m in cache.values():
        m.close()


@pytest.mark.parametrize("name", ["tiny", "ragged", "small"])
def test_small_models_golden(models, name):
    g = golden(f"model_{name}.npz")
    prompts = [g[f"serve_prompt{k}"] for k in range(3)]
    m = models(name, "fixed")
    stream = m.generate(g["prompt"], 9)
    assert np.array_equal(stream, g["fixed_stream"])
    assert bits_equal(m.forward_last(stream), g["fixed_logits"])
    assert bits_equal(m.forward(g["prompt"]), g["fixed_prefix_logits"])
    for k, s in enumerate(m.generate_serve(prompts, 6)):
        assert np.array_equal(s, g[f"fixed_serve{k}"])
    mf = models(name, "float")
    assert float_close(mf.forward_last(g["float_stream"]), g["float_logits"])
    assert float_close(mf.forward(g["prompt"]), g["float_prefix_logits"])
    assert np.array_equal(mf.generate(g["prompt"], 9), g["float_stream"])


@pytest.mark.parametrize("name", ["small", "370M"])
def test_layer_trace_matches_oracle(models, orc, blob_cache, name):
    """Every layer's recurrence output, residual and output, bit for bit (fixed mode)."""
    om = orc.model(B.Blob.open(B.cached_blob(name, 0, blob_cache)))
    ids = B.seeded_ids(9, 77, B.CONFIGS[name]["vocab_size"])
    lg, tr = models(name, "fixed").forward_trace(ids)
    olg, otr = om.forward_trace(ids, 1)
    for i in range(tr.shape[0]):
        layer, what = (i - 1) // 3, ("recur", "resid", "h")[(i - 1) % 3] if i else "embed"
        assert bits_equal(tr[i], otr[i]), f"layer {layer} {what} differs"
    assert bits_equal(lg, olg)


def test_packed_blob_loads_identically(cuda, tmp_path, blob_cache):
    """A model loaded from model.mmfree2 (weights uploaded packed, no repack) gives the same
    logits and ids as one loaded from model.mmfree."""
    src = B.cached_blob("small", 0, blob_cache)
    dst = B.write_packed_blob(src, str(tmp_path / "small.mmfree2"))
    ids = B.seeded_ids(40, 7, 2048)
    out = []
    for path in (src, dst):
        with api.Model(path, "fixed") as m:
            out.append((m.forward(ids), m.generate(ids[:9], 12), m.generate_serve([ids[:5], ids[5:12]], 6)))
    assert bits_equal(out[0][0], out[1][0])
    assert np.array_equal(out[0][1], out[1][1])
    for a, b in zip(out[0][2], out[1][2]):
        assert np.array_equal(a, b)


def test_float_fused_decode_matches_oracle(models, orc, blob_cache):
    """Float mode at 1-3 streams runs the fused decode phases (fp32 activations, sums in any
    order): the greedy ids equal the oracle's float streams, and the last-step logits of a
    single stream agree within the float tolerance."""
    m = models("small", "float")
    om = orc.model(B.Blob.open(B.cached_blob("small", 0, blob_cache)))
    prompts = [B.seeded_ids(6 + k, 720 + k, 2048) for k in range(3)]
    ref_ids, ref_logits = om.generate(prompts[0], 10, act_quant=0)
    got = m.generate(prompts[0], 10)
    assert np.array_equal(got, ref_ids)
    assert float_close(m.forward_last(got[:-1]), ref_logits)
    for k in (2, 3):
        for a, b in zip(m.generate_serve(prompts[:k], 8), om.generate_serve(prompts[:k], 8, act_quant=0)):
            assert np.array_equal(a, b)


def test_long_prefill_matches_oracle(models, orc, blob_cache):
    """A 1100-token forward through the grouped i/f/g and paired SwiGLU tensor-core launches
    without k-splits, and the fused mixer over 1100 steps; logits bit-identical to the oracle."""
    m = models("small", "fixed")
    om = orc.model(B.Blob.open(B.cached_blob("small", 0, blob_cache)))
    ids = B.seeded_ids(1100, 31, 2048)
    assert bits_equal(m.forward(ids), om.forward(ids))


def test_long_float_prefill_chunked_scan(models, orc, blob_cache):
    """Float mode runs the prefill recurrence as a chunked parallel scan (64-step chunks, 18
    of them here, carries propagated between chunks); every position's logits stay within
    the Float tolerance of the oracle's sequential scan, and a multi-sequence batch gives each
    sequence the logits it gets alone."""
    m = models("small", "float")
    om = orc.model(B.Blob.open(B.cached_blob("small", 0, blob_cache)))
    ids = B.seeded_ids(1100, 31, 2048)
    got, ref = m.forward(ids), om.forward(ids, act_quant=0)
    span = float(ref.max() - ref.min())
    assert float(np.abs(got - ref).max()) <= 1e-3 * span
    seqs = [ids[:300], ids[300:700], ids[700:1000]]  # equal lengths batch in one prefill
    seqs = [s[:300] for s in seqs]
    first = m.serve_begin(seqs)
    m.serve_end()
    for k, s in enumerate(seqs):
        assert first[k] == int(np.argmax(m.forward_last(s)))


def test_fused_and_unfused_decode_agree(cuda, blob_cache, monkeypatch):
    """The fused few-row decode kernels (<= 4 streams) and the general per-op path give
    identical ids (both are bit-exact restatements)."""
    path = B.cached_blob("small", 0, blob_cache)
    prompts = [B.seeded_ids(6, 500 + k, 2048) for k in range(3)]
    out = {}
    for flag in ("0", "1"):
        monkeypatch.setenv("MMFREE_FUSED_DECODE", flag)
        with api.Model(path, "fixed") as m:
            out[flag] = (m.generate(prompts[0], 10), m.generate_serve(prompts, 7))
    assert np.array_equal(out["0"][0], out["1"][0])
    for a, b in zip(out["0"][1], out["1"][1]):
        assert np.array_equal(a, b)


@pytest.mark.gpu
def test_persistent_step_matches_per_launch_step(cuda, monkeypatch, blob_cache, orc):
    """The persistent decode step (one cooperative launch per token) and the per-phase
    launches give identical ids, and both match the oracle, at 1, 2 and 3 streams."""
    path = B.cached_blob("small", 0, blob_cache)
    om = orc.model(B.Blob.open(path))
    prompts = [B.seeded_ids(7, 610 + k, 2048) for k in range(3)]
    out = {}
    for flag in ("0", "1"):
        monkeypatch.setenv("MMFREE_PERSIST", flag)  # 1: one cooperative launch per step
        with api.Model(path, "fixed") as m:
            out[flag] = (m.generate(prompts[0], 12), m.generate_serve(prompts[:2], 9),
                         m.generate_serve(prompts, 9))
    assert np.array_equal(out["0"][0], out["1"][0])
    assert np.array_equal(out["1"][0], om.generate(prompts[0], 12)[0])
    for k in (1, 2):
        ref = om.generate_serve(prompts[:2] if k == 1 else prompts, 9)
        for a, b, c in zip(out["0"][k], out["1"][k], ref):
            assert np.array_equal(a, b)
            assert np.array_equal(b, c)


def test_mixer_in_prep_matches_mixer_kernel(cuda, monkeypatch, blob_cache, orc):
    """A decode step runs the token mixer inside the o_proj prep; MMFREE_MIX_IN_PREP=0 runs
    it as its own kernel (mixer_decode_kernel). Both give the oracle's ids, through the
    tensor-core path (20 streams) and the per-op few-row path (3 streams, unfused)."""
    path = B.cached_blob("small", 0, blob_cache)
    om = orc.model(B.Blob.open(path))
    prompts = [B.seeded_ids(5, 700 + k, 2048) for k in range(20)]
    monkeypatch.setenv("MMFREE_FUSED_DECODE", "0")
    out = {}
    for flag in ("0", "1"):
        monkeypatch.setenv("MMFREE_MIX_IN_PREP", flag)
        with api.Model(path, "fixed") as m:
            out[flag] = (m.generate_serve(prompts, 6), m.generate_serve(prompts[:3], 6))
    for k, ps in ((0, prompts), (1, prompts[:3])):
        ref = om.generate_serve(ps, 6)
        for a, b, c in zip(out["0"][k], out["1"][k], ref):
            assert np.array_equal(a, b)
            assert np.array_equal(b, c)


def test_wide_serve_64_streams_matches_oracle(cuda, orc, blob_cache):
    """64 lockstep streams of the "wide" model (H 768, I 5632): the tensor-core BitLinears
    with their cluster split-K reductions (the SwiGLU pair epilogue of gate_proj included)
    against the oracle, bit for bit."""
    path = B.cached_blob("wide", 0, blob_cache)
    om = orc.model(B.Blob.open(path))
    prompts = [B.seeded_ids(3 + k % 3, 800 + k, 512) for k in range(64)]
    with api.Model(path, "fixed") as m:
        got = m.generate_serve(prompts, 3)
    for a, c in zip(got, om.generate_serve(prompts, 3)):
        assert np.array_equal(a, c)


def test_serve_many_streams_matches_oracle(models, orc, blob_cache):
    """20 lockstep streams: decode rows go through the tensor-core matmul (ragged tile)."""
    m = models("small", "fixed")
    om = orc.model(B.Blob.open(B.cached_blob("small", 0, blob_cache)))
    prompts = [B.seeded_ids(5, 900 + k, 2048) for k in range(20)]
    for a, b in zip(m.generate_serve(prompts, 5), om.generate_serve(prompts, 5)):
        assert np.array_equal(a, b)


def test_serve_identical_prompts_match_generate(models):
    """model.hpp:58-59: B identical prompts + greedy give identical streams = generate()."""
    m = models("small", "fixed")
    p = B.seeded_ids(11, 42, 2048)
    single = m.generate(p, 12)
    for s in m.generate_serve([p] * 5, 12):
        assert np.array_equal(s, single)


def test_serve_session_matches_generate_serve(models):
    m = models("small", "fixed")
    prompts = [B.seeded_ids(9, 70 + k, 2048) for k in range(4)]
    ref = m.generate_serve(prompts, 8)
    first = m.serve_begin(prompts)
    got = [[f] for f in first]
    last = first
    for _ in range(3):  # step-wise with host ids
        last = m.serve_step(last)
        for b in range(4):
            got[b].append(last[b])
    rest = m.serve_run(4)  # device loop
    m.serve_end()
    for b in range(4):
        assert np.array_equal(np.concatenate([prompts[b], got[b], rest[b]]), ref[b])


def test_ragged_prompt_lengths_and_zero_tokens(models, orc, blob_cache):
    m = models("ragged", "fixed")
    om = orc.model(B.Blob.open(B.cached_blob("ragged", 0, blob_cache)))
    prompts = [B.seeded_ids(n, 300 + n, 300) for n in (3, 3, 7, 1, 7)]
    for gen in (0, 1, 5):
        got = m.generate_serve(prompts, gen)
        ref = om.generate_serve(prompts, gen)
        for a, b in zip(got, ref):
            assert np.array_equal(a, b)
    assert np.array_equal(m.generate(prompts[2], 0), prompts[2])


def test_eos_stops_streams(models):
    m = models("small", "fixed")
    p = B.seeded_ids(10, 5, 2048)
    full = m.generate(p, 10)
    eos = int(full[p.size + 3])
    cut = m.generate(p, 10, eos_id=eos)
    first = p.size + int(np.argmax(full[p.size:] == eos))
    assert np.array_equal(cut, full[:first + 1])
    streams = m.generate_serve([p, B.seeded_ids(10, 6, 2048)], 10, eos_id=eos)
    assert np.array_equal(streams[0], cut)


def _reference():
    import oracle
    if not os.path.exists(oracle.REF_SO):
        pytest.fail("prebuilt reference library missing (oracle/_ref travels with the repo)")
    return oracle.Reference()


def test_device_sampling_matches_reference(models, blob_cache):
    """Full-vocabulary temperature sampling on the device draws the reference's tokens for the
    same seed: its candidates are every token in index order, as the reference's are
    (hgrn_model.cpp:274-300), and the uniforms are the reference's own mt19937_64 draws."""
    R = _reference()
    rm = R.model(B.cached_blob("small", 0, blob_cache), 1)
    m = models("small", "fixed")
    p = B.seeded_ids(6, 9, 2048)
    ps = [p, B.seeded_ids(4, 10, 2048), B.seeded_ids(4, 11, 2048)]
    for temp, seed in ((0.8, 1), (1.5, 7), (0.3, 3)):
        assert np.array_equal(m.generate(p, 12, temperature=temp, seed=seed),
                              rm.generate(p, 12, temperature=temp, seed=seed))
        for a, b in zip(m.generate_serve(ps, 6, temperature=temp, seed=seed),
                        rm.generate_serve(ps, 6, temperature=temp, seed=seed)):
            assert np.array_equal(a, b)
    # eos stops a stream (its slot stays, its later draws are dropped) as in the reference
    s = rm.generate_serve(ps, 8, temperature=1.5, seed=7)
    eos = int(s[1][len(ps[1]) + 2])
    for a, b in zip(m.generate_serve(ps, 8, eos_id=eos, temperature=1.5, seed=7),
                    rm.generate_serve(ps, 8, eos=eos, temperature=1.5, seed=7)):
        assert np.array_equal(a, b)
    rm.close()


def _device_rule(lg, u, temp, k):
    """The device sampler's rule on the host: the k highest logits (ties to the lower index)
    in ascending index order, float p = exp((l - max) / temperature), double running sum,
    the first candidate whose sum reaches u * total."""
    lg = np.asarray(lg, np.float32)
    V = lg.size
    k = k if 0 < k < V else V
    cand = np.sort(np.lexsort((np.arange(V), -lg))[:k])
    z = ((lg[cand] - lg[cand].max()) / np.float32(temp)).astype(np.float32)
    pr = np.exp(z.astype(np.float64)).astype(np.float32).astype(np.float64)
    acc = np.cumsum(pr)
    j = int(np.searchsorted(acc, u * acc[-1], side="left"))
    return int(cand[min(j, cand.size - 1)])


def test_device_top_k_sampling_follows_its_rule(models, blob_cache):
    """With top_k the reference walks its candidates in std::nth_element's order, which no
    other implementation reproduces; the device walks them in ascending index order (the same
    distribution). Every drawn token is checked against that rule applied to the logits of
    its position and the stream's reference uniform."""
    R = _reference()
    m = models("small", "fixed")
    p = B.seeded_ids(6, 9, 2048)
    temp, k, seed = 1.5, 40, 7
    s = m.generate(p, 12, temperature=temp, top_k=k, seed=seed)
    u = R.uniforms(seed, 12)
    for t in range(12):
        assert s[p.size + t] == _device_rule(m.forward_last(s[:p.size + t]), u[t], temp, k)
    ps = [p, B.seeded_ids(4, 10, 2048)]
    for b, sb in enumerate(m.generate_serve(ps, 5, temperature=temp, top_k=k, seed=seed)):
        ub = R.uniforms(seed + b, 5)
        n0 = ps[b].size
        for t in range(5):
            assert sb[n0 + t] == _device_rule(m.forward_last(sb[:n0 + t]), ub[t], temp, k)


def test_host_sampling_matches_reference_with_top_k(cuda, blob_cache, monkeypatch):
    """MMFREE_HOST_SAMPLING=1 samples on the host with the reference's own algorithm
    (nth_element order included): draw-identical with top_k too."""
    monkeypatch.setenv("MMFREE_HOST_SAMPLING", "1")
    R = _reference()
    path = B.cached_blob("small", 0, blob_cache)
    rm = R.model(path, 1)
    p = B.seeded_ids(6, 9, 2048)
    with api.Model(path, "fixed") as m:
        for temp, k, seed in ((0.8, 0, 1), (1.5, 40, 7)):
            assert np.array_equal(m.generate(p, 12, temperature=temp, top_k=k, seed=seed),
                                  rm.generate(p, 12, temperature=temp, top_k=k, seed=seed))
            ps = [p, B.seeded_ids(4, 10, 2048)]
            for a, b in zip(m.generate_serve(ps, 6, temperature=temp, top_k=k, seed=seed),
                            rm.generate_serve(ps, 6, temperature=temp, top_k=k, seed=seed)):
                assert np.array_equal(a, b)
    rm.close()


def test_bad_token_ids(models):
    m = models("tiny", "fixed")
    for bad in ([1, 512], [-1]):
        with pytest.raises(_lib.MmfreeError) as e:
            m.generate(bad, 3)
        assert e.value.code == _lib.E_RANGE
    with pytest.raises(_lib.MmfreeError) as e:
        m.serve_step([1, 2, 3])
    assert e.value.code in (_lib.E_STATE, _lib.E_INVALID)


def test_missing_blob(cuda, tmp_path):
    with pytest.raises(_lib.MmfreeError) as e:
        api.Model(str(tmp_path / "nope.mmfree"))
    assert e.value.code == _lib.E_IO


def test_config0_370m_golden(models):
    """Benchmark configuration 0 (370M, 16 ids, 32 greedy tokens) bit for bit."""
    g = golden("config_370M.npz")
    m = models("370M", "fixed")
    stream = m.generate(g["prompt"], 32)
    assert np.array_equal(stream, g["fixed_stream"])
    assert bits_equal(m.forward_last(stream), g["fixed_logits"])
    mf = models("370M", "float")
    assert float_close(mf.forward_last(g["float_stream"]), g["float_logits"])


@pytest.mark.slow
def test_config2_1p3b_golden(models):
    """Benchmark configuration 2 (1.3B, 128-id prompt, 256 greedy tokens) bit for bit."""
    g = golden("config_1.3B.npz")
    m = models("1.3B", "fixed")
    stream = m.generate(g["prompt"], 256)
    assert np.array_equal(stream, g["fixed_stream"])
    assert bits_equal(m.forward_last(stream), g["fixed_logits"])
    mf = models("1.3B", "float")
    assert float_close(mf.forward_last(g["float_stream"]), g["float_logits"])
