"""The two benchmarked workloads at their own sizes, against the reference engine's outputs.

* Configuration 3: the 1.3B model serving 64 streams with 256-id prompts (seeds 1000 + b) --
  the launch shapes bench.py times (the grouped i/f/g tensor-core BitLinear at K = N = 2048,
  M = 64, the SwiGLU pair epilogue at I = 5632, the split-K cluster size chosen for them, and
  a 16,384-row prefill). First token + 16 greedy steps of every stream, bit for bit
  (tests/golden/config3_serve_1.3B.npz, from Model::generate_serve of the reference).
* Configuration 4: the 2.7B model, a 2048-id prompt (seed 4000): the last position's logits
  bit for bit in FixedQ510 and within 1e-3 of their range in Float
  (tests/golden/config4_prefill_2.7B.npz, from Model::forward of the reference); and the
  8 x 2048 batched prefill of the benchmark, whose first sequence must give the same token.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import bits_equal, golden
from matmulfreellmcpu_b200 import api
from matmulfreellmcpu_b200 import blob as B

pytestmark = [pytest.mark.gpu, pytest.mark.slow]


def float_close(got, ref, rel=1e-3):
    span = float(ref.max() - ref.min())
    return float(np.abs(got - ref).max()) <= rel * span


def test_config3_serve_64_streams_1p3b(cuda, blob_cache):
    g = golden("config3_serve_1.3B.npz")
    ref = g["gen_ids"]  # [64, 17]
    prompts = [B.seeded_ids(256, int(s)) for s in g["prompt_seeds"]]
    with api.Model(B.cached_blob("1.3B", 0, blob_cache), "fixed") as m:
        streams = m.generate_serve(prompts, ref.shape[1])
        got = np.stack([s[256:] for s in streams])
        assert np.array_equal(got, ref), np.argwhere(got != ref)[:8]
        # the step-wise session the benchmark times (graph replays from resident state)
        first = m.serve_begin(prompts)
        ids = m.serve_run(ref.shape[1] - 1)
        m.serve_end()
        assert np.array_equal(first, ref[:, 0])
        assert np.array_equal(ids, ref[:, 1:])


def test_config3_serve_repeatable(cuda, blob_cache):
    """Three more 64-stream serves of configuration 3 in one model: every run's ids equal the
    reference's. A race between overlapping kernels (the prefill of 16,384 rows followed by
    decoding) showed here as a few streams going wrong in some runs only."""
    g = golden("config3_serve_1.3B.npz")
    ref = g["gen_ids"]
    prompts = [B.seeded_ids(256, int(s)) for s in g["prompt_seeds"]]
    with api.Model(B.cached_blob("1.3B", 0, blob_cache), "fixed") as m:
        for rep in range(3):
            got = np.stack([s[256:] for s in m.generate_serve(prompts, ref.shape[1])])
            assert np.array_equal(got, ref), (rep, np.argwhere(got != ref)[:8])


def test_config4_prefill_2p7b(cuda, blob_cache):
    g = golden("config4_prefill_2.7B.npz")
    path = B.cached_blob("2.7B", 0, blob_cache)
    with api.Model(path, "fixed") as m:
        assert bits_equal(m.forward_last(g["ids"]), g["fixed_logits"])
        # the benchmark's batched prefill: 8 sequences x 2048 rows in one pass per layer
        seqs = [g["ids"]] + [B.seeded_ids(2048, 4001 + b) for b in range(7)]
        first = m.serve_begin(seqs)
        m.serve_end()
        assert first[0] == int(g["fixed_argmax"][0])
    with api.Model(path, "float") as mf:
        assert float_close(mf.forward_last(g["ids"]), g["float_logits"])
