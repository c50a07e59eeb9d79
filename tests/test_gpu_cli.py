"""The CUDA mmfree-cli against the reference's own mmfree-cli (compiled from its sources):
same flags, same stdout, same --logits-out bytes (FixedQ510)."""
from __future__ import annotations

import os
import subprocess

import numpy as np
import pytest

from matmulfreellmcpu_b200 import blob as B
from matmulfreellmcpu_b200 import build as nb

pytestmark = pytest.mark.gpu


def _run(exe, args):
    r = subprocess.run([exe] + args, capture_output=True, text=True, timeout=600)
    return r.returncode, r.stdout, r.stderr


@pytest.mark.parametrize("mode", ["fixed", "float"])
def test_cli_matches_reference_cli(cuda, blob_cache, tmp_path, mode):
    import oracle
    assert os.path.exists(oracle.REF_CLI), "prebuilt reference CLI missing"
    blob = B.cached_blob("small", 0, blob_cache)
    ids = ",".join(str(int(v)) for v in B.seeded_ids(12, 3, 2048))
    common = ["--blob", blob, "--ids", ids, "--gen", "9", "--mode", mode]
    rc_r, out_r, _ = _run(oracle.REF_CLI, common + ["--logits-out", str(tmp_path / "r.bin")])
    rc_c, out_c, err_c = _run(nb.CLI, common + ["--logits-out", str(tmp_path / "c.bin")])
    assert rc_r == 0 and rc_c == 0, err_c
    lr = np.fromfile(tmp_path / "r.bin", np.float32)
    lc = np.fromfile(tmp_path / "c.bin", np.float32)
    assert lr.size == lc.size == 2048
    if mode == "fixed":
        assert out_c == out_r
        assert lr.tobytes() == lc.tobytes()
    else:
        assert np.abs(lc - lr).max() <= 1e-3 * float(lr.max() - lr.min())


def test_cli_errors(cuda, tmp_path):
    rc, _, err = _run(nb.CLI, ["--bogus"])
    assert rc == 2 and "unknown arg" in err
    # text mode without a tokenizer file beside the blob
    rc, _, err = _run(nb.CLI, ["some text prompt", "--blob", str(tmp_path / "model.mmfree")])
    assert rc == 1 and "tokenizer" in err
    rc, _, err = _run(nb.CLI, ["--ids", "1,2", "--blob", "/nonexistent.mmfree"])
    assert rc == 1 and "cannot open" in err


@pytest.mark.parametrize("extra", [[], ["--print-ids"], ["--mode", "float"], ["--no-eos"],
                                   ["--temp", "0.9", "--seed", "11"]])
def test_cli_text_mode_matches_reference_cli(cuda, blob_cache, extra):
    """Text in, text out (tokenize, generate with the EOS stop, stream the decoded text) with
    the synthetic tokenizer: stdout byte for byte equal to the reference CLI's (FixedQ510
    greedy, full-vocabulary sampling with a seed; Float greedy agrees on these prompts)."""
    import oracle
    from conftest import GOLDEN
    blob = B.cached_blob("small", 0, blob_cache)
    tok = os.path.join(GOLDEN, "tokenizer_toy.mmtok")
    for prompt in ("Once upon a time, there was", "Café crème 中文 😀"):
        common = ["--blob", blob, "--tokenizer", tok, "--gen", "24", *extra, prompt]
        # raw bytes: a random-init model emits byte-fallback tokens, not always valid UTF-8
        r = subprocess.run([oracle.REF_CLI] + common, capture_output=True, timeout=600)
        c = subprocess.run([nb.CLI] + common, capture_output=True, timeout=600)
        assert r.returncode == 0 and c.returncode == 0, c.stderr
        assert c.stdout == r.stdout, (prompt, c.stdout, r.stdout)
