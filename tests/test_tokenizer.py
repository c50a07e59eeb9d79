"""Text mode of the CLI against the reference CLI, on the CPU (no model is run).

Both binaries tokenize with --gen 0 --print-ids and decode with --decode-ids, using the
synthetic tests/golden/tokenizer_toy.mmtok (tests/golden/make_tokenizer.py): ours
(matmulfreellmcpu_b200/cli/tokenizer.cpp) and the reference's own tokenizer
(oracle/_ref/mmfree-cli, built from cpp/src/io/tokenizer.cpp). Ids and bytes must match.
"""
from __future__ import annotations

import os
import subprocess

import numpy as np
import pytest

from conftest import GOLDEN, ROOT

TOK = os.path.join(GOLDEN, "tokenizer_toy.mmtok")
OURS = os.path.join(ROOT, "matmulfreellmcpu_b200", "_lib", "mmfree-cli")
REF = os.path.join(ROOT, "oracle", "_ref", "mmfree-cli")

TEXTS = ["The quick brown fox jumps over the lazy dog.", "", " ", "a", "  two  spaces  ",
         "Café crème, naïve façade", "中文 文本 测试", "emoji 😀 and 𝔘 fall back to bytes",
         "numbers 1024 2048 5632 32000 1.3B", "tab\tand\nnewline", "\xff-free but é at end é"]


def run(binary, *args, stdin=None):
    """(exit status, stdout) -- an empty prompt without BOS is an error in both CLIs."""
    r = subprocess.run([binary, "--tokenizer", TOK, *args], capture_output=True, input=stdin,
                       timeout=60)
    return r.returncode, r.stdout


@pytest.fixture(scope="module")
def binaries():
    for b in (OURS, REF):
        if not os.path.exists(b):
            pytest.fail(f"{b} missing (python -m matmulfreellmcpu_b200.build; make -C oracle ref)")
    return OURS, REF


def random_texts(n, seed):
    rng = np.random.default_rng(seed)
    alphabet = list("abcdefghijklmnopqrstuvwxyz THEQUICKéèüß中文本.,-0123456789") + ["😀", "ñ"]
    return ["".join(rng.choice(alphabet, size=int(rng.integers(1, 40)))) for _ in range(n)]


def test_encode_matches_reference(binaries):
    ours, ref = binaries
    for t in TEXTS + random_texts(40, 5):
        t = t.replace("\xff", "y")
        for extra in ([], ["--no-bos"]):
            assert run(ours, "--gen", "0", "--print-ids", *extra, t) == \
                run(ref, "--gen", "0", "--print-ids", *extra, t), repr(t)


def test_prompt_from_stdin_matches_reference(binaries):
    ours, ref = binaries
    data = "Once upon a time,  \n\n".encode()
    assert run(ours, "--gen", "0", "--print-ids", stdin=data) == \
        run(ref, "--gen", "0", "--print-ids", stdin=data)


def test_decode_matches_reference(binaries):
    ours, ref = binaries
    rng = np.random.default_rng(3)
    for _ in range(30):
        ids = ",".join(str(int(v)) for v in rng.integers(0, 1000, size=int(rng.integers(1, 25))))
        assert run(ours, "--decode-ids", ids) == run(ref, "--decode-ids", ids), ids
    # byte tokens that fuse into UTF-8, specials skipped, a leading space stripped
    for ids in ("1,3", "1,198,172,2", "300,301,302", "0,1,2"):
        assert run(ours, "--decode-ids", ids) == run(ref, "--decode-ids", ids), ids


def test_bad_tokenizer_file_fails_cleanly(tmp_path):
    bad = tmp_path / "bad.mmtok"
    bad.write_bytes(b"NOTATOK\x00")
    r = subprocess.run([OURS, "--tokenizer", str(bad), "--gen", "0", "--print-ids", "hi"],
                       capture_output=True, timeout=60)
    assert r.returncode != 0 and b"tokenizer" in r.stderr
