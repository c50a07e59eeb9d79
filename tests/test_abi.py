"""CPU checks of the C ABI: the library loads, exports every symbol the header declares,
packs weights in the documented layout, parses blobs and rejects bad input cleanly."""
from __future__ import annotations

import ctypes as C
import os
import re
import struct

import numpy as np
import pytest

from conftest import ROOT
from matmulfreellmcpu_b200 import _lib, api
from matmulfreellmcpu_b200 import blob as B

HEADER = os.path.join(ROOT, "include", "mmfree_cuda.h")


def header_functions() -> set[str]:
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(r"\b(mmfree_cuda_\w+)\s*\(", text))


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    declared = header_functions()
    assert declared, "no declarations parsed"
    for name in declared:
        assert hasattr(lib, name), f"{name} declared but not exported"
    assert declared == set(_lib.SIGNATURES), "binding table and header disagree"
    assert lib.mmfree_cuda_abi_version() == 2


def numpy_pack(wq: np.ndarray) -> np.ndarray:
    """Restatement of the tiled 2-bit layout (csrc/common.cuh) in numpy."""
    n, k = wq.shape
    ng, kc = -(-n // 32), -(-k // 64)
    u = np.ones((ng * 32, kc * 64), np.uint32)
    u[:n, :k] = (wq.astype(np.int32) + 1).astype(np.uint32)
    u = u.reshape(ng, 32, kc, 4, 4, 4)  # group, row, chunk, word, g', j
    shifts = (8 * np.arange(4)[None, :] + 2 * np.arange(4)[:, None]).astype(np.uint32)  # [g', j]
    words = (u << shifts).sum(axis=(4, 5), dtype=np.uint64).astype(np.uint32)  # ng,32,kc,4
    return np.ascontiguousarray(words.transpose(0, 2, 1, 3)).view(np.uint8).reshape(-1)


@pytest.mark.parametrize("n,k", [(1, 1), (32, 64), (37, 100), (96, 1003), (300, 36)])
def test_host_pack_layout(n, k):
    rng = np.random.default_rng(n * 1000 + k)
    wq = rng.choice(np.array([-1, 0, 1], np.int8), size=(n, k))
    packed = api.pack_ternary_host(wq)
    assert packed.size == api.packed_bytes(n, k) == -(-n // 32) * -(-k // 64) * 512
    assert np.array_equal(packed, numpy_pack(wq))


def test_host_pack_rejects_non_ternary():
    wq = np.zeros((4, 8), np.int8)
    wq[1, 3] = 2
    with pytest.raises(_lib.MmfreeError) as e:
        api.pack_ternary_host(wq)
    assert e.value.code == _lib.E_RANGE


def test_blob_config_roundtrip(blob_cache):
    path = B.cached_blob("tiny", 0, blob_cache)
    c = api.blob_config(path)
    assert (c.vocab_size, c.hidden_size, c.num_hidden_layers, c.intermediate_size) == \
        (512, 64, 2, 96)
    assert c.use_lower_bound and abs(c.rms_norm_eps - 1e-6) < 1e-12


def test_blob_errors(tmp_path, blob_cache):
    bad = tmp_path / "bad.mmfree"
    bad.write_bytes(b"NOTMAGIC" + b"\0" * 64)
    with pytest.raises(_lib.MmfreeError) as e:
        api.blob_config(str(bad))
    assert e.value.code == _lib.E_IO and "bad magic" in str(e.value)
    with pytest.raises(_lib.MmfreeError) as e:
        api.blob_config(str(tmp_path / "missing.mmfree"))
    assert e.value.code == _lib.E_IO and "cannot open" in str(e.value)
    trunc = tmp_path / "trunc.mmfree"
    good = open(B.cached_blob("tiny", 0, blob_cache), "rb").read()
    trunc.write_bytes(good[:200])
    with pytest.raises(_lib.MmfreeError) as e:
        api.blob_config(str(trunc))
    assert e.value.code == _lib.E_IO
    past = tmp_path / "past.mmfree"
    hl = struct.unpack("<Q", good[8:16])[0]
    past.write_bytes(good[: 16 + hl + 64])  # header intact, data section cut
    with pytest.raises(_lib.MmfreeError) as e:
        api.blob_config(str(past))
    assert "past end of file" in str(e.value)


def test_model_open_without_gpu_fails_loudly(blob_cache):
    """No CPU fallback: on a machine without a device, opening a model is a CUDA error."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a CUDA device is present")
    with pytest.raises(_lib.MmfreeError) as e:
        api.Model(B.cached_blob("tiny", 0, blob_cache))
    assert e.value.code == _lib.E_CUDA


def test_null_arguments_are_rejected():
    lib = _lib.lib()
    rc = lib.mmfree_cuda_bitlinear(None, None, None, None, 1.0, 1, 8, 8, 1e-6, None, 1, 10,
                                   None, None)
    assert rc == _lib.E_INVALID
    rc = lib.mmfree_cuda_bitlinear(None, None, None, None, 1.0, 1, 8, 8, 1e-6, None, 7, 10,
                                   None, None)
    assert rc == _lib.E_INVALID
    assert lib.mmfree_cuda_serve_end(None) == _lib.E_INVALID
    cfg = C.create_string_buffer(128)
    assert lib.mmfree_cuda_blob_config(None, cfg) == _lib.E_INVALID


def test_seeded_blob_is_deterministic(tmp_path):
    a = B.write_random_blob(str(tmp_path / "a.mmfree"), 300, 36, 2, 52, seed=5)
    b = B.write_random_blob(str(tmp_path / "b.mmfree"), 300, 36, 2, 52, seed=5)
    c = B.write_random_blob(str(tmp_path / "c.mmfree"), 300, 36, 2, 52, seed=6)
    ra, rb, rc = (open(p, "rb").read() for p in (a, b, c))
    assert ra == rb and ra != rc
    blob = B.Blob.open(a)
    wq = blob["model.layers.1.gate_proj.wq"]
    assert wq.shape == (104, 36) and set(np.unique(wq)) <= {-1, 0, 1}
    assert np.allclose(blob["lower_bounds"][:, 0], np.arange(2) / 2)


# ---- model.mmfree2 (packed load cache)

@pytest.mark.parametrize("n,k", [(37, 100), (64, 128), (96, 1003), (1, 1), (300, 64)])
def test_numpy_packer_matches_c_abi_packer(n, k):
    """blob.pack_ternary (the converter's packer) writes exactly the library's format."""
    from matmulfreellmcpu_b200 import blob as B
    w = np.random.default_rng(n * 7 + k).integers(-1, 2, size=(n, k)).astype(np.int8)
    ref = np.zeros(B.packed_nbytes(n, k), np.uint8)
    assert _lib.lib().mmfree_cuda_pack_ternary_host(ref.ctypes.data, w.ctypes.data, n, k) == 0
    assert np.array_equal(B.pack_ternary(w), ref)


def test_packed_blob_roundtrip(tmp_path, blob_cache):
    """model.mmfree -> model.mmfree2 keeps every tensor; ternary weights become the tiled
    2-bit bytes of the same matrix."""
    from matmulfreellmcpu_b200 import blob as B
    src = B.cached_blob("ragged", 0, blob_cache)
    dst = B.write_packed_blob(src, str(tmp_path / "ragged.mmfree2"))
    a, b = B.Blob.open(src), B.Blob.open(dst)
    assert a.config == b.config and set(a.tensors) == set(b.tensors)
    npacked = 0
    for name, t in a.tensors.items():
        if name.endswith(".wq"):
            assert np.array_equal(b[name], B.pack_ternary(t))
            npacked += 1
        else:
            assert np.array_equal(b[name], t)
    assert npacked == 1 + 6 * a.config["num_hidden_layers"]
    with pytest.raises(ValueError):
        B.pack_ternary(np.full((2, 2), 2, np.int8))
