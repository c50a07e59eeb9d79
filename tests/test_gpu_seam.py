"""The reference engine's own Model with the CUDA TernaryBackend injected.

``oracle/_ref/seam_check`` links the unmodified reference (Model, bitlinear, CpuBackend;
compiled from its sources by ``oracle/Makefile``) with ``include/mmfree_cuda_backend.hpp``
and runs forward, generate and generate_serve once with the default CpuBackend and once
with ``mmfree::cuda::CudaTernaryBackend`` set through ``Model::set_backend``
(matmulfreellmCPU cpp/include/mmfree/model.hpp:74-79). Every result must be bit-identical.
The batch argument sets ``TernaryBackend::batch_size``, i.e. how many rows each seam call
carries (1: the per-row path; 7: ragged batches of the 37-token prefill).
"""
from __future__ import annotations

import os
import subprocess

import pytest

import oracle
from matmulfreellmcpu_b200 import blob as B

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name,batch", [("small", 256), ("small", 1), ("ragged", 7)])
def test_reference_model_with_cuda_backend_matches_cpu_backend(cuda, blob_cache, name, batch):
    assert os.path.exists(oracle.SEAM_CHECK), "seam_check not built (make -C oracle seam)"
    path = B.cached_blob(name, 0, blob_cache)
    r = subprocess.run([oracle.SEAM_CHECK, path, str(batch)], capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    for check in ("forward_logits", "generate_ids", "generate_serve_ids"):
        assert f"{check} match" in r.stdout, r.stdout
