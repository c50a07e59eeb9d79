"""B200-native (sm_100a) HGRN-Bit engine: a drop-in for the matmulfreellmCPU hot path.

The product is ``_lib/libmmfree_cuda.so`` (CUDA kernels + the C ABI of
``include/mmfree_cuda.h``); this package builds it (``build``), binds it (``_lib``), mirrors
the reference's C++ API in Python (``api``) and writes seeded ``model.mmfree`` blobs
(``blob``).
"""
from .api import (Config, Model, MmfreeError, bitlinear, bitlinear_cluster, hgrn_scan,  # noqa: F401
                  pack_ternary_host, packed_bytes, repack_ternary, rmsnorm,
                  rmsnorm_swishgate, swiglu, ternary_matmul)
