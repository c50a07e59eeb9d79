"""TEST INFRASTRUCTURE ONLY: CPU checkers for the CUDA path.

Two checkers, both loaded through ctypes:

* ``Oracle`` -- ``_build/liboracle.so``, the plain-C restatement of the reference numerics
  (``mmfree_oracle.c``). Builds anywhere with gcc.
* ``Reference`` -- ``_ref/libmmfree_ref.so``, the reference engine itself compiled from its
  own sources (``Makefile``), driven through ``ref_ops.cpp``. Built where the reference
  tree is present; the prebuilt library travels with the repository copy otherwise.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` use
this package. The product (``matmulfreellmcpu_b200``) never imports it.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "_build", "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libmmfree_ref.so")
REF_CLI = os.path.join(HERE, "_ref", "mmfree-cli")

F32P = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
I32P = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
I8P = np.ctypeslib.ndpointer(np.int8, flags="C_CONTIGUOUS")
I64P = np.ctypeslib.ndpointer(np.int64, flags="C_CONTIGUOUS")
SZ = C.c_size_t
VP = C.c_void_p


SEAM_CHECK = os.path.join(HERE, "_ref", "seam_check")


def reference_tree() -> str:
    """The reference checkout: $MMFREE_REFERENCE, else a sibling of this repository named
    ``reference`` (the Makefile's default too)."""
    return os.environ.get("MMFREE_REFERENCE",
                          os.path.abspath(os.path.join(HERE, "..", "..", "reference")))


def build(ref: bool | None = None) -> None:
    """Run the oracle Makefile: the restatement always; the reference engine, and the seam
    check that runs it with the CUDA backend injected, where the reference tree is present
    (``ref`` None: detect it)."""
    if ref is None:
        ref = os.path.isdir(os.path.join(reference_tree(), "cpp"))
    targets = ["oracle"] + (["ref", "seam"] if ref else [])
    env = dict(os.environ, MMFREE_REFERENCE=reference_tree())
    subprocess.run(["make", "-s", "-C", HERE] + targets, check=True, env=env)


def _f(a):
    return np.ascontiguousarray(a, np.float32)


def _ptr(a):
    return None if a is None else a.ctypes.data_as(VP)


class _Proj(C.Structure):
    _fields_ = [("wq", VP), ("normw", VP), ("scale_w", C.c_float), ("in_dim", SZ),
                ("out_dim", SZ)]


class _Layer(C.Structure):
    _fields_ = [("attn_norm", VP), ("mlp_norm", VP), ("g_norm", VP), ("proj", _Proj * 6)]


class _Model(C.Structure):
    _fields_ = [("vocab", SZ), ("hidden", SZ), ("layers", SZ), ("inter", SZ),
                ("use_lower_bound", C.c_int), ("eps", C.c_float), ("embeddings", VP),
                ("final_norm", VP), ("lower_bounds", VP), ("lm_head", _Proj),
                ("layer", C.POINTER(_Layer))]


_PROJS = ("i_proj", "f_proj", "g_proj", "o_proj", "gate_proj", "down_proj")


class Oracle:
    """ctypes front of the C restatement."""

    def __init__(self, path: str = ORACLE_SO):
        if not os.path.exists(path):
            build(ref=False)
        L = self.lib = C.CDLL(path)
        L.orc_sumsq.restype = C.c_float
        L.orc_sumsq.argtypes = [F32P, SZ]
        L.orc_exp8_lane.restype = C.c_float
        L.orc_exp8_lane.argtypes = [C.c_float]
        L.orc_expf_tail.restype = C.c_float
        L.orc_expf_tail.argtypes = [C.c_float]
        L.orc_quant_q510.argtypes = [I32P, F32P, C.c_float, SZ]
        for n in ("orc_sigmoid", "orc_silu"):
            getattr(L, n).argtypes = [F32P, F32P, SZ]
        L.orc_swiglu.argtypes = [F32P, F32P, F32P, SZ]
        L.orc_hgrn_step.argtypes = [F32P, F32P, F32P, F32P, SZ]
        L.orc_rmsnorm.argtypes = [F32P, F32P, F32P, SZ, SZ, C.c_float]
        L.orc_bitlinear.argtypes = [F32P, F32P, F32P, I8P, C.c_float, SZ, SZ, SZ, C.c_float, VP,
                                    C.c_int, C.c_int, VP]
        L.orc_hgrn_scan.argtypes = [F32P, F32P, F32P, SZ, SZ, VP]
        L.orc_rmsnorm_swishgate.argtypes = [F32P, F32P, F32P, F32P, SZ, SZ, C.c_float]
        for n in ("orc_model_forward", "orc_model_generate", "orc_model_generate_serve",
                  "orc_model_forward_trace"):
            getattr(L, n).restype = C.c_int

    # -- primitives
    def sumsq(self, x):
        x = _f(x)
        return np.float32(self.lib.orc_sumsq(x, x.size))

    def quant_q510(self, y, qs=1024.0):
        y = _f(y)
        out = np.empty(y.size, np.int32)
        self.lib.orc_quant_q510(out, y, qs, y.size)
        return out

    def _unary(self, name, x):
        x = _f(x)
        out = np.empty_like(x)
        getattr(self.lib, name)(out, x, x.size)
        return out

    def sigmoid(self, x):
        return self._unary("orc_sigmoid", x)

    def silu(self, x):
        return self._unary("orc_silu", x)

    def swiglu(self, a, b):
        a, b = _f(a), _f(b)
        out = np.empty_like(a)
        self.lib.orc_swiglu(out, a, b, a.size)
        return out

    def rmsnorm(self, x, w, eps=1e-6):
        x, w = _f(x), _f(w)
        rows, cols = x.shape
        y = np.empty_like(x)
        self.lib.orc_rmsnorm(y, x, w, rows, cols, eps)
        return y

    def bitlinear(self, x, nw, wq, scale_w, eps=1e-6, act_quant=1, frac_bits=10,
                  want_norm=False):
        """Returns (out [M,N], acc [M,N] int32 or None, norm [M,K] or None)."""
        x, nw = _f(x), _f(nw)
        wq = np.ascontiguousarray(wq, np.int8)
        M, K = x.shape
        N = wq.shape[0]
        out = np.empty((M, N), np.float32)
        acc = np.empty((M, N), np.int32) if act_quant == 1 else None
        norm = np.empty((M, K), np.float32) if want_norm else None
        self.lib.orc_bitlinear(out, x, nw, wq, float(scale_w), M, K, N, eps, _ptr(norm),
                               act_quant, frac_bits, _ptr(acc))
        return out, acc, norm

    def hgrn_scan(self, i, f, state=None):
        i, f = _f(i), _f(f)
        T, D = i.shape
        out = np.empty_like(i)
        st = None if state is None else _f(state).copy()
        self.lib.orc_hgrn_scan(out, i, f, T, D, _ptr(st))
        return out, st

    def rmsnorm_swishgate(self, g, o, w, eps=1e-6):
        g, o, w = _f(g), _f(o), _f(w)
        rows, cols = g.shape
        out = np.empty_like(g)
        self.lib.orc_rmsnorm_swishgate(out, g, o, w, rows, cols, eps)
        return out

    # -- model
    def model(self, blob) -> "OracleModel":
        return OracleModel(self, blob)


class OracleModel:
    """Binds an ``orc_model`` struct to the arrays of a ``matmulfreellmcpu_b200.blob.Blob``."""

    def __init__(self, oracle: Oracle, blob):
        self.o, self.blob = oracle, blob
        c = blob.config
        self.V, self.H = c["vocab_size"], c["hidden_size"]
        self.L, self.I = c["num_hidden_layers"], c["intermediate_size"]
        keep = []

        def arr(name):
            a = np.ascontiguousarray(blob[name])
            keep.append(a)
            return a.ctypes.data_as(VP)

        def proj(tag):
            wq = blob[f"{tag}.wq"]
            return _Proj(arr(f"{tag}.wq"), arr(f"{tag}.normw"),
                         float(blob[f"{tag}.scale_w"][0]), wq.shape[1], wq.shape[0])

        layers = (_Layer * self.L)()
        for l in range(self.L):
            p = f"model.layers.{l}"
            layers[l].attn_norm = arr(f"{p}.attn_norm.w")
            layers[l].mlp_norm = arr(f"{p}.mlp_norm.w")
            layers[l].g_norm = arr(f"{p}.g_norm.w")
            for j, tag in enumerate(_PROJS):
                layers[l].proj[j] = proj(f"{p}.{tag}")
        self._keep, self._layers = keep, layers
        self.s = _Model(self.V, self.H, self.L, self.I, int(c.get("use_lower_bound", True)),
                        float(c.get("rms_norm_eps", 1e-6)), arr("model.embeddings"),
                        arr("model.norm.w"),
                        arr("lower_bounds") if "lower_bounds" in blob.tensors else None,
                        proj("lm_head"), C.cast(layers, C.POINTER(_Layer)))

    def forward(self, ids, act_quant=1, frac_bits=10):
        ids = np.ascontiguousarray(ids, np.int64)
        lg = np.empty((ids.size, self.V), np.float32)
        rc = self.o.lib.orc_model_forward(C.byref(self.s), act_quant, frac_bits,
                                          ids.ctypes.data_as(VP), ids.size, lg.ctypes.data_as(VP))
        if rc:
            raise ValueError("oracle forward rejected its input")
        return lg

    def forward_trace(self, ids, act_quant=1, frac_bits=10):
        """(logits [T,V], trace [1+3L, T, H]: embeddings, then per layer recur/resid/h)."""
        ids = np.ascontiguousarray(ids, np.int64)
        lg = np.empty((ids.size, self.V), np.float32)
        tr = np.empty((1 + 3 * self.L, ids.size, self.H), np.float32)
        rc = self.o.lib.orc_model_forward_trace(C.byref(self.s), act_quant, frac_bits,
                                                ids.ctypes.data_as(VP), ids.size,
                                                lg.ctypes.data_as(VP), tr.ctypes.data_as(VP))
        if rc:
            raise ValueError("oracle forward rejected its input")
        return lg, tr

    def generate(self, ids, gen, act_quant=1, frac_bits=10):
        """Returns (full id stream, last-step logits)."""
        ids = np.ascontiguousarray(ids, np.int64)
        out = np.empty(ids.size + gen, np.int64)
        lg = np.empty(self.V, np.float32)
        rc = self.o.lib.orc_model_generate(C.byref(self.s), act_quant, frac_bits,
                                           ids.ctypes.data_as(VP), ids.size, gen,
                                           out.ctypes.data_as(VP), lg.ctypes.data_as(VP))
        if rc:
            raise ValueError("oracle generate rejected its input")
        return out, lg

    def generate_serve(self, prompts, gen, act_quant=1, frac_bits=10):
        ps = [np.ascontiguousarray(p, np.int64) for p in prompts]
        B = len(ps)
        stride = max(p.size for p in ps) + max(gen, 1)
        out = np.zeros((B, stride), np.int64)
        lens = np.zeros(B, np.uint64)
        parr = (VP * B)(*[p.ctypes.data_as(VP) for p in ps])
        larr = (SZ * B)(*[p.size for p in ps])
        rc = self.o.lib.orc_model_generate_serve(C.byref(self.s), act_quant, frac_bits, B, parr,
                                                 larr, gen, out.ctypes.data_as(VP), stride,
                                                 lens.ctypes.data_as(VP))
        if rc:
            raise ValueError("oracle generate_serve rejected its input")
        return [out[b, :int(lens[b])] for b in range(B)]


class Reference:
    """ctypes front of the reference engine compiled from its own sources."""

    def __init__(self, path: str = REF_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing: run `make -C oracle ref` where the "
                                    "reference tree is present")
        L = self.lib = C.CDLL(path)
        L.ref_last_error.restype = C.c_char_p
        L.ref_sumsq.restype = C.c_float
        L.ref_sumsq.argtypes = [F32P, SZ]
        L.ref_expf_poly.restype = C.c_float
        L.ref_expf_poly.argtypes = [C.c_float]
        L.ref_quant_q510.argtypes = [I32P, F32P, C.c_float, SZ]
        for n in ("ref_sigmoid", "ref_silu"):
            getattr(L, n).argtypes = [F32P, F32P, SZ]
        L.ref_swiglu.argtypes = [F32P, F32P, F32P, SZ]
        L.ref_hgrn_step.argtypes = [F32P, F32P, F32P, F32P, SZ]
        L.ref_rmsnorm.argtypes = [F32P, F32P, F32P, SZ, SZ, C.c_float]
        L.ref_bitlinear.argtypes = [F32P, F32P, F32P, I8P, C.c_float, SZ, SZ, SZ, C.c_float, VP,
                                    C.c_int, C.c_int, VP]
        L.ref_hgrn_scan.argtypes = [F32P, F32P, F32P, SZ, SZ, VP]
        L.ref_rmsnorm_swishgate.argtypes = [F32P, F32P, F32P, F32P, SZ, SZ, C.c_float]
        L.ref_model_open.restype = VP
        L.ref_model_open.argtypes = [C.c_char_p, C.c_int, C.c_int]
        L.ref_model_close.argtypes = [VP]
        L.ref_threads.restype = C.c_int
        L.ref_set_threads.argtypes = [C.c_int]
        for n in ("ref_model_generate", "ref_model_forward", "ref_model_generate_serve",
                  "ref_model_bench_generate", "ref_model_bench_serve"):
            getattr(L, n).restype = C.c_int

    def threads(self) -> int:
        return self.lib.ref_threads()

    def set_threads(self, n: int) -> None:
        self.lib.ref_set_threads(n)

    def uniforms(self, seed: int, n: int) -> np.ndarray:
        """The first n uniforms the reference's sampler draws for a stream seeded `seed`."""
        out = np.empty(n, np.float64)
        self.lib.ref_uniforms(C.c_uint64(seed), SZ(n), out.ctypes.data_as(VP))
        return out

    def sumsq(self, x):
        x = _f(x)
        return np.float32(self.lib.ref_sumsq(x, x.size))

    def quant_q510(self, y, qs=1024.0):
        y = _f(y)
        out = np.empty(y.size, np.int32)
        self.lib.ref_quant_q510(out, y, qs, y.size)
        return out

    def _unary(self, name, x):
        x = _f(x)
        out = np.empty_like(x)
        getattr(self.lib, name)(out, x, x.size)
        return out

    def sigmoid(self, x):
        return self._unary("ref_sigmoid", x)

    def silu(self, x):
        return self._unary("ref_silu", x)

    def swiglu(self, a, b):
        a, b = _f(a), _f(b)
        out = np.empty_like(a)
        self.lib.ref_swiglu(out, a, b, a.size)
        return out

    def rmsnorm(self, x, w, eps=1e-6):
        x, w = _f(x), _f(w)
        rows, cols = x.shape
        y = np.empty_like(x)
        self.lib.ref_rmsnorm(y, x, w, rows, cols, eps)
        return y

    def bitlinear(self, x, nw, wq, scale_w, eps=1e-6, act_quant=1, frac_bits=10,
                  want_norm=False):
        x, nw = _f(x), _f(nw)
        wq = np.ascontiguousarray(wq, np.int8)
        M, K = x.shape
        N = wq.shape[0]
        out = np.empty((M, N), np.float32)
        acc = np.empty((M, N), np.int32) if act_quant == 1 else None
        norm = np.empty((M, K), np.float32) if want_norm else None
        self.lib.ref_bitlinear(out, x, nw, wq, float(scale_w), M, K, N, eps, _ptr(norm),
                               act_quant, frac_bits, _ptr(acc))
        return out, acc, norm

    def hgrn_scan(self, i, f, state=None):
        i, f = _f(i), _f(f)
        T, D = i.shape
        out = np.empty_like(i)
        st = None if state is None else _f(state).copy()
        self.lib.ref_hgrn_scan(out, i, f, T, D, _ptr(st))
        return out, st

    def rmsnorm_swishgate(self, g, o, w, eps=1e-6):
        g, o, w = _f(g), _f(o), _f(w)
        rows, cols = g.shape
        out = np.empty_like(g)
        self.lib.ref_rmsnorm_swishgate(out, g, o, w, rows, cols, eps)
        return out

    def model(self, blob_path: str, act_quant: int = 1, frac_bits: int = 10) -> "RefModel":
        return RefModel(self, blob_path, act_quant, frac_bits)


class RefModel:
    def __init__(self, ref: Reference, path: str, act_quant: int, frac_bits: int):
        self.r = ref
        self.h = ref.lib.ref_model_open(path.encode(), act_quant, frac_bits)
        if not self.h:
            raise RuntimeError(ref.lib.ref_last_error().decode())
        cfg = (SZ * 6)()
        ref.lib.ref_model_config(VP(self.h), cfg)
        self.V = cfg[0]

    def close(self):
        if self.h:
            self.r.lib.ref_model_close(VP(self.h))
            self.h = None

    def __del__(self):
        self.close()

    def _err(self):
        return RuntimeError(self.r.lib.ref_last_error().decode())

    def generate(self, ids, gen, eos=-1, temperature=0.0, top_k=0, seed=0):
        ids = np.ascontiguousarray(ids, np.int64)
        out = np.empty(ids.size + gen, np.int64)
        n = SZ(0)
        rc = self.r.lib.ref_model_generate(VP(self.h), ids.ctypes.data_as(VP), SZ(ids.size),
                                           SZ(gen), C.c_int64(eos), C.c_float(temperature),
                                           C.c_int(top_k), C.c_uint64(seed),
                                           out.ctypes.data_as(VP), SZ(out.size), C.byref(n))
        if rc:
            raise self._err()
        return out[:n.value]

    def forward(self, ids):
        ids = np.ascontiguousarray(ids, np.int64)
        lg = np.empty((ids.size, self.V), np.float32)
        if self.r.lib.ref_model_forward(VP(self.h), ids.ctypes.data_as(VP), SZ(ids.size),
                                        lg.ctypes.data_as(VP)):
            raise self._err()
        return lg

    def generate_serve(self, prompts, gen, eos=-1, temperature=0.0, top_k=0, seed=0):
        ps = [np.ascontiguousarray(p, np.int64) for p in prompts]
        B = len(ps)
        stride = max(p.size for p in ps) + max(gen, 1)
        out = np.zeros((B, stride), np.int64)
        lens = np.zeros(B, np.uint64)
        parr = (VP * B)(*[p.ctypes.data_as(VP) for p in ps])
        larr = (SZ * B)(*[p.size for p in ps])
        rc = self.r.lib.ref_model_generate_serve(VP(self.h), SZ(B), parr, larr, SZ(gen),
                                                 C.c_int64(eos), C.c_float(temperature),
                                                 C.c_int(top_k), C.c_uint64(seed),
                                                 out.ctypes.data_as(VP), SZ(stride),
                                                 lens.ctypes.data_as(VP))
        if rc:
            raise self._err()
        return [out[b, :int(lens[b])] for b in range(B)]

    def bench_generate(self, ids, gen):
        ids = np.ascontiguousarray(ids, np.int64)
        p, d, n = C.c_double(), C.c_double(), SZ()
        if self.r.lib.ref_model_bench_generate(VP(self.h), ids.ctypes.data_as(VP), SZ(ids.size),
                                               SZ(gen), C.byref(p), C.byref(d), C.byref(n)):
            raise self._err()
        return p.value, d.value, n.value

    def bench_serve(self, prompts, gen):
        ps = [np.ascontiguousarray(p, np.int64) for p in prompts]
        B = len(ps)
        parr = (VP * B)(*[p.ctypes.data_as(VP) for p in ps])
        larr = (SZ * B)(*[p.size for p in ps])
        p, d, n = C.c_double(), C.c_double(), SZ()
        if self.r.lib.ref_model_bench_serve(VP(self.h), SZ(B), parr, larr, SZ(gen), C.byref(p),
                                            C.byref(d), C.byref(n)):
            raise self._err()
        return p.value, d.value, n.value
