"""Python front of the C ABI, mirroring the reference engine's C++ API.

``Model`` mirrors ``mmfree::Model`` (matmulfreellmCPU cpp/include/mmfree/model.hpp:33-80)
plus the step-wise serving session; the kernel functions mirror ``mmfree::bitlinear``,
``bitlinear_cluster``, ``rmsnorm``, ``swiglu``, ``hgrn_scan`` and ``rmsnorm_swishgate``
(kernels.hpp:29-68) on CUDA tensors (torch is used only to hold device memory and streams).
Errors raise :class:`MmfreeError`, the counterpart of the reference's std::runtime_error.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from ._lib import ACT_FIXED_Q510, ACT_FLOAT, MmfreeError, check, lib  # noqa: F401

ActQuant = {"float": ACT_FLOAT, "fixed": ACT_FIXED_Q510}


def _aq(mode) -> int:
    if isinstance(mode, str):
        return ActQuant[mode]
    return int(mode)


def _ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(stream=None) -> int | None:
    if stream is not None:
        return stream.cuda_stream
    import torch
    return torch.cuda.current_stream().cuda_stream


def _i64(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.int64))


@dataclass
class Config:  # mmfree::Config (config.hpp:8-21)
    vocab_size: int
    hidden_size: int
    num_hidden_layers: int
    num_heads: int
    expand_ratio: int
    intermediate_size: int
    use_lower_bound: bool
    use_short_conv: bool
    rms_norm_eps: float


class _CConfig(C.Structure):
    _fields_ = [(n, C.c_size_t) for n in ("vocab_size", "hidden_size", "num_hidden_layers",
                                           "num_heads", "expand_ratio", "intermediate_size")] + \
               [("use_lower_bound", C.c_int), ("use_short_conv", C.c_int),
                ("rms_norm_eps", C.c_float)]


def _config(c: "_CConfig") -> Config:
    return Config(c.vocab_size, c.hidden_size, c.num_hidden_layers, c.num_heads, c.expand_ratio,
                  c.intermediate_size, bool(c.use_lower_bound), bool(c.use_short_conv),
                  float(c.rms_norm_eps))


def blob_config(path: str) -> Config:
    """Header of a model.mmfree blob (host only, no GPU needed)."""
    c = _CConfig()
    check(lib().mmfree_cuda_blob_config(path.encode(), C.byref(c)))
    return _config(c)


class Model:
    """Device-resident HGRN-Bit model opened from a ``model.mmfree`` blob."""

    def __init__(self, blob_path: str, act_quant="fixed", frac_bits: int = 10, device: int = 0):
        h = C.c_void_p()
        check(lib().mmfree_cuda_model_open(blob_path.encode(), device, _aq(act_quant), frac_bits,
                                           C.byref(h)))
        self._h = h
        c = _CConfig()
        check(lib().mmfree_cuda_model_config(self._h, C.byref(c)))
        self.config = _config(c)
        self.device = device

    @classmethod
    def open_tp(cls, blob_path: str, act_quant, rank: int, world: int, nccl_id: bytes,
                frac_bits: int = 10, device: int = 0) -> "Model":
        """Rank ``rank`` of a ``world``-way tensor-parallel prefill handle (collective: every
        rank opens its handle with the same NCCL id; see ``matmulfreellmcpu_b200.tp``)."""
        if len(nccl_id) != 128:
            raise ValueError("an NCCL unique id has 128 bytes")
        self = cls.__new__(cls)
        h = C.c_void_p()
        buf = (C.c_ubyte * 128).from_buffer_copy(nccl_id)
        check(lib().mmfree_cuda_model_open_tp(blob_path.encode(), device, _aq(act_quant), frac_bits,
                                              rank, world, buf, C.byref(h)))
        self._h = h
        c = _CConfig()
        check(lib().mmfree_cuda_model_config(self._h, C.byref(c)))
        self.config = _config(c)
        self.device = device
        return self

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().mmfree_cuda_model_close(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def weight_bytes(self) -> int:
        return lib().mmfree_cuda_model_weight_bytes(self._h)

    def generate(self, ids, new_tokens: int, eos_id: int = -1, temperature: float = 0.0,
                 top_k: int = 0, seed: int = 0) -> np.ndarray:
        """Model::generate: prompt + generated ids."""
        ids = _i64(ids)
        out = np.empty(ids.size + new_tokens, np.int64)
        n = C.c_size_t()
        check(lib().mmfree_cuda_generate(self._h, ids.ctypes.data, ids.size, new_tokens, eos_id,
                                         temperature, top_k, seed, out.ctypes.data, out.size,
                                         C.byref(n)))
        return out[:n.value]

    def forward(self, ids) -> np.ndarray:
        """Model::forward: logits [T, vocab] from a zero state."""
        ids = _i64(ids)
        lg = np.empty((ids.size, self.config.vocab_size), np.float32)
        check(lib().mmfree_cuda_forward(self._h, ids.ctypes.data, ids.size, lg.ctypes.data))
        return lg

    def forward_trace(self, ids):
        """(logits [T, V], trace [1 + 3L, T, H]): embeddings, then per layer the recurrence
        output, the residual after o_proj and the layer output."""
        ids = _i64(ids)
        c = self.config
        lg = np.empty((ids.size, c.vocab_size), np.float32)
        tr = np.empty((1 + 3 * c.num_hidden_layers, ids.size, c.hidden_size), np.float32)
        check(lib().mmfree_cuda_forward_trace(self._h, ids.ctypes.data, ids.size, lg.ctypes.data,
                                              tr.ctypes.data))
        return lg, tr

    def forward_last(self, ids) -> np.ndarray:
        ids = _i64(ids)
        lg = np.empty(self.config.vocab_size, np.float32)
        check(lib().mmfree_cuda_forward_last(self._h, ids.ctypes.data, ids.size, lg.ctypes.data))
        return lg

    @staticmethod
    def _prompts(prompts):
        ps = [_i64(p) for p in prompts]
        arr = (C.c_void_p * len(ps))(*[p.ctypes.data for p in ps])
        lens = (C.c_size_t * len(ps))(*[p.size for p in ps])
        return ps, arr, lens

    def generate_serve(self, prompts, new_tokens: int, eos_id: int = -1,
                       temperature: float = 0.0, top_k: int = 0, seed: int = 0):
        """Model::generate_serve: list of B full id streams."""
        ps, arr, lens = self._prompts(prompts)
        B = len(ps)
        stride = max(p.size for p in ps) + max(new_tokens, 1)
        out = np.zeros((B, stride), np.int64)
        out_lens = np.zeros(B, np.uint64)
        check(lib().mmfree_cuda_generate_serve(self._h, B, arr, lens, new_tokens, eos_id,
                                               temperature, top_k, seed, out.ctypes.data, stride,
                                               out_lens.ctypes.data))
        return [out[b, :int(out_lens[b])] for b in range(B)]

    def serve_begin(self, prompts) -> np.ndarray:
        ps, arr, lens = self._prompts(prompts)
        first = np.empty(len(ps), np.int64)
        check(lib().mmfree_cuda_serve_begin(self._h, len(ps), arr, lens, first.ctypes.data))
        self._serve_b = len(ps)
        return first

    def serve_step(self, in_ids, out=None) -> np.ndarray:
        in_ids = _i64(in_ids)
        out = np.empty(in_ids.size, np.int64) if out is None else out
        check(lib().mmfree_cuda_serve_step(self._h, in_ids.ctypes.data, out.ctypes.data))
        return out

    def serve_step_ptr(self, in_ptr: int, out_ptr: int) -> None:
        """serve_step on raw host pointers (pinned buffers)."""
        check(lib().mmfree_cuda_serve_step(self._h, in_ptr, out_ptr))

    def serve_run(self, steps: int) -> np.ndarray:
        out = np.empty((self._serve_b, steps), np.int64)
        check(lib().mmfree_cuda_serve_run(self._h, steps, out.ctypes.data))
        return out

    def serve_end(self) -> None:
        check(lib().mmfree_cuda_serve_end(self._h))

    @property
    def stream_ptr(self) -> int:
        """cudaStream_t of every kernel this model launches (for CUDA-event timing)."""
        return lib().mmfree_cuda_model_stream(self._h)

    def serve_profile(self, steps: int) -> dict:
        """Per kernel class: {name: dict(ms, launches, bytes, ops)} over ``steps`` steps."""
        from ._lib import KernelStats
        buf = (KernelStats * 16)()
        n = C.c_int()
        check(lib().mmfree_cuda_serve_profile(self._h, steps, buf, 16, C.byref(n)))
        return {buf[i].name.decode(): dict(ms=buf[i].ms, launches=buf[i].launches,
                                           bytes=buf[i].bytes, ops=buf[i].ops)
                for i in range(n.value)}


# ---- kernels on CUDA tensors -----------------------------------------------------------------

def packed_bytes(out_dim: int, in_dim: int) -> int:
    return lib().mmfree_cuda_packed_bytes(out_dim, in_dim)


def pack_ternary_host(wq: np.ndarray) -> np.ndarray:
    """int8 [out, in] -> packed uint8 bytes (host)."""
    wq = np.ascontiguousarray(wq, np.int8)
    out = np.empty(packed_bytes(*wq.shape), np.uint8)
    check(lib().mmfree_cuda_pack_ternary_host(out.ctypes.data, wq.ctypes.data, *wq.shape))
    return out


def repack_ternary(wq, stream=None):
    """int8 CUDA tensor [out, in] -> packed uint8 CUDA tensor."""
    import torch
    out = torch.empty(packed_bytes(*wq.shape), dtype=torch.uint8, device=wq.device)
    check(lib().mmfree_cuda_repack_ternary(out.data_ptr(), wq.contiguous().data_ptr(),
                                           wq.shape[0], wq.shape[1], _stream(stream)))
    return out


def bitlinear(x, norm_weight, wpacked, scale_w: float, out_dim: int, eps: float = 1e-6,
              act_quant="fixed", frac_bits: int = 10, want_norm: bool = False,
              want_acc: bool = False, stream=None):
    """mmfree::bitlinear on CUDA tensors; returns (out, acc or None, norm or None)."""
    import torch
    rows, in_dim = x.shape
    out = torch.empty(rows, out_dim, dtype=torch.float32, device=x.device)
    norm = torch.empty_like(x) if want_norm else None
    acc = torch.empty(rows, out_dim, dtype=torch.int32, device=x.device) if want_acc else None
    check(lib().mmfree_cuda_bitlinear(out.data_ptr(), x.data_ptr(), norm_weight.data_ptr(),
                                      wpacked.data_ptr(), scale_w, rows, in_dim, out_dim, eps,
                                      _ptr(norm), _aq(act_quant), frac_bits, _ptr(acc),
                                      _stream(stream)))
    return out, acc, norm


def nccl_unique_id() -> bytes:
    """128 bytes that identify a new NCCL communicator (rank 0 makes it, every rank uses it)."""
    buf = (C.c_ubyte * 128)()
    check(lib().mmfree_cuda_nccl_unique_id(buf))
    return bytes(buf)


def kernel_status(stream=None) -> None:
    """Synchronizes ``stream`` and raises MmfreeError (code E_TIMEOUT) when a kernel of an
    asynchronous entry point (bitlinear, bitlinear_cluster, bitlinear_noalloc) gave up a
    bounded wait since the last check; the recorded error is cleared."""
    check(lib().mmfree_cuda_kernel_status(_stream(stream)))


def set_wait_limit(polls: int) -> None:
    """Diagnostic: polls of the BitLinear prologue's row wait before it gives up (negative =
    default); 0 makes the staged waits give up at once."""
    lib().mmfree_cuda_set_wait_limit(int(polls))


def bitlinear_cluster(x, norm_weights, wpacked, scale_w, out_dim: int, eps: float = 1e-6,
                      frac_bits: int = 10, want_acc: bool = False, stream=None):
    import torch
    rows, in_dim = x.shape
    k = len(norm_weights)
    outs = [torch.empty(rows, out_dim, dtype=torch.float32, device=x.device) for _ in range(k)]
    acc = torch.empty(k, rows, out_dim, dtype=torch.int32, device=x.device) if want_acc else None
    o = (C.c_void_p * k)(*[t.data_ptr() for t in outs])
    n = (C.c_void_p * k)(*[t.data_ptr() for t in norm_weights])
    w = (C.c_void_p * k)(*[t.data_ptr() for t in wpacked])
    s = (C.c_float * k)(*[float(v) for v in scale_w])
    check(lib().mmfree_cuda_bitlinear_cluster(o, x.data_ptr(), n, w, s, k, rows, in_dim, out_dim,
                                              eps, frac_bits, _ptr(acc), _stream(stream)))
    return outs, acc


def ternary_matmul(x_codes, wpacked, out_dim: int, stream=None):
    """TernaryBackend::matmul_batch: int32 codes [b, N] -> int32 acc [b, M]."""
    import torch
    b, n = x_codes.shape
    acc = torch.empty(b, out_dim, dtype=torch.int32, device=x_codes.device)
    check(lib().mmfree_cuda_ternary_matmul(acc.data_ptr(), x_codes.data_ptr(), wpacked.data_ptr(),
                                           n, out_dim, b, _stream(stream)))
    return acc


def rmsnorm(x, weight, eps: float = 1e-6, stream=None):
    import torch
    y = torch.empty_like(x)
    check(lib().mmfree_cuda_rmsnorm(y.data_ptr(), x.data_ptr(), weight.data_ptr(), x.shape[0],
                                    x.shape[1], eps, _stream(stream)))
    return y


def swiglu(a, b, stream=None):
    import torch
    out = torch.empty_like(a)
    check(lib().mmfree_cuda_swiglu(out.data_ptr(), a.data_ptr(), b.data_ptr(), a.numel(),
                                   _stream(stream)))
    return out


def hgrn_scan(i, f, state=None, stream=None):
    """mmfree::hgrn_scan; ``state`` (CUDA tensor [D]) is updated in place when given."""
    import torch
    out = torch.empty_like(i)
    T, D = i.shape
    check(lib().mmfree_cuda_hgrn_scan(out.data_ptr(), i.data_ptr(), f.data_ptr(), T, D,
                                      _ptr(state), _stream(stream)))
    return out


def rmsnorm_swishgate(g, o, weight, eps: float = 1e-6, stream=None):
    import torch
    out = torch.empty_like(g)
    check(lib().mmfree_cuda_rmsnorm_swishgate(out.data_ptr(), g.data_ptr(), o.data_ptr(),
                                              weight.data_ptr(), g.shape[0], g.shape[1], eps,
                                              _stream(stream)))
    return out
