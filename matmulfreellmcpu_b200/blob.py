"""Seeded random-init ``model.mmfree`` writer and a reader for the same format.

The blob format is the reference engine's (matmulfreellmCPU ``tools/provision.py:126-163``,
parsed by ``cpp/src/io/weights.cpp:191-254``):

    [8]  magic ``b"MMFREE1\\n"``
    [8]  little-endian u64 header length
    [hl] JSON ``{"config": {...}, "tensors": {name: {dtype, shape, offset, nbytes}}}``
    zero padding to a 64-byte boundary, then the data section; every tensor starts on a
    64-byte boundary and ``offset`` is relative to the data-section start.

Tensor names follow ``tools/provision.py:101-124``: ``model.embeddings`` f32 [V,H],
``model.norm.w`` f32 [H], ``lm_head.{wq,scale_w,normw}``, ``lower_bounds`` f32 [L,H], and per
layer ``model.layers.{l}.{attn_norm,mlp_norm,g_norm}.w`` plus
``model.layers.{l}.{i,f,g,o,gate,down}_proj.{wq,scale_w,normw}`` (``wq`` int8 [out,in]).

Random init (there is no checkpoint): ``numpy.random.default_rng(seed)`` draws float32
``standard_normal * std`` latent weights in the order embeddings, lm_head, then per layer
i, f, g, o, gate, down. Each latent matrix W is ternarised per tensor as in
``tools/reference.py:138-142``: ``scale_w = 1 / max(mean|W|, 1e-5)`` and
``wq = clip(round_half_even(W * scale_w), -1, 1)``. Norm weights are 1. ``lower_bounds`` is
the packer's transform (``provision.py:108-111``) of an all-zero raw parameter: softmax over
layers, cumulative sum, minus the first entry, i.e. ``lb[l] = l / L``.
"""
from __future__ import annotations

import json
import os
import struct
from dataclasses import dataclass, field

import numpy as np

MAGIC = b"MMFREE1\n"
MAGIC2 = b"MMFREE2\n"  # the load cache: ternary weights as dtype "t2" (tiled 2-bit)
ALIGN = 64
PROJS = ("i_proj", "f_proj", "g_proj", "o_proj", "gate_proj", "down_proj")

#: Model shapes named by the benchmark configurations (vocab, hidden, layers, intermediate).
CONFIGS = {
    "370M": dict(vocab_size=32000, hidden_size=1024, num_hidden_layers=24, intermediate_size=2816),
    "1.3B": dict(vocab_size=32000, hidden_size=2048, num_hidden_layers=24, intermediate_size=5632),
    "2.7B": dict(vocab_size=32000, hidden_size=2560, num_hidden_layers=32, intermediate_size=6912),
    # small shapes for parity tests; "ragged" has dims that are not multiples of 8
    "tiny": dict(vocab_size=512, hidden_size=64, num_hidden_layers=2, intermediate_size=96),
    "small": dict(vocab_size=2048, hidden_size=256, num_hidden_layers=4, intermediate_size=704),
    "ragged": dict(vocab_size=300, hidden_size=36, num_hidden_layers=2, intermediate_size=52),
    # the 1.3B intermediate size on a narrow, one-layer model: at 64 decode rows its gate_proj
    # (SwiGLU pair epilogue), i/f/g, o and down run split-K over 2- and 8-CTA clusters
    "wide": dict(vocab_size=512, hidden_size=768, num_hidden_layers=1, intermediate_size=5632),
}


def _align(n: int) -> int:
    return (n + ALIGN - 1) // ALIGN * ALIGN


def ternarize(w: np.ndarray) -> tuple[np.ndarray, np.float32]:
    """Per-tensor ternary quantisation (``tools/reference.py:138-142``)."""
    mean = np.float32(np.abs(w).mean(dtype=np.float64))
    scale = np.float32(1.0) / max(mean, np.float32(1e-5))
    wq = np.clip(np.rint(w * scale), -1, 1).astype(np.int8)
    return wq, np.float32(scale)


def lower_bounds(layers: int, hidden: int) -> np.ndarray:
    """``provision.py:108-111`` applied to a zero raw parameter, in float32."""
    raw = np.zeros((layers, hidden), np.float32)
    e = np.exp(raw - raw.max(axis=0, keepdims=True))
    sm = (e / e.sum(axis=0, keepdims=True)).astype(np.float32)
    cs = np.cumsum(sm, axis=0, dtype=np.float32)
    return (cs - sm[0]).astype(np.float32)


def tensor_specs(cfg: dict) -> list[tuple[str, str, tuple[int, ...]]]:
    """(name, dtype, shape) of every tensor, in file order."""
    V, H, L, I = (cfg["vocab_size"], cfg["hidden_size"], cfg["num_hidden_layers"],
                  cfg["intermediate_size"])
    specs = [("model.embeddings", "f32", (V, H)), ("model.norm.w", "f32", (H,)),
             ("lm_head.wq", "i8", (V, H)), ("lm_head.scale_w", "f32", (1,)),
             ("lm_head.normw", "f32", (H,)), ("lower_bounds", "f32", (L, H))]
    dims = {"i_proj": (H, H), "f_proj": (H, H), "g_proj": (H, H), "o_proj": (H, H),
            "gate_proj": (2 * I, H), "down_proj": (H, I)}
    for l in range(L):
        p = f"model.layers.{l}"
        specs += [(f"{p}.attn_norm.w", "f32", (H,)), (f"{p}.mlp_norm.w", "f32", (H,)),
                  (f"{p}.g_norm.w", "f32", (H,))]
        for tag in PROJS:
            n_out, n_in = dims[tag]
            specs += [(f"{p}.{tag}.wq", "i8", (n_out, n_in)), (f"{p}.{tag}.scale_w", "f32", (1,)),
                      (f"{p}.{tag}.normw", "f32", (n_in,))]
    return specs


def write_random_blob(path: str, vocab_size: int, hidden_size: int, num_hidden_layers: int,
                      intermediate_size: int, seed: int = 0, std: float = 0.02,
                      rms_norm_eps: float = 1e-6) -> str:
    """Write a seeded random-init HGRN-Bit blob to ``path``; returns ``path``."""
    cfg = dict(vocab_size=vocab_size, hidden_size=hidden_size,
               num_hidden_layers=num_hidden_layers, intermediate_size=intermediate_size)
    specs = tensor_specs(cfg)
    meta, off = {}, 0
    for name, dt, shape in specs:
        nbytes = int(np.prod(shape)) * (1 if dt == "i8" else 4)
        meta[name] = {"dtype": dt, "shape": list(shape), "offset": off, "nbytes": nbytes}
        off = _align(off + nbytes)
    data_len = off
    header = {"config": {**cfg, "num_heads": 1, "expand_ratio": 1, "use_lower_bound": True,
                         "use_short_conv": False, "rms_norm_eps": rms_norm_eps},
              "tensors": meta}
    hb = json.dumps(header).encode()
    data_start = _align(len(MAGIC) + 8 + len(hb))

    rng = np.random.default_rng(seed)
    f32 = np.float32(std)

    def latent(shape):
        return rng.standard_normal(shape, dtype=np.float32) * f32

    H, L = hidden_size, num_hidden_layers
    tmp = path + ".tmp"
    os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
    with open(tmp, "wb") as f:
        f.write(MAGIC)
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)

        def put(name, arr):
            pos = data_start + meta[name]["offset"]
            f.write(b"\0" * (pos - f.tell()))
            assert arr.nbytes == meta[name]["nbytes"], name
            f.write(np.ascontiguousarray(arr).tobytes())

        ones_h = np.ones(H, np.float32)
        put("model.embeddings", latent((vocab_size, H)))
        put("model.norm.w", ones_h)
        wq, s = ternarize(latent((vocab_size, H)))
        put("lm_head.wq", wq)
        put("lm_head.scale_w", np.array([s], np.float32))
        put("lm_head.normw", ones_h)
        put("lower_bounds", lower_bounds(L, H))
        for l in range(L):
            p = f"model.layers.{l}"
            for nm in ("attn_norm", "mlp_norm", "g_norm"):
                put(f"{p}.{nm}.w", ones_h)
            for tag in PROJS:
                n_out, n_in = meta[f"{p}.{tag}.wq"]["shape"]
                wq, s = ternarize(latent((n_out, n_in)))
                put(f"{p}.{tag}.wq", wq)
                put(f"{p}.{tag}.scale_w", np.array([s], np.float32))
                put(f"{p}.{tag}.normw", np.ones(n_in, np.float32))
        f.write(b"\0" * (data_start + data_len - f.tell()))
    os.replace(tmp, path)
    return path


def write_config_blob(path: str, name: str, seed: int = 0) -> str:
    """Write the named configuration (``CONFIGS``) with the given seed."""
    return write_random_blob(path, seed=seed, **CONFIGS[name])


def cached_blob(name: str, seed: int = 0, cache_dir: str | None = None) -> str:
    """Path of a seeded blob for ``name``, written once into ``cache_dir``."""
    cache_dir = cache_dir or os.environ.get("MMFREE_BLOB_CACHE", "/tmp/mmfree_blobs")
    path = os.path.join(cache_dir, f"{name}_seed{seed}.mmfree")
    if not os.path.exists(path):
        write_config_blob(path, name, seed)
    return path


def packed_nbytes(out: int, k: int) -> int:
    """Bytes of the tiled 2-bit format of an [out, k] ternary matrix."""
    return -(-out // 32) * -(-k // 64) * 512


def pack_ternary(wq: np.ndarray) -> np.ndarray:
    """int8 ternary [out, k] -> the engine's tiled 2-bit format (csrc/common.cuh): 32-row
    groups x 64-column chunks of 512 bytes, row r of a group at bytes 16r..16r+15, 32-bit
    word w holding the codes u = w + 1 of columns 16w + 4g + j at bit 8j + 2g; padding rows
    and columns hold u = 1 (weight 0). Entries outside {-1, 0, 1} are rejected."""
    wq = np.asarray(wq)
    if wq.ndim != 2 or ((wq < -1) | (wq > 1)).any():
        raise ValueError("pack_ternary: expected a 2-D array of -1/0/+1")
    out, k = wq.shape
    ng, kc = -(-out // 32), -(-k // 64)
    u = np.ones((ng * 32, kc * 64), np.uint8)
    u[:out, :k] = (wq.astype(np.int16) + 1).astype(np.uint8)
    u6 = u.reshape(ng, 32, kc, 4, 4, 4)  # [group, row, chunk, word, g, j]
    b = u6[:, :, :, :, 0, :] | (u6[:, :, :, :, 1, :] << 2) | (u6[:, :, :, :, 2, :] << 4) | \
        (u6[:, :, :, :, 3, :] << 6)      # [group, row, chunk, word, byte j]
    return np.ascontiguousarray(b.transpose(0, 2, 1, 3, 4)).reshape(-1)


def write_packed_blob(src: str, dst: str) -> str:
    """model.mmfree -> model.mmfree2: the same header and tensors, every ternary *.wq
    stored packed (dtype "t2", shape kept as [out, in]); returns ``dst``."""
    with open(src, "rb") as f:
        if f.read(8) != MAGIC:
            raise ValueError(f"bad magic in {src}")
        (hl,) = struct.unpack("<Q", f.read(8))
        header = json.loads(f.read(hl))
    data_start = _align(16 + hl)
    mm = np.memmap(src, dtype=np.uint8, mode="r")
    meta, off, parts = {}, 0, []
    for name, m in header["tensors"].items():
        raw = mm[data_start + m["offset"]:data_start + m["offset"] + m["nbytes"]]
        if m["dtype"] == "i8" and name.endswith(".wq"):
            body = pack_ternary(raw.view(np.int8).reshape(m["shape"]))
            meta[name] = {"dtype": "t2", "shape": m["shape"], "offset": off, "nbytes": body.size}
        else:
            body = raw
            meta[name] = dict(m, offset=off)
        parts.append((off, body))
        off = _align(off + body.size)
    hb = json.dumps({"config": header["config"], "tensors": meta}).encode()
    start = _align(len(MAGIC2) + 8 + len(hb))
    tmp = dst + ".tmp"
    with open(tmp, "wb") as f:
        f.write(MAGIC2)
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for o, body in parts:
            f.write(b"\0" * (start + o - f.tell()))
            f.write(np.ascontiguousarray(body).tobytes())
    os.replace(tmp, dst)
    return dst


@dataclass
class Blob:
    """Read-only view of a ``model.mmfree`` file (numpy memmap, zero copy)."""
    path: str
    config: dict = field(default_factory=dict)
    tensors: dict = field(default_factory=dict)

    @classmethod
    def open(cls, path: str) -> "Blob":
        with open(path, "rb") as f:
            magic = f.read(8)
            if magic not in (MAGIC, MAGIC2):
                raise ValueError(f"bad magic in {path}")
            (hl,) = struct.unpack("<Q", f.read(8))
            header = json.loads(f.read(hl))
        data_start = _align(16 + hl)
        mm = np.memmap(path, dtype=np.uint8, mode="r")
        tensors = {}
        for name, m in header["tensors"].items():
            start = data_start + m["offset"]
            if m["dtype"] == "t2":  # packed ternary (model.mmfree2): the raw tiled bytes
                tensors[name] = mm[start:start + packed_nbytes(*m["shape"])]
                continue
            dt = np.int8 if m["dtype"] == "i8" else np.float32
            n = int(np.prod(m["shape"]))
            tensors[name] = mm[start:start + n * dt().itemsize].view(dt).reshape(m["shape"])
        return cls(path, header["config"], tensors)

    def __getitem__(self, name: str) -> np.ndarray:
        return self.tensors[name]


def seeded_ids(n: int, seed: int, vocab: int = 32000, low: int = 3) -> np.ndarray:
    """Prompt ids: uniform integers in [low, vocab) from ``default_rng(seed)``."""
    return np.random.default_rng(seed).integers(low, vocab, size=n, dtype=np.int64)


def main(argv=None) -> int:
    """python -m matmulfreellmcpu_b200.blob pack SRC.mmfree DST.mmfree2"""
    import sys
    args = sys.argv[1:] if argv is None else argv
    if len(args) != 3 or args[0] != "pack":
        print(main.__doc__, file=sys.stderr)
        return 2
    write_packed_blob(args[1], args[2])
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
