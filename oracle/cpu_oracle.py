"""CPU ORACLE (test infrastructure only) — ctypes view of ``liboracle_cpu.so``.

``liboracle_cpu.so`` is ``oracle/cpu_inference.cpp``, a line-by-line C++ restatement of the
reference CPU engine ``metal_infrence_engine/src/cpu_inference.rs``. Only the tests,
``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg use it, as the checker; the CUDA
engine never calls it. Parity status: unpinned against the reference's own golden vectors (they
need the real Qwen3-0.6B checkpoint); cross-checked against transformers' Qwen3 on seeded random
weights (tests/golden/).

The Python surface mirrors the Rust one: ``Model.load_model(path)``, ``model.config``,
``model.forward(token, pos, cache) -> logits``, ``KVCache(config)`` and ``argmax``.
"""
from __future__ import annotations

import ctypes
import subprocess
from dataclasses import dataclass
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_LIB_PATH = _HERE / "liboracle_cpu.so"
_lib = None


def build(force: bool = False) -> Path:
    """Compile liboracle_cpu.so with the flags that keep Rust's f32 semantics (no FMA contraction)."""
    src = _HERE / "cpu_inference.cpp"
    if force or not _LIB_PATH.exists() or _LIB_PATH.stat().st_mtime < src.stat().st_mtime:
        subprocess.run(["g++", "-O2", "-std=c++17", "-ffp-contract=off", "-fno-fast-math", "-fPIC",
                        "-shared", "-pthread", str(src), "-o", str(_LIB_PATH)], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(str(_LIB_PATH))
        vp, sz = ctypes.c_void_p, ctypes.c_size_t
        L.oracle_last_error.restype = ctypes.c_char_p
        L.oracle_load.argtypes = [ctypes.c_char_p, ctypes.POINTER(vp)]
        L.oracle_load.restype = ctypes.c_int
        L.oracle_free.argtypes = [vp]
        L.oracle_config.argtypes = [vp, ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_float),
                                    ctypes.POINTER(ctypes.c_float), ctypes.POINTER(ctypes.c_uint32)]
        L.oracle_weight_bytes_per_token.argtypes = [vp]
        L.oracle_weight_bytes_per_token.restype = ctypes.c_uint64
        L.oracle_cache_new.argtypes = [vp]
        L.oracle_cache_new.restype = vp
        L.oracle_cache_free.argtypes = [vp]
        L.oracle_cache_len.argtypes = [vp, vp]
        L.oracle_cache_len.restype = sz
        L.oracle_cache_read.argtypes = [vp, sz, vp, vp]
        L.oracle_cache_read.restype = ctypes.c_int
        L.oracle_cache_fill.argtypes = [vp, vp, sz, ctypes.c_uint64]
        L.oracle_cache_fill.restype = ctypes.c_int
        L.oracle_forward.argtypes = [vp, vp, ctypes.c_uint32, sz, vp]
        L.oracle_forward.restype = ctypes.c_int
        L.oracle_forward_seq.argtypes = [vp, vp, vp, sz, sz, vp, sz, vp]
        L.oracle_forward_seq.restype = ctypes.c_int
        L.oracle_matvec.argtypes = [vp, vp, vp, sz, sz]
        L.oracle_matvec.restype = None
        L.oracle_argmax.argtypes = [vp, sz]
        L.oracle_argmax.restype = ctypes.c_uint32
        L.oracle_set_threads.argtypes = [ctypes.c_int]
        L.oracle_threads.restype = ctypes.c_int
        _lib = L
    return _lib


@dataclass
class Config:
    """cpu_inference.rs:21-33"""
    hidden_size: int
    intermediate_size: int
    num_hidden_layers: int
    num_attention_heads: int
    num_key_value_heads: int
    head_dim: int
    vocab_size: int
    rms_norm_eps: float
    rope_theta: float
    eos_token_id: int


class KVCache:
    """cpu_inference.rs:44-55 — per-layer f32 K/V history, [t][kv_heads*head_dim]."""

    def __init__(self, model: "Model"):
        self._model = model
        self._h = lib().oracle_cache_new(model._h)

    def __len__(self) -> int:
        return lib().oracle_cache_len(self._model._h, self._h)

    def layer(self, l: int) -> tuple[np.ndarray, np.ndarray]:
        c = self._model.config
        kv_dim = c.num_key_value_heads * c.head_dim
        n = len(self)
        k = np.empty((n, kv_dim), np.float32)
        v = np.empty((n, kv_dim), np.float32)
        if lib().oracle_cache_read(self._h, l, k.ctypes.data, v.ctypes.data) != 0:
            raise IndexError(lib().oracle_last_error().decode())
        return k, v

    def fill_synthetic(self, npos: int, seed: int = 0) -> None:
        lib().oracle_cache_fill(self._model._h, self._h, npos, seed)

    def __del__(self):
        if getattr(self, "_h", None) and _lib is not None:
            _lib.oracle_cache_free(self._h)
            self._h = None


class Model:
    """cpu_inference.rs:35-179 — load_model / forward."""

    def __init__(self, handle):
        self._h = handle
        f = (ctypes.c_uint64 * 7)()
        eps, theta, eos = ctypes.c_float(), ctypes.c_float(), ctypes.c_uint32()
        lib().oracle_config(handle, f, ctypes.byref(eps), ctypes.byref(theta), ctypes.byref(eos))
        self.config = Config(*[int(x) for x in f], eps.value, theta.value, int(eos.value))

    @classmethod
    def load_model(cls, path: str | Path) -> "Model":
        h = ctypes.c_void_p()
        if lib().oracle_load(str(path).encode(), ctypes.byref(h)) != 0:
            raise OSError(lib().oracle_last_error().decode())
        return cls(h)

    def weight_bytes_per_token(self) -> int:
        """tests/mbu.rs:19-30"""
        return int(lib().oracle_weight_bytes_per_token(self._h))

    def forward(self, token: int, pos: int, cache: KVCache) -> np.ndarray:
        out = np.empty(self.config.vocab_size, np.float32)
        if lib().oracle_forward(self._h, cache._h, token, pos, out.ctypes.data) != 0:
            raise RuntimeError(lib().oracle_last_error().decode())
        return out

    def forward_seq(self, tokens, start_pos: int, cache: KVCache, out_positions=None) -> np.ndarray:
        """``forward`` for consecutive tokens at positions start_pos.., computed layer by layer
        over all of them; the cache and the logits are bit-identical to calling ``forward`` once per
        token. Returns the logits of the positions in ``out_positions`` (indices into ``tokens``;
        default: every position) as [len(out_positions)][vocab]."""
        toks = np.ascontiguousarray(tokens, np.uint32)
        idx = np.arange(toks.size) if out_positions is None else np.asarray(out_positions)
        idx = np.ascontiguousarray(idx, np.uint64)
        out = np.empty((idx.size, self.config.vocab_size), np.float32)
        rc = lib().oracle_forward_seq(self._h, cache._h, toks.ctypes.data, toks.size, start_pos,
                                      idx.ctypes.data, idx.size, out.ctypes.data)
        if rc != 0:
            raise RuntimeError(lib().oracle_last_error().decode())
        return out

    def __del__(self):
        if getattr(self, "_h", None) and _lib is not None:
            _lib.oracle_free(self._h)
            self._h = None


def argmax(x: np.ndarray) -> int:
    """tests/common/mod.rs:17-22 — first strict maximum (a NaN at index 0 sticks)."""
    x = np.ascontiguousarray(x, np.float32)
    return int(lib().oracle_argmax(x.ctypes.data, x.size))


def top2_margin(x: np.ndarray) -> float:
    """Gap between the largest and second-largest logit (greedy-flip risk when below 1e-2)."""
    p = np.partition(np.asarray(x, np.float64), -2)[-2:]
    return float(p[1] - p[0])


def matvec(w_bf16: np.ndarray, x: np.ndarray) -> np.ndarray:
    """cpu_inference.rs:225-257: y = W x, W given as uint16 bf16 bit patterns [rows][cols]."""
    w = np.ascontiguousarray(w_bf16, np.uint16)
    xx = np.ascontiguousarray(x, np.float32)
    rows, cols = w.shape
    assert xx.size == cols
    out = np.empty(rows, np.float32)
    lib().oracle_matvec(w.ctypes.data, xx.ctypes.data, out.ctypes.data, rows, cols)
    return out


def set_threads(n: int) -> None:
    lib().oracle_set_threads(n)


def threads() -> int:
    return int(lib().oracle_threads())
