"""Python binding of ``libcuda_inference.so`` (include/cuda_inference.h).

The surface mirrors the reference's GPU engine, ``metal_infrence_engine/src/metal_inference.rs``:
``CudaModel.load_model(path)`` (metal_inference.rs:157), ``model.config`` (:170),
``model.forward(token, pos, cache) -> logits`` (:286), ``model.decode(first, start_pos, steps,
cache, on_token)`` (:297) and ``CudaKVCache(model, max_seq)`` (:129, ``max_seq`` :121), so tests
and benchmarks read like the reference's ``tests/metal_parity.rs`` and ``src/bin/bench.rs``.

There is no fallback: if the shared library is missing or a call fails, an exception is raised.
Where the reference panics (missing tensor, non-BF16 weights, ``pos >= max_seq``), the C ABI
returns a status code and this module raises ``QwError``.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from pathlib import Path
from typing import Callable

import numpy as np

_HERE = Path(__file__).resolve().parent
LIB_PATH = _HERE / "libcuda_inference.so"
HEADER = _HERE.parent / "include" / "cuda_inference.h"

QW_OK, QW_ERR_IO, QW_ERR_FORMAT, QW_ERR_UNSUPPORTED, QW_ERR_ARG, QW_ERR_CUDA, QW_ERR_DEVICE_TIMEOUT, QW_ERR_NOMEM = range(8)
_ERR_NAMES = ["OK", "IO", "FORMAT", "UNSUPPORTED", "ARG", "CUDA", "DEVICE_TIMEOUT", "NOMEM"]


class QwError(RuntimeError):
    def __init__(self, code: int, msg: str):
        self.code = code
        name = _ERR_NAMES[code] if 0 <= code < len(_ERR_NAMES) else str(code)
        super().__init__(f"QW_ERR_{name}: {msg}")


class _Config(ctypes.Structure):
    _fields_ = [("hidden_size", ctypes.c_uint64), ("intermediate_size", ctypes.c_uint64),
                ("num_hidden_layers", ctypes.c_uint64), ("num_attention_heads", ctypes.c_uint64),
                ("num_key_value_heads", ctypes.c_uint64), ("head_dim", ctypes.c_uint64),
                ("vocab_size", ctypes.c_uint64), ("rms_norm_eps", ctypes.c_float),
                ("rope_theta", ctypes.c_float), ("eos_token_id", ctypes.c_uint32)]


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

    @classmethod
    def _from(cls, c: _Config) -> "Config":
        return cls(*(int(getattr(c, f)) for f, _ in _Config._fields_[:7]), float(c.rms_norm_eps),
                   float(c.rope_theta), int(c.eos_token_id))


TOKEN_FN = ctypes.CFUNCTYPE(None, ctypes.c_void_p, ctypes.c_uint32)
LOOKUP_DRAFT_MAX = 15


class _LookupStats(ctypes.Structure):
    _fields_ = [("passes", ctypes.c_uint64), ("drafted", ctypes.c_uint64), ("accepted", ctypes.c_uint64)]
_lib = None


def lib() -> ctypes.CDLL:
    """Load libcuda_inference.so (raises if it was not built: there is no fallback path)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(f"{LIB_PATH} is missing; build it with `python {_HERE / 'build.py'}`")
        L = ctypes.CDLL(str(LIB_PATH))
        vp, sz, i32, u32, u64 = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_uint32, ctypes.c_uint64
        sig = {
            "qw_last_error": (ctypes.c_char_p, []),
            "qw_inspect": (i32, [ctypes.c_char_p, ctypes.POINTER(_Config)]),
            "qw_load": (i32, [ctypes.c_char_p, i32, ctypes.POINTER(vp)]),
            "qw_free": (None, [vp]),
            "qw_config_get": (i32, [vp, ctypes.POINTER(_Config)]),
            "qw_weight_bytes_per_token": (u64, [vp]),
            "qw_cache_new": (i32, [vp, sz, ctypes.POINTER(vp)]),
            "qw_cache_free": (None, [vp]),
            "qw_cache_max_seq": (sz, [vp]),
            "qw_forward": (i32, [vp, vp, u32, sz, vp]),
            "qw_prefill": (i32, [vp, vp, vp, sz, sz, vp]),
            "qw_prefill_device": (i32, [vp, vp, vp, sz, sz, vp, vp]),
            "qw_decode": (i32, [vp, vp, u32, sz, sz, TOKEN_FN, vp]),
            "qw_forward_batch": (i32, [vp, vp, sz, vp, vp, vp]),
            "qw_decode_lookup": (i32, [vp, vp, vp, sz, u32, sz, sz, u32, u32, vp, ctypes.POINTER(_LookupStats)]),
            "qw_decode_batch": (i32, [vp, vp, sz, vp, vp, sz, vp]),
            "qw_decode_batch_device": (i32, [vp, vp, sz, vp, vp, sz, vp, vp]),
            "qw_forward_device": (i32, [vp, vp, vp, sz, vp, vp]),
            "qw_decode_device": (i32, [vp, vp, vp, sz, sz, vp]),
            "qw_sync": (i32, [vp, vp]),
            "qw_cache_read": (i32, [vp, sz, sz, vp, vp]),
            "qw_num_ctas": (i32, [vp]),
            "qw_decoder_kind": (i32, [vp]),
            "qw_batch_decoder_kind": (i32, [vp]),
            "qw_model_stream": (vp, [vp]),
            "qw_trace_stride": (sz, [vp]),
            "qw_set_trace": (i32, [vp, i32]),
            "qw_read_trace": (i32, [vp, ctypes.POINTER(ctypes.c_uint64), sz]),
            "qw_gemv_bf16": (i32, [i32, vp, vp, vp, sz, sz, vp]),
            "qw_gemv_bf16_seq": (i32, [i32, vp, vp, vp, sz, sz, sz, vp]),
            "qw_argmax_workspace_size": (sz, [sz]),
            "qw_argmax_f32": (i32, [i32, vp, sz, vp, vp, vp]),
            "qw_argmax_f32_noalloc": (i32, [i32, vp, sz, vp, vp]),
            "qw_read_probe": (i32, [i32, vp, sz, vp, sz, ctypes.POINTER(sz), vp]),
            "qw_gemm_bf16x2": (i32, [i32, vp, vp, vp, vp, sz, sz, sz, vp]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _check(rc: int) -> None:
    if rc != QW_OK:
        raise QwError(rc, lib().qw_last_error().decode(errors="replace"))


def inspect(path: str | Path) -> Config:
    """Parse and validate a checkpoint directory's safetensors + config.json (no GPU needed)."""
    c = _Config()
    _check(lib().qw_inspect(str(path).encode(), ctypes.byref(c)))
    return Config._from(c)


class CudaModel:
    """metal_inference.rs:100-113 MetalModel — weights on one B200, one stream."""

    def __init__(self, handle: ctypes.c_void_p, device: int):
        self._h = handle
        self.device = device
        c = _Config()
        _check(lib().qw_config_get(handle, ctypes.byref(c)))
        self.config = Config._from(c)

    @classmethod
    def load_model(cls, path: str | Path, device: int = 0) -> "CudaModel":
        h = ctypes.c_void_p()
        _check(lib().qw_load(str(path).encode(), device, ctypes.byref(h)))
        return cls(h, device)

    def weight_bytes_per_token(self) -> int:
        """tests/mbu.rs:19-30"""
        return int(lib().qw_weight_bytes_per_token(self._h))

    @property
    def num_ctas(self) -> int:
        return int(lib().qw_num_ctas(self._h))

    @property
    def decoder_kind(self) -> str:
        """'grid' (one CTA per SM, the default) or 'cluster' (8 clusters of 8 CTAs, QW_DECODER=cluster)."""
        return {0: "grid", 1: "cluster"}.get(int(lib().qw_decoder_kind(self._h)), "?")

    @property
    def batch_decoder_kind(self) -> str:
        """'rows' (captured row-mode step graphs, the default) or 'persistent' (one persistent launch
        for batches of at most 8 rows: QW_BATCH_DECODER=persistent at load, where the shapes fit)."""
        return {0: "rows", 1: "persistent"}.get(int(lib().qw_batch_decoder_kind(self._h)), "?")

    @property
    def stream(self) -> int:
        """The model's cudaStream_t handle (forward/decode run on it)."""
        return int(lib().qw_model_stream(self._h) or 0)

    def set_trace(self, enable: bool) -> None:
        """Record a per-CTA phase timeline of each launch's first step (see include/cuda_inference.h)."""
        _check(lib().qw_set_trace(self._h, 1 if enable else 0))

    def read_trace(self) -> np.ndarray:
        """[num_ctas, stride] uint64 globaltimer stamps (ns) of the most recent launch's first step."""
        stride = int(lib().qw_trace_stride(self._h))
        out = np.zeros((self.num_ctas, stride), np.uint64)
        _check(lib().qw_read_trace(self._h, out.ctypes.data_as(ctypes.POINTER(ctypes.c_uint64)), out.size))
        return out

    def forward(self, token: int, pos: int, cache: "CudaKVCache") -> np.ndarray:
        out = np.empty(self.config.vocab_size, np.float32)
        _check(lib().qw_forward(self._h, cache._h, token, pos, out.ctypes.data))
        return out

    def prefill(self, ids, start_pos: int, cache: "CudaKVCache", logits: bool = True,
                out: np.ndarray | None = None) -> np.ndarray | None:
        """One batched pass over the prompt ids at positions start_pos.. (qw_prefill): fills the KV
        cache like len(ids) forward calls; returns the [len(ids), vocab] logits when asked.

        `out`, if given, is a C-contiguous float32 [len(ids), vocab] array that receives the logits
        (and is returned) instead of a new array. A caller that decodes many prompts can keep one,
        for instance the numpy view of a page-locked torch tensor, which the copy then reaches by
        one DMA; a new or pageable array goes through the library's pinned stages."""
        a = np.ascontiguousarray(np.asarray(ids, dtype=np.uint32))
        if out is not None:
            if not logits:
                raise ValueError("out given with logits=False")
            if (out.dtype != np.float32 or out.shape != (a.size, self.config.vocab_size)
                    or not out.flags.c_contiguous or not out.flags.writeable):
                raise ValueError(f"out must be a writeable C-contiguous float32 array of shape "
                                 f"({a.size}, {self.config.vocab_size})")
        elif logits:
            out = np.empty((a.size, self.config.vocab_size), np.float32)
        _check(lib().qw_prefill(self._h, cache._h, a.ctypes.data, a.size, start_pos,
                                out.ctypes.data if out is not None else None))
        return out

    def prefill_device(self, cache: "CudaKVCache", d_ids: int, n: int, start_pos: int, d_logits: int = 0,
                       stream: int = 0) -> None:
        _check(lib().qw_prefill_device(self._h, cache._h, d_ids, n, start_pos, d_logits or None, stream or None))

    def decode(self, first: int, start_pos: int, steps: int, cache: "CudaKVCache",
               on_token: Callable[[int], None] | None = None) -> list[int]:
        """Greedy decode; on_token(t) is called as each token arrives. Returns the tokens too."""
        got: list[int] = []

        def cb(_user, tok):
            got.append(int(tok))
            if on_token is not None:
                on_token(int(tok))

        fn = TOKEN_FN(cb)
        _check(lib().qw_decode(self._h, cache._h, first, start_pos, steps, fn, None))
        return got

    def decode_lookup(self, context, first: int, start_pos: int, steps: int, cache: "CudaKVCache",
                      max_ngram: int = 3, draft_max: int = 7) -> tuple[list[int], dict]:
        """Prompt-lookup speculative greedy decode (qw_decode_lookup): the tokens decode() would give,
        with drafts looked up in `context` + the output so far; returns (tokens, stats)."""
        ctx = np.ascontiguousarray(np.asarray(context, dtype=np.uint32))
        out = np.empty(steps, np.uint32)
        st = _LookupStats()
        _check(lib().qw_decode_lookup(self._h, cache._h, ctx.ctypes.data if ctx.size else None, ctx.size, first,
                                      start_pos, steps, max_ngram, draft_max, out.ctypes.data, ctypes.byref(st)))
        return [int(t) for t in out], {"passes": st.passes, "drafted": st.drafted, "accepted": st.accepted}

    # batch decode: B independent sequences, one cache each, stepping together (qw_*_batch)
    @staticmethod
    def _caches(caches) -> "ctypes.Array":
        return (ctypes.c_void_p * len(caches))(*[c._h for c in caches])

    def forward_batch(self, tokens, positions, caches) -> np.ndarray:
        """Row b feeds tokens[b] at positions[b] into caches[b]; returns [B, vocab] logits."""
        t = np.ascontiguousarray(np.asarray(tokens, dtype=np.uint32))
        p = np.ascontiguousarray(np.asarray(positions, dtype=np.uint64))
        out = np.empty((t.size, self.config.vocab_size), np.float32)
        _check(lib().qw_forward_batch(self._h, self._caches(caches), t.size, t.ctypes.data, p.ctypes.data,
                                      out.ctypes.data))
        return out

    def decode_batch(self, firsts, start_pos, steps: int, caches) -> np.ndarray:
        """decode() for every row at once; returns [B, steps] output tokens."""
        f = np.ascontiguousarray(np.asarray(firsts, dtype=np.uint32))
        p = np.ascontiguousarray(np.asarray(start_pos, dtype=np.uint64))
        out = np.empty((f.size, steps), np.uint32)
        _check(lib().qw_decode_batch(self._h, self._caches(caches), f.size, f.ctypes.data, p.ctypes.data, steps,
                                     out.ctypes.data))
        return out

    def decode_batch_device(self, d_firsts: int, start_pos, steps: int, caches, d_out: int, stream: int = 0) -> None:
        """Stream-ordered decode_batch: device first tokens, device record d_out[steps][B]."""
        p = np.ascontiguousarray(np.asarray(start_pos, dtype=np.uint64))
        _check(lib().qw_decode_batch_device(self._h, self._caches(caches), p.size, d_firsts, p.ctypes.data, steps,
                                            d_out, stream or None))

    # device-resident variants: raw device pointers (ints) and an optional cudaStream_t handle
    def forward_device(self, cache: "CudaKVCache", d_token: int, pos: int, d_logits: int, stream: int = 0) -> None:
        _check(lib().qw_forward_device(self._h, cache._h, d_token, pos, d_logits, stream or None))

    def decode_device(self, cache: "CudaKVCache", d_tokens: int, start_pos: int, steps: int, stream: int = 0) -> None:
        _check(lib().qw_decode_device(self._h, cache._h, d_tokens, start_pos, steps, stream or None))

    def sync(self, stream: int = 0) -> None:
        _check(lib().qw_sync(self._h, stream or None))

    def close(self) -> None:
        if getattr(self, "_h", None) and _lib is not None:
            _lib.qw_free(self._h)
            self._h = None

    def __del__(self):
        self.close()


class CudaKVCache:
    """metal_inference.rs:115-137 MetalKVCache — f32 K/V for max_seq positions + RoPE table."""

    def __init__(self, model: CudaModel, max_seq: int):
        self._model = model
        self._h = ctypes.c_void_p()
        _check(lib().qw_cache_new(model._h, max_seq, ctypes.byref(self._h)))
        self.max_seq = int(lib().qw_cache_max_seq(self._h))

    def layer(self, l: int, n: int) -> tuple[np.ndarray, np.ndarray]:
        """K, V of layer l for positions [0, n) in the reference layout [t][kv_heads*head_dim]."""
        c = self._model.config
        kvd = c.num_key_value_heads * c.head_dim
        k = np.empty((n, kvd), np.float32)
        v = np.empty((n, kvd), np.float32)
        _check(lib().qw_cache_read(self._h, l, n, k.ctypes.data, v.ctypes.data))
        return k, v

    def close(self) -> None:
        if getattr(self, "_h", None) and _lib is not None:
            _lib.qw_cache_free(self._h)
            self._h = None

    def __del__(self):
        self.close()


# ---- standalone kernels ----------------------------------------------------------------------
def gemv_bf16(device: int, d_w: int, d_x: int, d_y: int, rows: int, cols: int, stream: int = 0) -> None:
    _check(lib().qw_gemv_bf16(device, d_w, d_x, d_y, rows, cols, stream or None))


def gemv_bf16_seq(device: int, d_w: int, d_x: int, d_y: int, rows: int, cols: int, count: int, stream: int = 0) -> None:
    """y[m] = W[m] x for `count` back-to-back matrices in one launch (see qw_gemv_bf16_seq)."""
    _check(lib().qw_gemv_bf16_seq(device, d_w, d_x, d_y, rows, cols, count, stream or None))


def argmax_workspace_size(n: int) -> int:
    return int(lib().qw_argmax_workspace_size(n))


def argmax_f32(device: int, d_x: int, n: int, d_out: int, d_workspace: int, stream: int = 0) -> None:
    _check(lib().qw_argmax_f32(device, d_x, n, d_out, d_workspace, stream or None))


def argmax_f32_noalloc(device: int, d_x: int, n: int, d_out: int, stream: int = 0) -> None:
    """argmax_f32 without a caller workspace (see qw_argmax_f32_noalloc in the header)."""
    _check(lib().qw_argmax_f32_noalloc(device, d_x, n, d_out, stream or None))


def gemm_bf16x2(device: int, d_a_hi: int, d_a_lo: int, d_b: int, d_y: int, M: int, N: int, K: int,
                stream: int = 0) -> None:
    """d_y[M][N] = (a_hi + a_lo)[M][K] . b[N][K]^T on the tensor cores (see qw_gemm_bf16x2)."""
    _check(lib().qw_gemm_bf16x2(device, d_a_hi, d_a_lo, d_b, d_y, M, N, K, stream or None))


def read_probe(device: int, d_src: int, n_floats: int, d_partials: int, n_partials: int, stream: int = 0) -> int:
    n = ctypes.c_size_t()
    _check(lib().qw_read_probe(device, d_src, n_floats, d_partials, n_partials, ctypes.byref(n), stream or None))
    return int(n.value)


def declared_symbols() -> list[str]:
    """Every function the C header declares (what the ABI promises to export)."""
    import re
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(qw_[a-z0-9_]+)\s*\(", text)))
