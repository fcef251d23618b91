"""C-ABI boundary checks that need no GPU: the library loads, exports every symbol the header
declares, and qw_inspect validates checkpoints the way the reference loader's panics would
(cpu_inference.rs:58-96, metal_inference.rs:172-176, :244-248), but as status codes."""
from __future__ import annotations

import ctypes
import json
import shutil
import struct

import numpy as np
import pytest

import cuda_inference as ci


def test_library_exports_every_declared_symbol():
    L = ci.lib()
    syms = ci.declared_symbols()
    assert len(syms) >= 20
    for name in syms:
        assert hasattr(L, name), name
    # the dynamic symbol table carries exactly these extern "C" names (no C++ mangling)
    assert isinstance(ctypes.cast(getattr(L, "qw_decode"), ctypes.c_void_p).value, int)


def test_inspect_reads_config(tiny_model_path):
    c = ci.inspect(tiny_model_path)
    assert (c.hidden_size, c.intermediate_size, c.num_hidden_layers) == (256, 768, 2)
    assert (c.num_attention_heads, c.num_key_value_heads, c.head_dim, c.vocab_size) == (4, 2, 128, 1000)
    assert c.rope_theta == 1e6 and abs(c.rms_norm_eps - 1e-6) < 1e-12 and c.eos_token_id == 151645


def test_inspect_full_geometry(full_model_path):
    c = ci.inspect(full_model_path)
    assert (c.hidden_size, c.num_hidden_layers, c.vocab_size) == (1024, 28, 151936)


def _copy_model(src, dst):
    dst.mkdir(parents=True, exist_ok=True)
    shutil.copy(src, dst / "model.safetensors")
    shutil.copy(src.parent / "config.json", dst / "config.json")
    return dst / "model.safetensors"


def _rewrite_header(path, mutate):
    b = path.read_bytes()
    hl = struct.unpack("<Q", b[:8])[0]
    hdr = json.loads(b[8:8 + hl])
    mutate(hdr)
    h = json.dumps(hdr).encode()
    h += b" " * ((-len(h) - 8) % 16)
    path.write_bytes(struct.pack("<Q", len(h)) + h + b[8 + hl:])


def _code(path):
    with pytest.raises(ci.QwError) as e:
        ci.inspect(path)
    return e.value.code


def test_inspect_errors(tiny_model_path, tmp_path):
    assert _code(tmp_path / "nope.safetensors") == ci.QW_ERR_IO

    p = _copy_model(tiny_model_path, tmp_path / "trunc")
    p.write_bytes(p.read_bytes()[:-4096])                       # truncated data section
    assert _code(p) == ci.QW_ERR_FORMAT

    p = _copy_model(tiny_model_path, tmp_path / "badjson")
    b = bytearray(p.read_bytes())
    b[9] = ord("#")                                             # corrupt JSON header
    p.write_bytes(bytes(b))
    assert _code(p) == ci.QW_ERR_FORMAT

    p = _copy_model(tiny_model_path, tmp_path / "hdrlen")
    b = bytearray(p.read_bytes())
    b[:8] = struct.pack("<Q", 1 << 40)                          # header length past EOF
    p.write_bytes(bytes(b))
    assert _code(p) == ci.QW_ERR_FORMAT

    p = _copy_model(tiny_model_path, tmp_path / "dtype")       # reference: "only BF16 is supported"
    _rewrite_header(p, lambda h: h["model.norm.weight"].update(dtype="F16"))
    assert _code(p) == ci.QW_ERR_UNSUPPORTED

    p = _copy_model(tiny_model_path, tmp_path / "missing")     # reference: panic "missing tensor"
    _rewrite_header(p, lambda h: h.pop("model.layers.1.mlp.down_proj.weight"))
    assert _code(p) == ci.QW_ERR_FORMAT

    p = _copy_model(tiny_model_path, tmp_path / "shape")
    _rewrite_header(p, lambda h: h["model.layers.0.self_attn.q_norm.weight"].update(shape=[64]))
    assert _code(p) == ci.QW_ERR_FORMAT

    p = _copy_model(tiny_model_path, tmp_path / "cfg")
    cfg = json.loads((p.parent / "config.json").read_text())
    del cfg["rope_theta"]
    (p.parent / "config.json").write_text(json.dumps(cfg))
    assert _code(p) == ci.QW_ERR_FORMAT

    p = _copy_model(tiny_model_path, tmp_path / "hd")          # head_dim the kernels do not support
    cfg = json.loads((p.parent / "config.json").read_text())
    cfg.update(head_dim=64)
    (p.parent / "config.json").write_text(json.dumps(cfg))
    assert _code(p) in (ci.QW_ERR_FORMAT, ci.QW_ERR_UNSUPPORTED)


def test_load_without_gpu_fails_loudly(tiny_model_path):
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is present; covered by the GPU tests")
    with pytest.raises(ci.QwError) as e:
        ci.CudaModel.load_model(tiny_model_path)
    assert e.value.code == ci.QW_ERR_CUDA


def test_standalone_kernels_reject_bad_arguments():
    with pytest.raises(ci.QwError):
        ci.gemv_bf16(0, 0, 0, 0, 16, 1024)
    with pytest.raises(ci.QwError):
        ci.argmax_f32(0, 0, 10, 0, 0)
    assert ci.argmax_workspace_size(151936) >= 256


def test_inspect_rejects_widths_the_kernel_cannot_segment(tmp_path):
    # intermediate 1536 is a multiple of 256 but neither <= 1024 nor a whole number of 1024-column
    # segments: the GEMV segmentation cannot split it, so the loader must refuse it up front
    import randmodel
    d = tmp_path / "odd"
    d.mkdir()
    st = d / "model.safetensors"
    g = dict(randmodel.GEOMETRIES["tiny"], intermediate_size=1536, num_hidden_layers=1)
    rc = randmodel._lib().rm_write_model(str(st).encode(), g["hidden_size"], g["intermediate_size"],
                                         g["num_hidden_layers"], g["num_attention_heads"],
                                         g["num_key_value_heads"], g["head_dim"], g["vocab_size"], 0, 0)
    assert rc == 0
    cfg = randmodel.config_dict("tiny")
    cfg.update(intermediate_size=1536, num_hidden_layers=1)
    (d / "config.json").write_text(json.dumps(cfg))
    assert _code(st) == ci.QW_ERR_UNSUPPORTED
