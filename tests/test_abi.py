"""The C-ABI library loads without a GPU and exports exactly what include/h3b.h declares.

Only argument-validation paths are called here (they return before touching CUDA).
"""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from h3_flash_b200 import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "h3b.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(h3b_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_hot_path():
    names = declared_functions()
    for expected in (
        "h3b_rmsnorm_modulate", "h3b_residual_gate_rmsnorm_modulate", "h3b_modulate", "h3b_gated_residual",
        "h3b_swiglu", "h3b_gelu_tanh", "h3b_qknorm_rope", "h3b_qknorm_rope_pack", "h3b_pack_qkv",
        "h3b_merge_heads", "h3b_attention", "h3b_attention_workspace_size", "h3b_last_error",
        "h3b_abi_version",
    ):
        assert expected in names


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in declared_functions():
        assert hasattr(lib, name), name
    assert set(declared_functions()) <= set(_lib.exported_symbols())


def test_abi_version():
    assert _lib.load().h3b_abi_version() == _lib.ABI_VERSION


def test_shape_errors_map_to_value_error_without_a_gpu():
    lib = _lib.load()
    code = lib.h3b_rmsnorm_modulate(None, None, None, None, None, None, -1, 8, 1, 8, 8, 8, 8,
                                    ctypes.c_float(1e-6), None)
    assert code == _lib.H3B_ERR_VALUE
    assert "negative shape" in lib.h3b_last_error().decode()
    with pytest.raises(ValueError, match="must divide Ulysses degree"):
        _lib.call("h3b_pack_qkv", None, None, None, None, 4, 6, 128, 4, 0, 0, 0, 0, 0, 0, None)
    with pytest.raises(ValueError, match="rotary dimension"):
        _lib.call("h3b_qknorm_rope", None, None, None, None, None, 1, 4, 2, 128, 7, 1e-6, None)


def test_unsupported_head_dim_is_a_runtime_error():
    with pytest.raises(RuntimeError, match="head_dim must be 128"):
        _lib.call("h3b_attention", None, None, None, None, *([1] * 4), 64, *([64] * 12), 1.0, None, 0, None)


def test_empty_inputs_are_noops():
    # rows == 0 returns before any launch
    _lib.call("h3b_swiglu", None, None, 0, 16, 32, 16, None)
    _lib.call("h3b_merge_heads", None, None, 2, 0, 128, None)
    _lib.call("h3b_attention", None, None, None, None, 1, 0, 5, 1, 128, *([128] * 12), 1.0, None, 0, None)


def test_attention_p2p_argument_errors_without_a_gpu():
    """Validation returns before any CUDA call; the pointers are never dereferenced."""

    fake = 1 << 20  # a 16-byte aligned address
    ptrs = (ctypes.c_void_p * 2)(fake, None)
    counts = (ctypes.c_int64 * 2)(4, 4)
    with pytest.raises(ValueError, match="merged buffer of rank 1"):
        _lib.call("h3b_attention_p2p", ptrs, counts, 2, 0, fake, 1, 128, 0.1, None, 0, None)
    with pytest.raises(ValueError, match="rank 2 outside"):
        _lib.call("h3b_attention_p2p", ptrs, counts, 2, 2, fake, 1, 128, 0.1, None, 0, None)
    with pytest.raises(ValueError, match="world size"):
        _lib.call("h3b_attention_p2p", ptrs, counts, 17, 0, fake, 1, 128, 0.1, None, 0, None)
    with pytest.raises(RuntimeError, match="head_dim must be 128"):
        _lib.call("h3b_attention_p2p", ptrs, counts, 2, 0, fake, 1, 64, 0.1, None, 0, None)


def test_launch_counter_counts_launches_only():
    """The library counts kernels at launch; calls rejected by validation launch nothing."""

    _lib.reset_launch_count()
    assert _lib.launch_count() == 0
    with pytest.raises(ValueError):
        _lib.call("h3b_pack_qkv", None, None, None, None, 4, 6, 128, 4, 0, 0, 0, 0, 0, 0, None)
    assert _lib.launch_count() == 0


def test_qkv_gemm_pack_argument_errors_without_a_gpu():
    """Shape and layout checks return before any CUDA call."""

    fake = 1 << 20
    args = dict(x=fake, rows=64, dim=256, stride=256, w=fake, b=None, wq=fake, wk=fake, cos=fake, sin=fake)

    def call(heads, head_dim, rot, world=1, dim=256):
        _lib.call("h3b_qkv_gemm_pack", fake, world, args["x"], args["rows"], dim, dim, args["w"], None,
                  args["wq"], args["wk"], args["cos"], args["sin"], heads, head_dim, rot, 1e-6, 1e-6, fake,
                  args["rows"] * rot * 8, None)

    with pytest.raises(ValueError, match="must divide Ulysses degree"):
        call(heads=4, head_dim=128, rot=96, world=3)
    with pytest.raises(RuntimeError, match="head_dim 128"):
        call(heads=4, head_dim=64, rot=96)
    with pytest.raises(RuntimeError, match="even head count"):
        call(heads=3, head_dim=128, rot=96)
    with pytest.raises(RuntimeError, match="rotary dimension"):
        call(heads=4, head_dim=128, rot=48)
    with pytest.raises(RuntimeError, match="dim % 64"):
        call(heads=4, head_dim=128, rot=96, dim=200)
    with pytest.raises(ValueError, match="workspace of 49152 bytes"):
        _lib.call("h3b_qkv_gemm_pack", fake, 1, fake, 64, 256, 256, fake, None, fake, fake, fake, fake, 4, 128, 96,
                  1e-6, 1e-6, fake, 64 * 96 * 8 - 16, None)
    need = ctypes.c_int64(-1)
    _lib.call("h3b_qkv_gemm_pack_workspace_size", 64, 96, ctypes.byref(need))
    assert need.value == 64 * 96 * 8


def test_qkv_gemm_pack_without_rows_is_a_noop_without_a_gpu():
    """No rows: nothing is projected and no CUDA call is made (empty tensors may carry null pointers)."""

    _lib.reset_launch_count()
    _lib.call("h3b_qkv_gemm_pack", None, 1, None, 0, 256, 256, None, None, None, None, None, None,
              2, 128, 96, 1e-6, 1e-6, None, 0, None)
    _lib.call("h3b_qkv_gemm_pack_p2p", (ctypes.c_void_p * 1)(1 << 20), 1, 0, 0, None, 0, 256, 256, None, None,
              None, None, None, None, 2, 128, 96, 1e-6, 1e-6, None, 0, None)
    assert _lib.launch_count() == 0


def test_every_declared_entry_point_has_a_python_signature():
    """The ctypes layer binds every function the header declares (argument types set)."""

    special = {"h3b_abi_version", "h3b_last_error", "h3b_device_status", "h3b_peer_flags_bytes",
               "h3b_kernel_launches", "h3b_reset_kernel_launches"}
    missing = [name for name in declared_functions() if name not in _lib.SIGNATURES and name not in special]
    assert not missing, missing


def test_python_signatures_match_the_header_arity():
    """Each bound function passes as many arguments as the header declares."""

    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    arity = {}
    for name, params in re.findall(r"\b(h3b_[a-z0-9_]+)\s*\(([^)]*)\)\s*;", text):
        params = params.strip()
        arity[name] = 0 if params in ("", "void") else len(params.split(","))
    for name, argtypes in _lib.SIGNATURES.items():
        assert arity.get(name) == len(argtypes), (name, arity.get(name), len(argtypes))
