"""The C-ABI library loads on a machine without a GPU and exports every
function include/metallora_b200.h declares; host-only entry points answer
without touching a device."""
import ctypes
import re
from pathlib import Path

import pytest

from metallora_b200 import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "metallora_b200.h"


def declared_functions():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"MLORA_API\s+[\w\s\*]+?\b(mlora_\w+)\s*\(", text)))


def test_header_declares_functions():
    names = declared_functions()
    assert "mlora_lora_forward" in names and "mlora_lora_backward" in names
    assert len(names) >= 10


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, f"not exported: {missing}"


def test_bindings_cover_header():
    assert set(declared_functions()) == set(_lib.SIGNATURES)


def test_host_only_queries():
    lib = _lib.load()
    assert lib.mlora_version() >= 100
    assert lib.mlora_status_string(0) == b"ok"
    assert lib.mlora_status_string(-1) == b"invalid argument"
    fwd = lib.mlora_lora_forward_workspace_bytes(8192, 4096, 4096, 16, _lib.DTYPE_BF16)
    bwd = lib.mlora_lora_backward_workspace_bytes(8192, 4096, 4096, 16, _lib.DTYPE_BF16)
    assert 0 < fwd < (64 << 20) and 0 < bwd < (64 << 20)
    assert lib.mlora_lora_forward_workspace_bytes(0, 4096, 4096, 16, 0) == 0
    f32 = lib.mlora_lora_forward_workspace_bytes(2048, 4096, 4096, 16, _lib.DTYPE_F32)
    assert f32 > 3 * 2048 * 4096 * 2
    assert lib.mlora_linear_workspace_bytes(128, 256, 256, _lib.DTYPE_BF16) == 0
    # quantised bases: the staged workspace holds a bf16 copy of deq(W); the
    # lean one (fused in-loop dequant) does not
    for bwd_flag, fn in ((0, lib.mlora_qlora_forward_workspace_bytes),
                         (1, lib.mlora_qlora_backward_workspace_bytes)):
        staged = fn(4096, 4096, 11008, 64, _lib.QUANT_NF4, 64)
        lean = lib.mlora_qlora_lean_workspace_bytes(4096, 4096, 11008, 64, _lib.QUANT_NF4, 64,
                                                    bwd_flag)
        assert 0 < lean < 11008 * 4096 * 2 <= staged < lean + 11008 * 4096 * 2 + (1 << 20)


def test_invalid_arguments_rejected_before_launch():
    lib = _lib.load()
    st = lib.mlora_lora_forward(None, None, None, None, None, None, 128, 256, 256, 16, 32.0,
                                _lib.DTYPE_BF16, None, 0, None)
    assert st == _lib.MLORA_ERR_INVALID_ARG
    assert b"NULL" in lib.mlora_last_error_message()
    st = lib.mlora_lora_forward(None, None, None, None, None, None, 128, 250, 256, 16, 32.0,
                                _lib.DTYPE_BF16, None, 0, None)
    assert st == _lib.MLORA_ERR_UNSUPPORTED
    st = lib.mlora_lora_forward(None, None, None, None, None, None, 128, 256, 256, 300, 32.0,
                                _lib.DTYPE_BF16, None, 0, None)
    assert st == _lib.MLORA_ERR_INVALID_ARG
    with pytest.raises(Exception):
        _lib.check(_lib.MLORA_ERR_INVALID_ARG, "x")
