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


_SWEEP = r'''
import ctypes as C, json, sys
sys.path.insert(0, sys.argv[1])
from metallora_b200 import _lib
lib = _lib.load()
host_only = {"mlora_device_supported", "mlora_launch_count", "mlora_profile_enable",
             "mlora_version"}
out = {}
for name in sorted(_lib.SIGNATURES):
    fn = getattr(lib, name)
    if fn.restype is not C.c_int or name in host_only:
        continue
    for fill in (64, 0):
        args = []
        for t in fn.argtypes or []:
            if t in (C.c_float, C.c_double):
                args.append(1.0)
            elif t in (C.c_int, C.c_int32, C.c_int64, C.c_uint32, C.c_uint64, C.c_size_t,
                       C.c_longlong, C.c_long):
                args.append(fill)
            else:
                args.append(None)
        out.setdefault(name, []).append(int(fn(*args)))
print(json.dumps(out))
'''


@pytest.mark.skipif(__import__("torch").cuda.is_available(),
                    reason="a host-only check: run it where no GPU can be reached")
def test_every_launching_entry_point_rejects_null_pointers():
    """Every status-returning entry point, called with NULL pointers (and
    sizes of 64 or 0), returns a negative status instead of touching memory or
    a device; the sweep runs in a child process so a crash fails the test."""
    import json
    import subprocess
    import sys
    root = Path(__file__).resolve().parents[1]
    p = subprocess.run([sys.executable, "-c", _SWEEP, str(root)], capture_output=True,
                       text=True, timeout=300)
    assert p.returncode == 0, p.stderr[-2000:]
    res = json.loads(p.stdout.strip().splitlines()[-1])
    assert "mlora_lora_forward" in res and "mlora_peer_allreduce" in res
    bad = {k: v for k, v in res.items() if any(s >= 0 for s in v)}
    assert not bad, bad


_C_CALLER = r'''
#include <stdio.h>
#include "metallora_b200.h"
int main(void) {
  printf("%d %s %zu %zu\n", mlora_version(), mlora_status_string(MLORA_OK),
         mlora_lora_forward_workspace_bytes(8192, 4096, 4096, 16, MLORA_DTYPE_BF16),
         mlora_lora_grads_static_scratch_bytes());
  return mlora_lora_forward(NULL, NULL, NULL, NULL, NULL, NULL, 128, 256, 256, 16, 32.0f,
                            MLORA_DTYPE_BF16, NULL, 0, NULL) < 0 ? 0 : 1;
}
'''


@pytest.mark.skipif(__import__("shutil").which("gcc") is None, reason="gcc not installed")
def test_plain_c_caller(tmp_path):
    """The header is valid C99 (-Wall -Wextra -pedantic -Werror) and a plain C
    program links the library and calls its host-only entry points (no GPU
    needed), getting the same answers as the Python binding."""
    import subprocess
    root = Path(__file__).resolve().parents[1]
    inc, libdir = root / "include", _lib.LIB_PATH.parent
    subprocess.run(["gcc", "-fsyntax-only", "-std=c99", "-Wall", "-Wextra", "-pedantic",
                    "-Werror", "-x", "c", str(HEADER)], check=True)
    src = tmp_path / "caller.c"
    src.write_text(_C_CALLER)
    exe = tmp_path / "caller"
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", f"-I{inc}", str(src), f"-L{libdir}",
                    "-lmetallora_b200", f"-Wl,-rpath,{libdir}", "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stderr
    version, status, fwd_ws, scratch = out.stdout.split()
    lib = _lib.load()
    assert int(version) == lib.mlora_version() and status == "ok"
    assert int(fwd_ws) == lib.mlora_lora_forward_workspace_bytes(8192, 4096, 4096, 16,
                                                                 _lib.DTYPE_BF16)
    assert int(scratch) == lib.mlora_lora_grads_static_scratch_bytes()
