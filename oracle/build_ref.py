"""Build recipe for ``oracle/_ref/libmlref.so`` -- test infrastructure only.

Compiles the reference's own Metal compute shaders as host C++ (through the
shim headers in ``oracle/msl_shim``) so the numpy oracle can be checked against
the reference itself.  Inputs are read where they lie in the reference tree:

* ``kernels/lora_quantized.metal`` and ``kernels/lora_train.metal``, included
  directly by ``oracle/ref_driver.cpp``;
* the inline MSL kernel bodies of ``python/metal_lora/kernels.py``
  (``LORA_FORWARD_FUSED_SOURCE`` :41, ``LORA_BACKWARD_SOURCE`` :249,
  ``LORA_ADAMW_SOURCE`` :314, ``LORA_MAINTENANCE_SOURCE`` :351), pulled out with
  ``ast`` (the module imports MLX, which is not installed, so it is parsed, not
  imported) and written to ``oracle/_ref/gen/*.inc``;
* from ``kernels/lora_kernels.metal``, the ``LoRAConfig`` struct (:12) and the
  kernels ``lora_multi_adapter`` (:440) and ``lora_kv_cache_update`` (:514),
  cut out by brace matching into ``oracle/_ref/gen/lora_kernels_subset.inc``
  (the file as a whole needs simdgroup-matrix types the shim does not have).

Everything this writes goes to ``oracle/_ref/`` (git-ignored).  Nothing here
runs the reference's build system.  The reference tree must be named, by
argument or by the ``MLORA_REFERENCE_DIR`` environment variable; there is no
default location.  Usage::

    python oracle/build_ref.py --reference /path/to/MetalLora
    MLORA_REFERENCE_DIR=/path/to/MetalLora python oracle/build_ref.py
"""
from __future__ import annotations

import argparse
import ast
import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"

# kernels.py string constant -> generated include name
INLINE_BODIES = {
    "LORA_FORWARD_FUSED_SOURCE": "lora_forward_fused.inc",
    "LORA_BACKWARD_SOURCE": "lora_backward_fused.inc",
    "LORA_ADAMW_SOURCE": "lora_adamw_step.inc",
    "LORA_MAINTENANCE_SOURCE": "lora_maintenance.inc",
}


def extract_inline_bodies(kernels_py: Path) -> dict[str, str]:
    tree = ast.parse(kernels_py.read_text())
    found: dict[str, str] = {}
    for node in tree.body:
        if (
            isinstance(node, ast.Assign)
            and len(node.targets) == 1
            and isinstance(node.targets[0], ast.Name)
            and node.targets[0].id in INLINE_BODIES
            and isinstance(node.value, ast.Constant)
            and isinstance(node.value.value, str)
        ):
            found[node.targets[0].id] = node.value.value
    missing = set(INLINE_BODIES) - set(found)
    if missing:
        raise RuntimeError(f"inline kernel sources not found in {kernels_py}: {sorted(missing)}")
    return found


# blocks of kernels/lora_kernels.metal compiled for the oracle, by their first words
METAL_BLOCKS = ("struct LoRAConfig", "kernel void lora_multi_adapter",
                "kernel void lora_kv_cache_update")


def extract_metal_blocks(path: Path, heads=METAL_BLOCKS) -> str:
    """The source text of each named struct / kernel of a .metal file, from
    its first word to its matching closing brace (and ';' for a struct),
    each preceded by a #line directive pointing at the original file."""
    src = path.read_text()
    out = []
    for head in heads:
        start = src.find(head)
        if start < 0:
            raise RuntimeError(f"{head!r} not found in {path}")
        depth, end = 0, -1
        for k in range(src.index("{", start), len(src)):
            if src[k] == "{":
                depth += 1
            elif src[k] == "}":
                depth -= 1
                if depth == 0:
                    end = k + 1
                    break
        if end < 0:
            raise RuntimeError(f"unbalanced braces after {head!r} in {path}")
        if head.startswith("struct"):
            end = src.index(";", end) + 1
        line = src.count("\n", 0, start) + 1
        out.append(f'#line {line} "{path.name}"\n{src[start:end]}')
    return "\n\n".join(out) + "\n"


def build(reference: str | os.PathLike | None = None, quiet: bool = False) -> Path | None:
    """Build ``oracle/_ref/libmlref.so``; returns its path, or None when no
    reference tree is named or the named one is absent (the prebuilt library
    is then used as is)."""
    named = reference or os.environ.get("MLORA_REFERENCE_DIR")
    if not named:
        if not quiet:
            print("[oracle/_ref] no reference tree named (--reference or MLORA_REFERENCE_DIR); "
                  "skipping", file=sys.stderr)
        return None
    ref = Path(named)
    kernels_py = ref / "python" / "metal_lora" / "kernels.py"
    kernels_dir = ref / "kernels"
    if not kernels_py.is_file() or not (kernels_dir / "lora_quantized.metal").is_file():
        if not quiet:
            print(f"[oracle/_ref] reference tree not found at {ref}; skipping", file=sys.stderr)
        return None
    gen = OUT / "gen"
    gen.mkdir(parents=True, exist_ok=True)
    for const, fname in INLINE_BODIES.items():
        body = extract_inline_bodies(kernels_py)[const]
        (gen / fname).write_text(body)
    (gen / "lora_kernels_subset.inc").write_text(
        extract_metal_blocks(kernels_dir / "lora_kernels.metal"))
    lib = OUT / "libmlref.so"
    cmd = [
        "g++", "-O2", "-std=c++17", "-fopenmp", "-ffp-contract=off", "-fPIC", "-shared",
        "-Wno-attributes", "-Wno-unused-variable", "-Wno-unused-parameter",
        "-I", str(HERE / "msl_shim"), "-I", str(kernels_dir), "-I", str(gen),
        str(HERE / "ref_driver.cpp"), "-o", str(lib),
    ]
    subprocess.run(cmd, check=True)
    if not quiet:
        print(f"[oracle/_ref] built {lib}")
    return lib


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=None,
                    help="reference tree (default: $MLORA_REFERENCE_DIR)")
    args = ap.parse_args()
    if not (args.reference or os.environ.get("MLORA_REFERENCE_DIR")):
        ap.error("name the reference tree with --reference or MLORA_REFERENCE_DIR")
    if build(args.reference) is None:
        sys.exit(1)
