"""Stage the reference's own Python package as compiled bytecode under ``oracle/_ref/``.

Benchmark / test infrastructure only (the oracle's side of the repository): the reference
arm of ``bench.py`` and its CPU baseline run light-moe's own ``SparseMoEBlock``
(python/light_moe/model/moe_block.py:63-169) on the host cores.  The reference checkout is
not available where the benchmark runs, so this recipe byte-compiles every module of its
``light_moe`` package into ``oracle/_ref/light_moe/`` in the sourceless layout
(``module.pyc`` beside where ``module.py`` would be), which Python imports directly.  The
output is a build product, git-ignored, produced by running this script where the
checkout exists:

    python oracle/stage_reference.py /path/to/light-moe/python

The bytecode must match the interpreter that runs it (same Python minor version).
"""
from __future__ import annotations

import os
import py_compile
import shutil
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")


def stage(ref_python_dir: str, out_dir: str = OUT) -> int:
    """Byte-compile ``<ref_python_dir>/light_moe/**.py`` into ``out_dir``; returns the module count."""
    src_root = os.path.join(ref_python_dir, "light_moe")
    if not os.path.isdir(src_root):
        raise FileNotFoundError(f"{src_root} is not a light_moe package directory")
    dst_root = os.path.join(out_dir, "light_moe")
    if os.path.isdir(dst_root):
        shutil.rmtree(dst_root)
    n = 0
    for dirpath, dirnames, filenames in os.walk(src_root):
        dirnames[:] = [d for d in dirnames if d != "__pycache__"]
        rel = os.path.relpath(dirpath, src_root)
        dst = os.path.normpath(os.path.join(dst_root, rel))
        os.makedirs(dst, exist_ok=True)
        for fn in filenames:
            if fn.endswith(".py"):
                py_compile.compile(os.path.join(dirpath, fn), cfile=os.path.join(dst, fn[:-3] + ".pyc"),
                                   doraise=True)
                n += 1
    with open(os.path.join(out_dir, "STAGED_FROM"), "w") as f:
        f.write(f"light_moe\npython {sys.version_info.major}.{sys.version_info.minor}\n")
    return n


def available(out_dir: str = OUT) -> bool:
    """True when a staged package compiled for this interpreter is present."""
    marker = os.path.join(out_dir, "STAGED_FROM")
    if not os.path.exists(os.path.join(out_dir, "light_moe", "__init__.pyc")) or not os.path.exists(marker):
        return False
    with open(marker) as f:
        lines = f.read().splitlines()
    return len(lines) > 1 and lines[1] == f"python {sys.version_info.major}.{sys.version_info.minor}"


def import_sparse_moe_block(out_dir: str = OUT):
    """light_moe.model.moe_block.SparseMoEBlock from the staged bytecode."""
    if out_dir not in sys.path:
        sys.path.insert(0, out_dir)
    from light_moe.model.moe_block import SparseMoEBlock  # noqa: E402
    return SparseMoEBlock


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: python oracle/stage_reference.py <light-moe checkout>/python")
    print(f"staged {stage(sys.argv[1])} modules into {OUT}")
