"""Stage the reference's own Python package as compiled code objects under ``oracle/_ref/``.

Benchmark / test infrastructure only (the oracle's side of the repository): the reference
arm of ``bench.py`` and its CPU baseline run light-moe's own ``SparseMoEBlock``
(python/light_moe/model/moe_block.py:63-169) on the host cores.  The reference checkout is
not available where the benchmark runs, so this recipe compiles every module of its
``light_moe`` package and writes the marshalled code objects into
``oracle/_ref/light_moe/`` (``module.lmc`` beside where ``module.py`` would be; a ``.pyc``
suffix is avoided because file syncs commonly skip those).  ``import_sparse_moe_block``
imports the package from there through a small path finder.  The output is a build product,
git-ignored, produced by running this script where the checkout exists:

    python oracle/stage_reference.py /path/to/light-moe/python

The code objects must match the interpreter that runs them (same Python minor version).
"""
from __future__ import annotations

import importlib.abc
import importlib.util
import marshal
import os
import shutil
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
PKG = "light_moe"
SUFFIX = ".lmc"


def _version() -> str:
    return f"python {sys.version_info.major}.{sys.version_info.minor}"


def stage(ref_python_dir: str, out_dir: str = OUT) -> int:
    """Compile ``<ref_python_dir>/light_moe/**.py`` into ``out_dir``; returns the module count."""
    src_root = os.path.join(ref_python_dir, PKG)
    if not os.path.isdir(src_root):
        raise FileNotFoundError(f"{src_root} is not a light_moe package directory")
    dst_root = os.path.join(out_dir, PKG)
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
                path = os.path.join(dirpath, fn)
                with open(path, "rb") as f:
                    code = compile(f.read(), os.path.join(PKG, rel, fn), "exec", dont_inherit=True)
                with open(os.path.join(dst, fn[:-3] + SUFFIX), "wb") as f:
                    f.write(marshal.dumps(code))
                n += 1
    with open(os.path.join(out_dir, "STAGED_FROM"), "w") as f:
        f.write(f"{PKG}\n{_version()}\n")
    return n


def available(out_dir: str = OUT) -> bool:
    """True when a staged package compiled for this interpreter is present."""
    marker = os.path.join(out_dir, "STAGED_FROM")
    if not os.path.exists(os.path.join(out_dir, PKG, "__init__" + SUFFIX)) or not os.path.exists(marker):
        return False
    with open(marker) as f:
        lines = f.read().splitlines()
    return len(lines) > 1 and lines[1] == _version()


class _StagedLoader(importlib.abc.Loader):
    def __init__(self, path: str):
        self.path = path

    def create_module(self, spec):
        return None

    def exec_module(self, module):
        with open(self.path, "rb") as f:
            code = marshal.loads(f.read())
        exec(code, module.__dict__)


class _StagedFinder(importlib.abc.MetaPathFinder):
    def __init__(self, root: str):
        self.root = root

    def find_spec(self, fullname, path=None, target=None):
        if fullname != PKG and not fullname.startswith(PKG + "."):
            return None
        base = os.path.join(self.root, *fullname.split("."))
        if os.path.isdir(base) and os.path.exists(os.path.join(base, "__init__" + SUFFIX)):
            return importlib.util.spec_from_file_location(fullname, os.path.join(base, "__init__" + SUFFIX),
                                                          loader=_StagedLoader(os.path.join(base, "__init__" + SUFFIX)),
                                                          submodule_search_locations=[base])
        if os.path.exists(base + SUFFIX):
            return importlib.util.spec_from_file_location(fullname, base + SUFFIX, loader=_StagedLoader(base + SUFFIX))
        return None


def import_sparse_moe_block(out_dir: str = OUT):
    """light_moe.model.moe_block.SparseMoEBlock from the staged code objects."""
    if not any(isinstance(f, _StagedFinder) for f in sys.meta_path):
        sys.meta_path.insert(0, _StagedFinder(out_dir))
    from light_moe.model.moe_block import SparseMoEBlock  # noqa: E402
    return SparseMoEBlock


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: python oracle/stage_reference.py <light-moe checkout>/python")
    print(f"staged {stage(sys.argv[1])} modules into {OUT}")
