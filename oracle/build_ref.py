#!/usr/bin/env python3
"""Build recipe for ``oracle/_ref/``: the reference's own Python package,
byte-compiled — TEST AND BASELINE INFRASTRUCTURE ONLY.

The reference (alpha2beta/EXL3_Intel_Arc_quantizer) is Python: its CPU
encoder ``exl3_quant.reference_encoder.ReferenceTrellisEncoder`` is the CPU
path the benchmark times as its reference line, and its ``ldlq`` /
``layer_quant`` are what the drop-in tests drive with the B200 encoder. The
reference checkout exists only in the build container, so this recipe
compiles each module of its ``exl3_quant`` package where it lies into
byte code (the ``.pyc`` format, under the suffix ``.refc`` so that tools
which drop ``.pyc`` files from a copy of the tree keep these) in
``oracle/_ref/exl3_quant/``: a build output, like the ``.so`` of a compiled C
reference, that travels with the tree (git ignores it). No source file is
copied. :func:`enable` adds an import finder that loads the package from
there with Python's sourceless loader (same interpreter version only).

    python oracle/build_ref.py --reference /path/to/EXL3_Intel_Arc_quantizer

Only ``tests/`` and ``bench.py``'s reference leg import ``oracle/_ref``.
"""

from __future__ import annotations

import argparse
import importlib.abc
import importlib.machinery
import importlib.util
import py_compile
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
PACKAGE = "exl3_quant"
SUFFIX = ".refc"


def build(reference: Path, out: Path = OUT) -> Path:
    src_pkg = reference / PACKAGE
    if not (src_pkg / "__init__.py").is_file():
        raise FileNotFoundError(f"{src_pkg} is not the reference's {PACKAGE} package")
    dst_pkg = out / PACKAGE
    dst_pkg.mkdir(parents=True, exist_ok=True)
    stamp = out / "VERSION"
    tag = f"{sys.version_info.major}.{sys.version_info.minor}"
    for src in sorted(src_pkg.glob("*.py")):
        dst = dst_pkg / (src.stem + SUFFIX)
        if dst.exists() and dst.stat().st_mtime >= src.stat().st_mtime and stamp.exists() \
                and stamp.read_text().strip() == tag:
            continue
        py_compile.compile(str(src), cfile=str(dst), doraise=True,
                           invalidation_mode=py_compile.PycInvalidationMode.UNCHECKED_HASH)
    stamp.write_text(tag + "\n")
    return dst_pkg


def available() -> bool:
    """True when the compiled reference package is present and was built by
    this interpreter version."""
    stamp = OUT / "VERSION"
    tag = f"{sys.version_info.major}.{sys.version_info.minor}"
    return ((OUT / PACKAGE / ("__init__" + SUFFIX)).is_file() and stamp.is_file()
            and stamp.read_text().strip() == tag)


class _Finder(importlib.abc.MetaPathFinder):
    """Finds ``exl3_quant`` and its modules among the compiled files."""

    def find_spec(self, fullname, path=None, target=None):
        parts = fullname.split(".")
        if parts[0] != PACKAGE or len(parts) > 2:
            return None
        pkg_dir = OUT / PACKAGE
        if len(parts) == 1:
            f = pkg_dir / ("__init__" + SUFFIX)
            return importlib.util.spec_from_file_location(
                fullname, str(f), loader=importlib.machinery.SourcelessFileLoader(fullname, str(f)),
                submodule_search_locations=[str(pkg_dir)])
        f = pkg_dir / (parts[1] + SUFFIX)
        if not f.is_file():
            return None
        return importlib.util.spec_from_file_location(
            fullname, str(f), loader=importlib.machinery.SourcelessFileLoader(fullname, str(f)))


_FINDER = _Finder()


def enable() -> None:
    """Make ``import exl3_quant`` load the compiled reference package (ahead
    of any other ``exl3_quant`` on ``sys.path``)."""
    if _FINDER not in sys.meta_path:
        sys.meta_path.insert(0, _FINDER)


def disable() -> None:
    if _FINDER in sys.meta_path:
        sys.meta_path.remove(_FINDER)


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, type=Path)
    print(build(ap.parse_args().reference))
