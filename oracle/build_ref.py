#!/usr/bin/env python3
"""Build recipe for ``oracle/_ref/``: the reference's own Python package,
byte-compiled — TEST AND BASELINE INFRASTRUCTURE ONLY.

The reference (alpha2beta/EXL3_Intel_Arc_quantizer) is Python: its CPU
encoder ``exl3_quant.reference_encoder.ReferenceTrellisEncoder`` is the CPU
path the benchmark times as its reference line, and its ``ldlq`` /
``layer_quant`` are what the drop-in tests drive with the B200 encoder. The
reference checkout exists only in the build container, so this recipe
compiles each module of its ``exl3_quant`` package where it lies into a
sourceless ``.pyc`` under ``oracle/_ref/exl3_quant/``: a build output, like
the ``.so`` of a compiled C reference, that travels with the tree (git
ignores it). No source file is copied. Python imports a package of sourceless
``.pyc`` files of the same interpreter version directly.

    python oracle/build_ref.py --reference /path/to/EXL3_Intel_Arc_quantizer

Only ``tests/`` and ``bench.py``'s reference leg import ``oracle/_ref``.
"""

from __future__ import annotations

import argparse
import py_compile
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
PACKAGE = "exl3_quant"


def build(reference: Path, out: Path = OUT) -> Path:
    src_pkg = reference / PACKAGE
    if not (src_pkg / "__init__.py").is_file():
        raise FileNotFoundError(f"{src_pkg} is not the reference's {PACKAGE} package")
    dst_pkg = out / PACKAGE
    dst_pkg.mkdir(parents=True, exist_ok=True)
    stamp = out / "VERSION"
    tag = f"{sys.version_info.major}.{sys.version_info.minor}"
    for src in sorted(src_pkg.glob("*.py")):
        dst = dst_pkg / (src.stem + ".pyc")
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
    return ((OUT / PACKAGE / "__init__.pyc").is_file() and stamp.is_file()
            and stamp.read_text().strip() == tag)


def import_path() -> str:
    """The directory to put on ``sys.path`` to import ``exl3_quant``."""
    return str(OUT)


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, type=Path)
    print(build(ap.parse_args().reference))
