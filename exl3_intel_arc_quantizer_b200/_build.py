"""In-tree build of the native layer.

Two artefacts land in ``exl3_intel_arc_quantizer_b200/_lib/``:

* ``libexl3k.so`` — every CUDA kernel behind the C ABI of ``include/exl3k.h``,
  compiled by nvcc for ``sm_100a`` only;
* ``exl3_b200_ext.so`` — the PyTorch binding (``csrc/torch_ext.cpp``), which
  validates tensors and calls the C ABI; its dependency on ``libexl3k.so``
  (by SONAME) resolves against the copy the loader opens first.

Each artefact carries a stamp with the SHA-256 of its inputs (sources, headers,
flags). A stamp that matches means the shipped binary is current, so a copy of
the tree (for instance on a GPU host) loads it without recompiling.
"""

from __future__ import annotations

import concurrent.futures as _futures
import hashlib
import os
import shutil
import subprocess
import sys
from pathlib import Path
from typing import Iterable, List

PKG_DIR = Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent
CSRC_DIR = PKG_DIR / "csrc"
INCLUDE_DIR = REPO_DIR / "include"
LIB_DIR = PKG_DIR / "_lib"

LIB_NAME = "libexl3k.so"
EXT_NAME = "exl3_b200_ext"

CU_SOURCES = ["abi.cu", "encoder.cu", "acs_pair.cu", "acs_cluster.cu", "noalloc.cu", "linalg.cu", "hessian.cu", "storage.cu", "ldlq.cu", "regularize.cu"]
EXT_SOURCES = ["torch_ext.cpp", "torch_ext_linalg.cpp"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC",
    "--expt-relaxed-constexpr",
]
LINK_FLAGS = ["-shared", "-gencode", "arch=compute_100a,code=sm_100a",
              "-Xlinker", f"-soname={LIB_NAME}", "-lcudart"]


def _nvcc() -> str:
    cand = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    path = Path(cand) / "bin" / "nvcc"
    if path.exists():
        return str(path)
    found = shutil.which("nvcc")
    if not found:
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libexl3k")
    return found


def _existing(names: Iterable[str]) -> List[Path]:
    return [CSRC_DIR / n for n in names if (CSRC_DIR / n).exists()]


def _digest(paths: Iterable[Path], extra: Iterable[str]) -> str:
    h = hashlib.sha256()
    for p in sorted(paths):
        h.update(p.name.encode())
        h.update(p.read_bytes())
    for e in extra:
        h.update(e.encode())
    return h.hexdigest()


def _headers() -> List[Path]:
    hs = sorted(CSRC_DIR.glob("*.cuh")) + sorted(CSRC_DIR.glob("*.h"))
    hs += sorted(INCLUDE_DIR.glob("*.h"))
    return hs


def _stamp_ok(artefact: Path, digest: str) -> bool:
    stamp = artefact.with_name(artefact.name + ".sha256")
    return artefact.exists() and stamp.exists() and stamp.read_text().strip() == digest


def _write_stamp(artefact: Path, digest: str) -> None:
    artefact.with_name(artefact.name + ".sha256").write_text(digest + "\n")


def library_digest() -> str:
    return _digest(_existing(CU_SOURCES) + _headers(), NVCC_FLAGS + LINK_FLAGS)


def library_path() -> Path:
    return LIB_DIR / LIB_NAME


def build_library(force: bool = False, verbose: bool = False) -> Path:
    """Compile every ``.cu`` source and link ``libexl3k.so`` (sm_100a)."""
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    out = library_path()
    digest = library_digest()
    if not force and _stamp_ok(out, digest):
        return out
    nvcc = _nvcc()
    obj_dir = LIB_DIR / "obj"
    obj_dir.mkdir(exist_ok=True)
    sources = _existing(CU_SOURCES)

    def compile_one(src: Path) -> Path:
        obj = obj_dir / (src.stem + ".o")
        cmd = [nvcc, *NVCC_FLAGS, "-I", str(INCLUDE_DIR), "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stdout}\n{res.stderr}")
        return obj

    with _futures.ThreadPoolExecutor(max_workers=max(1, min(len(sources), os.cpu_count() or 1))) as ex:
        objs = list(ex.map(compile_one, sources))
    tmp = out.with_name(out.name + ".tmp")
    cmd = [nvcc, *LINK_FLAGS[:-1], *map(str, objs), "-o", str(tmp), LINK_FLAGS[-1]]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link of {LIB_NAME} failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, out)
    _write_stamp(out, digest)
    return out


def extension_path() -> Path:
    return LIB_DIR / f"{EXT_NAME}.so"


def extension_digest() -> str:
    import torch

    return _digest(_existing(EXT_SOURCES) + _headers(),
                   [torch.__version__, sys.version.split()[0]])


def build_extension(force: bool = False, verbose: bool = False) -> Path:
    """Build the PyTorch binding ``exl3_b200_ext.so`` against libexl3k."""
    import ctypes

    from torch.utils import cpp_extension

    lib_path = build_library(force=False, verbose=verbose)
    # The binding's DT_NEEDED entry resolves against this already-loaded
    # SONAME, wherever the tree is copied.
    ctypes.CDLL(str(lib_path), mode=ctypes.RTLD_GLOBAL)
    out = extension_path()
    digest = extension_digest()
    if not force and _stamp_ok(out, digest):
        return out
    build_dir = LIB_DIR / "ext_build"
    build_dir.mkdir(parents=True, exist_ok=True)
    cpp_extension.load(
        name=EXT_NAME,
        sources=[str(p) for p in _existing(EXT_SOURCES)],
        build_directory=str(build_dir),
        extra_cflags=["-O2", "-std=c++17"],
        extra_include_paths=[str(INCLUDE_DIR)],
        extra_ldflags=[f"-L{LIB_DIR}", "-lexl3k"],
        with_cuda=True,
        verbose=verbose,
        is_python_module=True,
    )
    built = build_dir / f"{EXT_NAME}.so"
    shutil.copy2(built, out)
    _write_stamp(out, digest)
    return out


def build_all(force: bool = False, verbose: bool = False) -> None:
    build_library(force=force, verbose=verbose)
    build_extension(force=force, verbose=verbose)


if __name__ == "__main__":
    build_all(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(library_path())
    print(extension_path())
