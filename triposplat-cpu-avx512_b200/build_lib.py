"""Build the product library ``libtriposplat_b200.so`` in-tree with nvcc.

Every ``csrc/*.cu`` file is compiled for sm_100a only
(``-gencode arch=compute_100a,code=sm_100a``) and linked into one shared
library exporting the C-ABI declared in ``include/triposplat_b200.h``.  The
CUDA runtime is linked statically so the library needs nothing but the driver.
"""
from __future__ import annotations

import concurrent.futures as cf
import hashlib
import os
import shutil
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
BUILD = HERE / "_build"
LIB = HERE / "libtriposplat_b200.so"
STAMP = HERE / "libtriposplat_b200.so.sha256"  # digest of the sources the library was built from
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-O3",
         "--expt-relaxed-constexpr", "-DNDEBUG"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _compile(src: Path, verbose: bool) -> Path:
    obj = BUILD / (src.stem + ".o")
    cmd = [nvcc(), *ARCH, *FLAGS, "-c", str(src), "-o", str(obj)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stderr}")
    if verbose and res.stderr:
        print(res.stderr)
    return obj


def source_digest() -> str:
    """sha256 over the compiler command and every source and header, in name order."""
    h = hashlib.sha256(" ".join([*ARCH, *FLAGS]).encode())
    for p in sorted([*CSRC.glob("*.cu"), *CSRC.glob("*.cuh"), *CSRC.glob("*.h")]):
        h.update(p.name.encode() + b"\0" + p.read_bytes() + b"\0")
    return h.hexdigest()


def build(verbose: bool = False, force: bool = False) -> Path:
    """Compile and link unless the library was built from exactly these sources (the
    digest recorded beside it matches); file times are not trusted."""
    sources = sorted(CSRC.glob("*.cu"))
    digest = source_digest()
    if LIB.exists() and not force and STAMP.is_file() and STAMP.read_text().strip() == digest:
        return LIB
    BUILD.mkdir(exist_ok=True)
    with cf.ThreadPoolExecutor(max_workers=min(8, len(sources))) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), sources))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-cudart", "static"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stderr}")
    os.replace(tmp, LIB)
    STAMP.write_text(digest + "\n")
    return LIB


if __name__ == "__main__":
    import sys

    print(build(verbose="-v" in sys.argv, force=True))
