"""Build the C-ABI shared library ``libhyfft.so`` in-tree with nvcc (sm_100a).

    python -m nvsubquadratic_b200.build            # build if sources changed
    python -m nvsubquadratic_b200.build --force    # always rebuild

The library links the CUDA runtime statically and exports only the ``hyfft_*``
symbols declared in ``include/hyfft.h``.
"""

from __future__ import annotations

import argparse
import hashlib
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "libhyfft.so"
STAMP = PKG / ".libhyfft.stamp"

SOURCES = ["engine.cu", "cp.cu", "fused.cu", "toeplitz.cu", "big2d.cu", "shortconv.cu", "transpose_tma.cu", "fft_long.cu", "siren.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found (set NVCC or put /usr/local/cuda/bin on PATH)")


def _digest() -> str:
    h = hashlib.sha256()
    for p in sorted(CSRC.glob("*")) + sorted((ROOT / "include").glob("*.h")):
        if p.is_file():
            h.update(p.name.encode())
            h.update(p.read_bytes())
    h.update(" ".join(ARCH).encode())
    return h.hexdigest()


def _object_digest(src: Path, common: list[str]) -> str:
    """Inputs of one object file: the source, every shared header, the flags."""
    h = hashlib.sha256()
    for p in [src] + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted((ROOT / "include").glob("*.h")):
        h.update(p.name.encode())
        h.update(p.read_bytes())
    h.update(" ".join(common).encode())
    return h.hexdigest()


def build(force: bool = False, verbose: bool = False) -> Path:
    digest = _digest()
    if not force and LIB.exists() and STAMP.exists() and STAMP.read_text().strip() == digest:
        return LIB
    nvcc = _nvcc()
    tmp = PKG / "_build"
    tmp.mkdir(exist_ok=True)
    common = [
        "-O3", "-std=c++17", "-lineinfo", *ARCH, "-Xcompiler", "-fPIC,-fvisibility=hidden",
        "-I", str(ROOT / "include"), "--expt-relaxed-constexpr",
    ]
    if verbose:
        common += ["-Xptxas", "-v"]

    def compile_one(src: str) -> str:
        s = CSRC / src
        o = tmp / (s.stem + ".o")
        stamp = tmp / (s.stem + ".o.stamp")
        od = _object_digest(s, common)
        if not force and o.exists() and stamp.exists() and stamp.read_text().strip() == od:
            return str(o)
        r = subprocess.run([nvcc, *common, "-c", str(s), "-o", str(o)], capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
        if verbose and r.stderr:
            print(r.stderr, file=sys.stderr)
        stamp.write_text(od)
        return str(o)

    srcs = [s for s in SOURCES if (CSRC / s).exists()]
    with ThreadPoolExecutor(max_workers=len(srcs)) as pool:
        objs = list(pool.map(compile_one, srcs))
    out_tmp = tmp / "libhyfft.so"
    cmd = [nvcc, *ARCH, "-shared", "-cudart", "static", "-o", str(out_tmp), *objs]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(out_tmp, LIB)
    STAMP.write_text(digest)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))
