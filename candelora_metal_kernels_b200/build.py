"""Builds the CUDA library of this package for sm_100a, in place.

    python -m candelora_metal_kernels_b200.build        (or build() from Python)

Output: candelora_metal_kernels_b200/lib/libcandelora_iq2.so, a C-ABI shared library (the
symbols of include/candelora_iq2.h) with the CUDA runtime linked statically, so it runs in any
process that has a CUDA driver, next to whatever runtime that process already loaded.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
LIB_DIR = PKG / "lib"
LIB = LIB_DIR / "libcandelora_iq2.so"
SOURCES = ["iq2xxs_capi.cu", "iq2xxs_gemv.cu", "iq2xxs_gemm.cu", "iq2xxs_dequant.cu", "iq2xxs_noalloc.cu",
           "iq2xxs_sharded.cu", "iq2_variants.cu"]
HEADERS = ["iq2xxs_common.cuh", "iq2xxs_codebook.h", "iq2xxs_internal.h", "iq2_variant_grids.h"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).is_file():
            return cand
    raise FileNotFoundError("nvcc not found")


def _stale() -> bool:
    if not LIB.is_file():
        return True
    t = LIB.stat().st_mtime
    deps = [CSRC / s for s in SOURCES + HEADERS] + [PKG.parent / "include" / h for h in
                                                    ("candelora_iq2.h", "candelora_iq2_testing.h")] + [Path(__file__)]
    return any(d.stat().st_mtime > t for d in deps if d.is_file())


def build(force: bool = False, verbose: bool = False, jobs: int | None = None) -> Path:
    if not force and not _stale():
        return LIB
    LIB_DIR.mkdir(exist_ok=True)
    obj_dir = LIB_DIR / "obj"
    obj_dir.mkdir(exist_ok=True)
    common = ["-std=c++17", "-O3", "-lineinfo", *ARCH, "-Xcompiler", "-fPIC,-O2", "--expt-relaxed-constexpr",
              "-I", str(CSRC), "-I", str(PKG.parent / "include")]
    if verbose:
        common += ["-Xptxas", "-v"]
    objs = []
    procs = []
    for src in SOURCES:
        obj = obj_dir / (Path(src).stem + ".o")
        objs.append(obj)
        cmd = [nvcc(), *common, "-c", str(CSRC / src), "-o", str(obj)]
        procs.append((cmd, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)))
    failed = []
    for cmd, p in procs:
        out, _ = p.communicate()
        text = out.decode(errors="replace")
        if p.returncode != 0:
            failed.append(" ".join(cmd) + "\n" + text)
        elif verbose and text.strip():
            print(text)
    if failed:
        raise RuntimeError("nvcc failed:\n" + "\n".join(failed))
    tmp = LIB.with_suffix(".so.tmp")
    link = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs), "-lnccl"]
    subprocess.run(link, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
