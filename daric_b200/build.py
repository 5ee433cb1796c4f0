"""Build recipe of the native library ``daric_b200/libdaric_b200.so``.

The library is compiled in-tree with nvcc for sm_100a only
(``-gencode arch=compute_100a,code=sm_100a``) and links the CUDA runtime
statically, so it does not depend on which libcudart the host process has
loaded. Run ``python -m daric_b200.build`` (or ``__graft_entry__.build()``).
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
OUT = PKG / "libdaric_b200.so"
BUILD = ROOT / "_build"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
SOURCES = ["capi.cpp", "page_kernels.cu", "bulk_kernels.cu", "inplace_kernels.cu", "select_kernels.cu"]


def nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    return cand


def _flags() -> list[str]:
    # -fmad=false: the rotation is specified as separately rounded products
    # and sums (the reference's math without contraction); no mul+add pair
    # may be fused into an FMA.
    return [
        "-O3", "-std=c++17", "-lineinfo", "-fmad=false", "-Xcompiler", "-fPIC", "-Xcompiler",
        "-fvisibility=hidden", "-I", str(ROOT / "include"), "-DNDEBUG",
    ]


def _compile(src: Path, obj: Path, extra: list[str]) -> None:
    cmd = [nvcc(), *ARCH, *_flags(), *extra, "-x", "cu" if src.suffix == ".cu" else "c++",
           "-c", str(src), "-o", str(obj)]
    if src.suffix == ".cpp":
        cmd = [nvcc(), *ARCH, *_flags(), *extra, "-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
    if r.stderr.strip():
        sys.stderr.write(r.stderr)


def up_to_date() -> bool:
    if not OUT.exists():
        return False
    t = OUT.stat().st_mtime
    deps = list(CSRC.glob("*")) + [ROOT / "include" / "daric_b200.h", Path(__file__)]
    return all(d.stat().st_mtime <= t for d in deps if d.exists())


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> Path:
    if not force and up_to_date():
        return OUT
    BUILD.mkdir(exist_ok=True)
    extra = ["-Xptxas", "-v"] if ptxas_info else []
    objs = []
    with cf.ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        futs = []
        for s in SOURCES:
            src = CSRC / s
            obj = BUILD / (src.stem + ".o")
            objs.append(obj)
            futs.append(ex.submit(_compile, src, obj, extra))
        for f in futs:
            f.result()
    tmp = OUT.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static",
           "-Xlinker", f"--version-script={CSRC / 'exports.map'}", "-o", str(tmp), *map(str, objs)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, OUT)
    if verbose:
        print(f"built {OUT}")
    return OUT


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True, ptxas_info="--ptxas-info" in sys.argv)
