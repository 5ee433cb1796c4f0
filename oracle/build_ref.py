"""TEST INFRASTRUCTURE ONLY — compiles the reference's own native module
(csrc/cache_ops/{bindings.cpp, copier.cpp, helpers.cu, kernels.cu} of the
reference checkout) for sm_100a into oracle/_ref/, where the GPU tests load it
as a bit-exact checker of scatter_pages / gather_pages. The sources are read
in place; nothing is copied into this repository.

    python oracle/build_ref.py --reference <path-to-DARIC-checkout>
"""
from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
SOURCES = ["bindings.cpp", "copier.cpp", "helpers.cu", "kernels.cu"]


def ref_module_path() -> Path | None:
    cands = sorted(OUT.glob("build/cache_ops*.so"))
    return cands[0] if cands else None


def build_ref(reference: str, verbose: bool = False) -> Path:
    src = Path(reference) / "csrc" / "cache_ops"
    if not all((src / s).exists() for s in SOURCES):
        raise FileNotFoundError(f"reference sources not found under {src}")
    existing = ref_module_path()
    if existing is not None:
        return existing
    from torch.utils.cpp_extension import load
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
    bdir = OUT / "build"
    bdir.mkdir(parents=True, exist_ok=True)
    load(name="cache_ops", sources=[str(src / s) for s in SOURCES], extra_include_paths=[str(src)],
         extra_cflags=["-O3", "-std=c++17"],
         extra_cuda_cflags=["-O3", "--use_fast_math", "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a"],
         build_directory=str(bdir), verbose=verbose, is_python_module=True)
    p = ref_module_path()
    if p is None:
        raise RuntimeError("reference module did not build")
    return p


def load_ref():
    """Imports the compiled reference module, or returns None if absent."""
    import importlib.util
    p = ref_module_path()
    if p is None:
        return None
    import torch  # noqa: F401  (the module links against torch)
    spec = importlib.util.spec_from_file_location("cache_ops", str(p))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    a = ap.parse_args()
    print(build_ref(a.reference, verbose=True))
