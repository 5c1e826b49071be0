"""Build recipe for the reference's own CUDA decode kernel (test and benchmark
infrastructure only -- never part of the product path).

Compiles ``learning/10_cuda_decode/warp_gemv.cu`` of the reference checkout,
unmodified and from where it lies, into a torch extension under
``oracle/_ref/`` with the reference's own flags (``cuda_decode.py:9-14``:
``-O3 -lineinfo``) for sm_100.  The built module is what ``bench.py`` times as
GPU context for the reference's decode projection (``project(x, w, scales,
inverse, group, warps, persistent, swiglu)``, ``warp_gemv.cu:56-91``).  The
reference checkout exists only where the sources are built; the GPU box loads
the prebuilt ``.so`` with :func:`load`.
"""
from __future__ import annotations

import importlib.util
import os
from pathlib import Path

REF = Path(os.environ.get("KL_REFERENCE_ROOT", "/root/reference"))
SOURCE = REF / "learning" / "10_cuda_decode" / "warp_gemv.cu"
OUT = Path(__file__).resolve().parent / "_ref"
NAME = "kernellab_warp_decode_v1"        # the reference's extension name


def built_path() -> Path:
    return OUT / f"{NAME}.so"


def build(verbose: bool = False) -> Path | None:
    """Compile the reference kernel if its sources are present; returns the .so."""
    if not SOURCE.exists():
        return None
    so = built_path()
    if so.exists() and so.stat().st_mtime >= SOURCE.stat().st_mtime:
        return so
    OUT.mkdir(exist_ok=True)
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0")
    os.environ.setdefault("MAX_JOBS", "4")
    from torch.utils.cpp_extension import load
    load(name=NAME, sources=[str(SOURCE)], extra_cuda_cflags=["-O3", "-lineinfo"], build_directory=str(OUT),
         verbose=verbose)
    return so if so.exists() else None


def load():
    """The prebuilt reference extension module, or None if it was not built."""
    so = built_path()
    if not so.exists():
        return None
    import torch  # noqa: F401  (its libraries must be loaded first)
    spec = importlib.util.spec_from_file_location(NAME, so)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    print(build(verbose=True))
