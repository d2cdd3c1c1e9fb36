"""Build and load the in-tree sm_100a extensions (`saelens_b200/ops/_build/_C*.so` and the debug-bounds
module `saelens_b200/ops/_build_debug/_C_debug*.so`).

The extension is compiled once, in-tree, with `-gencode arch=compute_100a,code=sm_100a`
(nvcc cross-compiles without a GPU).  At import time on a CUDA machine the prebuilt `.so` is
loaded directly from the package directory; if it is missing the import fails loudly instead
of silently falling back to PyTorch ops.

The debug-bounds module compiles the kernels that dereference data-dependent indices (sparse
decode / CSC / latent gradients, top-k merges, ring gather and row router, with their bindings)
with `-DSB_DEBUG_BOUNDS=1`: every such index is checked before use, and a violation is skipped
and recorded instead of touching memory out of range (see `csrc/bounds.cuh`).
"""

from __future__ import annotations

import glob
import importlib.util
import os
import sys
from types import ModuleType

_HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(_HERE, "csrc")
BUILD_DIR = os.path.join(_HERE, "_build")
EXT_NAME = "_C"
DEBUG_BUILD_DIR = os.path.join(_HERE, "_build_debug")
DEBUG_EXT_NAME = "_C_debug"
DEBUG_SOURCES = ["bindings.cpp", "topk.cu", "sparse.cu", "p2p.cu"]

SOURCES = [
    "bindings.cpp",
    "gemm_tc.cu",
    "topk.cu",
    "sparse.cu",
    "adam.cu",
    "noalloc_csc.cu",
    "p2p.cu",
    "symm.cpp",
    "lm_kernels.cu",
    "attention.cu",
    "mp.cu",
    "rows.cu",
]

NVCC_FLAGS = [
    "-gencode=arch=compute_100a,code=sm_100a",
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "--expt-extended-lambda",
    "-U__CUDA_NO_HALF_OPERATORS__",
    "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT162_OPERATORS__",
    "-U__CUDA_NO_BFLOAT162_CONVERSIONS__",
]


def _so_path(build_dir: str = BUILD_DIR, name: str = EXT_NAME) -> str | None:
    hits = sorted(glob.glob(os.path.join(build_dir, f"{name}*.so")))
    return hits[0] if hits else None


def _build_one(name: str, sources: list[str], build_dir: str, defines: list[str], verbose: bool) -> str:
    from torch.utils import cpp_extension

    os.makedirs(build_dir, exist_ok=True)
    # torch's own arch list must not add other targets: the flags above pin sm_100a.
    os.environ["TORCH_CUDA_ARCH_LIST"] = "10.0a"
    os.environ.setdefault("MAX_JOBS", str(max(1, (os.cpu_count() or 4))))
    cpp_extension.load(
        name=name,
        sources=[os.path.join(CSRC, s) for s in sources],
        extra_cflags=["-O3", "-std=c++17", *defines],
        extra_cuda_cflags=NVCC_FLAGS + defines,
        extra_include_paths=[CSRC],
        build_directory=build_dir,
        verbose=verbose,
        with_cuda=True,
        is_python_module=True,
    )
    path = _so_path(build_dir, name)
    if path is None:
        raise RuntimeError(f"extension build produced no .so in {build_dir}")
    return path


def build(verbose: bool = False, debug_bounds: bool = True) -> str:
    """Compile the extension (and, by default, the debug-bounds module) in-tree; returns the path
    of the main `.so`."""
    path = _build_one(EXT_NAME, SOURCES, BUILD_DIR, [], verbose)
    if debug_bounds:
        _build_one(DEBUG_EXT_NAME, DEBUG_SOURCES, DEBUG_BUILD_DIR, ["-DSB_DEBUG_BOUNDS=1"], verbose)
    return path


_MODULE: ModuleType | None = None
_DEBUG_MODULE: ModuleType | None = None


def _import_so(name: str, path: str) -> ModuleType:
    import torch  # noqa: F401  (the extension links against libtorch)

    spec = importlib.util.spec_from_file_location(name, path)
    assert spec is not None and spec.loader is not None
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    sys.modules[f"saelens_b200.ops.{name}"] = mod
    return mod


def load() -> ModuleType:
    """Import the prebuilt extension from the package directory."""
    global _MODULE
    if _MODULE is not None:
        return _MODULE
    path = _so_path()
    if path is None:
        raise ImportError(
            "saelens_b200 native extension is not built; run "
            "`python -c 'import __graft_entry__ as g; g.build()'` or "
            "`python -m saelens_b200.ops._build`"
        )
    _MODULE = _import_so(EXT_NAME, path)
    return _MODULE


def load_debug() -> ModuleType:
    """Import the prebuilt debug-bounds module (index-dereferencing kernels with bounds checks)."""
    global _DEBUG_MODULE
    if _DEBUG_MODULE is not None:
        return _DEBUG_MODULE
    path = _so_path(DEBUG_BUILD_DIR, DEBUG_EXT_NAME)
    if path is None:
        raise ImportError("saelens_b200 debug-bounds module is not built; run `python -m saelens_b200.ops._build`")
    _DEBUG_MODULE = _import_so(DEBUG_EXT_NAME, path)
    return _DEBUG_MODULE


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
