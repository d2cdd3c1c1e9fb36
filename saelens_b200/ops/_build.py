"""Build and load the in-tree sm_100a extension (`saelens_b200/ops/_build/_C*.so`).

The extension is compiled once, in-tree, with `-gencode arch=compute_100a,code=sm_100a`
(nvcc cross-compiles without a GPU).  At import time on a CUDA machine the prebuilt `.so` is
loaded directly from the package directory; if it is missing the import fails loudly instead
of silently falling back to PyTorch ops.
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


def _so_path() -> str | None:
    hits = sorted(glob.glob(os.path.join(BUILD_DIR, f"{EXT_NAME}*.so")))
    return hits[0] if hits else None


def build(verbose: bool = False) -> str:
    """Compile the extension in-tree and return the path of the built `.so`."""
    from torch.utils import cpp_extension

    os.makedirs(BUILD_DIR, exist_ok=True)
    # torch's own arch list must not add other targets: the flags above pin sm_100a.
    os.environ["TORCH_CUDA_ARCH_LIST"] = "10.0a"
    os.environ.setdefault("MAX_JOBS", str(max(1, (os.cpu_count() or 4))))
    cpp_extension.load(
        name=EXT_NAME,
        sources=[os.path.join(CSRC, s) for s in SOURCES],
        extra_cflags=["-O3", "-std=c++17"],
        extra_cuda_cflags=NVCC_FLAGS,
        extra_include_paths=[CSRC],
        build_directory=BUILD_DIR,
        verbose=verbose,
        with_cuda=True,
        is_python_module=True,
    )
    path = _so_path()
    if path is None:
        raise RuntimeError(f"extension build produced no .so in {BUILD_DIR}")
    return path


_MODULE: ModuleType | None = None


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
    import torch  # noqa: F401  (the extension links against libtorch)

    spec = importlib.util.spec_from_file_location(EXT_NAME, path)
    assert spec is not None and spec.loader is not None
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    sys.modules[f"saelens_b200.ops.{EXT_NAME}"] = mod
    _MODULE = mod
    return mod


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
