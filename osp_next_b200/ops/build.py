"""Build the in-tree sm_100a extension ``osp_next_b200/ops/_C.so``.

``python -m osp_next_b200.ops.build`` compiles every ``csrc/*.cu|cpp`` with
``nvcc -gencode arch=compute_100a,code=sm_100a -lineinfo`` through
``torch.utils.cpp_extension`` (ninja, incremental) into ``_build/ops`` at the
repository root and copies the module next to this file, so the built library
travels with the source tree.  No GPU is needed to build.
"""
from __future__ import annotations

import glob
import os
import shutil
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
CUDA_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "--expt-relaxed-constexpr", "-std=c++17",
    "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_BFLOAT16_CONVERSIONS__", "-U__CUDA_NO_HALF2_OPERATORS__",
]


def sources():
    return sorted(glob.glob(os.path.join(HERE, "csrc", "*.cu")) + glob.glob(os.path.join(HERE, "csrc", "*.cpp")))


def build(verbose: bool = False) -> str:
    os.environ["TORCH_CUDA_ARCH_LIST"] = "10.0a"
    os.environ.setdefault("MAX_JOBS", str(min(16, os.cpu_count() or 4)))
    from torch.utils import cpp_extension
    bdir = os.path.join(ROOT, "_build", "ops")
    os.makedirs(bdir, exist_ok=True)
    cpp_extension.load(
        name="_C",
        sources=sources(),
        extra_cflags=["-O3", "-std=c++17"],
        extra_cuda_cflags=CUDA_FLAGS + (["-Xptxas", "-v"] if verbose else []),
        extra_include_paths=[os.path.join(HERE, "csrc")],
        build_directory=bdir,
        verbose=verbose,
        is_python_module=True,
    )
    src = os.path.join(bdir, "_C.so")
    dst = os.path.join(HERE, "_C.so")
    shutil.copy2(src, dst + ".tmp")
    os.replace(dst + ".tmp", dst)
    return dst


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
