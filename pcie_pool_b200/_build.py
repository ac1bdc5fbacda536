"""In-tree build of the native core ``pcie_pool_b200._C``.

CUDA sources are compiled by nvcc for sm_100a only
(``-gencode arch=compute_100a,code=sm_100a``); host sources by g++.  The CUDA
runtime is linked statically and the driver is reached through
``cudaGetDriverEntryPointByVersion``, so the module builds and imports on a
machine without a GPU.  Objects are cached under ``_build/`` and rebuilt when
their source or any header in ``csrc/`` is newer.

The reference builds its ``_turbobus`` module through CMake without an
architecture list (cpp/CMakeLists.txt:1-45); this build pins the Blackwell
target explicitly.
"""

from __future__ import annotations

import os
import subprocess
import sys
import sysconfig
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
CSRC = PKG_DIR / "csrc"
BUILD_DIR = PKG_DIR / "_build"
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))

CU_SOURCES = ["ppb_common.cu", "pool_kernels.cu", "engine.cu", "native_ops.cu", "noalloc.cu", "vmm.cu"]
CC_SOURCES = ["planner.cc", "host_ops.cc", "bindings.cc", "bind_ops.cc"]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def extension_path() -> Path:
    suffix = sysconfig.get_config_var("EXT_SUFFIX") or ".so"
    return PKG_DIR / f"_C{suffix}"


def _includes() -> list[str]:
    import pybind11

    return [
        f"-I{CSRC}",
        f"-I{pybind11.get_include()}",
        f"-I{sysconfig.get_paths()['include']}",
        f"-I{CUDA_HOME / 'include'}",
    ]


def _newest_header() -> float:
    heads = list(CSRC.glob("*.h")) + list(CSRC.glob("*.cuh"))
    return max((p.stat().st_mtime for p in heads), default=0.0)


def _stale(src: Path, obj: Path, head_mtime: float) -> bool:
    if not obj.exists():
        return True
    m = obj.stat().st_mtime
    return m < src.stat().st_mtime or m < head_mtime


def _compile(cmd: list[str]) -> None:
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(
            "native build failed:\n" + " ".join(cmd) + "\n" + res.stdout + res.stderr
        )


def build(force: bool = False, verbose: bool = False, jobs: int | None = None) -> Path:
    """Compile (if needed) and link ``_C``; returns the extension path."""
    BUILD_DIR.mkdir(exist_ok=True)
    nvcc = str(CUDA_HOME / "bin" / "nvcc")
    inc = _includes()
    head = _newest_header()
    cmds: list[list[str]] = []
    objs: list[Path] = []
    for name in CU_SOURCES:
        src = CSRC / name
        obj = BUILD_DIR / (name + ".o")
        objs.append(obj)
        if force or _stale(src, obj, head):
            cmds.append(
                [nvcc, *ARCH_FLAGS, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC",
                 "-Xcompiler", "-fvisibility=hidden", *inc, "-c", str(src), "-o", str(obj)]
            )
    for name in CC_SOURCES:
        src = CSRC / name
        obj = BUILD_DIR / (name + ".o")
        objs.append(obj)
        if force or _stale(src, obj, head):
            cmds.append(
                ["g++", "-O2", "-std=c++17", "-fPIC", "-fvisibility=hidden", *inc, "-c", str(src),
                 "-o", str(obj)]
            )
    if cmds:
        with ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 4)) as pool:
            list(pool.map(_compile, cmds))
    out = extension_path()
    if force or cmds or not out.exists():
        link = ["g++", "-shared", "-o", str(out), *map(str, objs),
                f"-L{CUDA_HOME / 'lib64'}", "-lcudart_static", "-lrt", "-lpthread", "-ldl"]
        _compile(link)
    if verbose:
        print(f"built {out}")
    return out


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
