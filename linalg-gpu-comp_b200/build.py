"""Build recipe for libqrb200.so (sm_100a) -- the CUDA kernels and the C ABI.

``python build.py`` (or ``build()`` from Python) compiles every ``csrc/*.cu`` with
nvcc for ``sm_100a`` and links ``qr_b200/libqrb200.so`` in-tree, so the built
library travels with the source tree.  Objects are rebuilt only when a source or
header is newer than the library.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
INCLUDE = PKG.parent / "include"
OUT = PKG / "qr_b200" / "libqrb200.so"
OBJ = PKG / "_build"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr", f"-I{INCLUDE}", f"-I{CSRC}"]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; CUDA 12.8+ is required to build libqrb200")
    return cand


def _stale() -> bool:
    if not OUT.exists():
        return True
    t = OUT.stat().st_mtime
    srcs = list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h")) + [Path(__file__)]
    return any(s.stat().st_mtime > t for s in srcs)


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not _stale():
        return OUT
    nvcc = _nvcc()
    OBJ.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))

    def compile_one(src: Path) -> Path:
        obj = OBJ / (src.stem + ".o")
        cmd = [nvcc, *ARCH, *FLAGS, "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
        return obj

    with cf.ThreadPoolExecutor(max_workers=min(len(sources), os.cpu_count() or 4)) as ex:
        objs = list(ex.map(compile_one, sources))
    tmp = OUT.with_suffix(".so.tmp")
    cmd = [nvcc, *ARCH, "-shared", "-cudart", "static", *map(str, objs), "-o", str(tmp)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, OUT)
    return OUT


ENTRY_SRC = PKG / "qr_b200" / "_entry.cpp"


def _entry_out() -> Path:
    import sysconfig
    return PKG / "qr_b200" / ("_entry" + sysconfig.get_config_var("EXT_SUFFIX"))


def build_entry(force: bool = False, verbose: bool = False) -> Path:
    """Compile qr_b200/_entry.cpp (the torch-facing call path, pybind11) against the
    in-tree libqrb200.so, with rpath $ORIGIN so the pair travels together."""
    import sysconfig

    import torch
    import torch.utils.cpp_extension as ce

    out = _entry_out()
    deps = [ENTRY_SRC, OUT, INCLUDE / "qrb200.h", Path(__file__)]
    if not force and out.exists() and all(d.stat().st_mtime <= out.stat().st_mtime for d in deps):
        return out
    cxx = shutil.which("g++") or "c++"
    inc = [f"-I{p}" for p in ce.include_paths()] + [f"-I{sysconfig.get_paths()['include']}", f"-I{INCLUDE}",
                                                   "-I/usr/local/cuda/include"]
    libdirs = ce.library_paths()
    cmd = [cxx, "-O2", "-shared", "-fPIC", "-std=c++17", "-fvisibility=hidden",
           f"-D_GLIBCXX_USE_CXX11_ABI={int(torch._C._GLIBCXX_USE_CXX11_ABI)}",
           "-DTORCH_EXTENSION_NAME=_entry", "-DTORCH_API_INCLUDE_EXTENSION_H", *inc, str(ENTRY_SRC),
           "-o", str(out.with_suffix(".tmp")), *[f"-L{d}" for d in libdirs], f"-L{OUT.parent}",
           "-lqrb200", "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_python",
           "-Wl,-rpath,$ORIGIN", *[f"-Wl,-rpath,{d}" for d in libdirs]]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"g++ failed on {ENTRY_SRC.name}:\n{r.stdout}\n{r.stderr}")
    os.replace(out.with_suffix(".tmp"), out)
    return out


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
    print(build_entry(force="--force" in sys.argv, verbose=True))
