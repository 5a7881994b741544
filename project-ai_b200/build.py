"""Build recipes for the native parts of the package.

* ``libprojectai_cuda.so`` — the sm_100a compute backend behind the C ABI in ``include/projectai_cuda.h``.
* ``_paihost`` — the C++ host runtime (tensor views, autograd tape, Llama modules, trainer) as a Python extension.

Everything is built in-tree so the shared objects travel with the repository snapshot. Objects are rebuilt only
when a source or header is newer than the object.
"""
from __future__ import annotations

import os
import subprocess
import sys
import sysconfig
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
HOST = PKG / "host"
INCLUDE = ROOT / "include"
BUILD = PKG / "_build"
LIB = PKG / "lib"
CUDA_LIB = LIB / "libprojectai_cuda.so"

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
# The system compiler: the image also exports CXX=/opt/gcc/bin/g++, which lacks parts of the runtime (libgomp).
CXX = "/usr/bin/g++"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
                     "--expt-relaxed-constexpr", f"-I{INCLUDE}", f"-I{CSRC}", "-ccbin", CXX]


def _newer(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"command failed ({r.returncode}): {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")


def nccl_lib_dir() -> Path | None:
    """The NCCL that PyTorch ships (the image also has an older system NCCL with the same soname). Linking against
    PyTorch's copy, with an rpath to it, keeps one NCCL in the process whichever of the two is loaded first."""
    import importlib.util

    spec = importlib.util.find_spec("nvidia")
    for base in (spec.submodule_search_locations or []) if spec else []:
        d = Path(base) / "nccl" / "lib"
        if (d / "libnccl.so.2").exists():
            return d
    return None


def build_cuda(verbose: bool = False) -> Path:
    """Compiles every ``csrc/*.cu`` for sm_100a and links ``lib/libprojectai_cuda.so``."""
    BUILD.mkdir(exist_ok=True)
    LIB.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    headers = sorted(CSRC.glob("*.cuh")) + [INCLUDE / "projectai_cuda.h"]
    jobs = []
    for src in sources:
        obj = BUILD / (src.stem + ".o")
        if _newer(obj, [src] + headers):
            jobs.append([NVCC, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)])
    if jobs:
        with ThreadPoolExecutor(max_workers=min(8, len(jobs))) as ex:
            list(ex.map(_run, jobs))
    objs = [BUILD / (s.stem + ".o") for s in sources]
    if _newer(CUDA_LIB, objs):
        nccl = nccl_lib_dir()
        link_nccl = ["-L" + str(nccl), "-l:libnccl.so.2", "-Xlinker", "-rpath," + str(nccl)] if nccl else ["-lnccl"]
        _run([NVCC, *ARCH, "-shared", "-ccbin", CXX, "-o", str(CUDA_LIB), *map(str, objs), *link_nccl,
              "-Xlinker", "--no-undefined"])
    if verbose:
        print(f"built {CUDA_LIB}")
    return CUDA_LIB


def host_module_path() -> Path:
    suffix = sysconfig.get_config_var("EXT_SUFFIX") or ".so"
    return PKG / f"_paihost{suffix}"


def build_host(verbose: bool = False) -> Path:
    """Compiles the C++ host runtime (``host/*.cpp``) into the ``_paihost`` Python extension."""
    import pybind11

    out = host_module_path()
    sources = sorted(HOST.glob("*.cpp"))
    headers = sorted(HOST.glob("*.h")) + [INCLUDE / "projectai_cuda.h"]
    if not sources:
        return out
    BUILD.mkdir(exist_ok=True)
    py_inc = sysconfig.get_paths()["include"]
    flags = ["-O2", "-std=c++17", "-fPIC", "-fvisibility=hidden", "-Wall", "-pthread", f"-I{INCLUDE}", f"-I{HOST}",
             f"-I{pybind11.get_include()}", f"-I{py_inc}"]
    jobs = []
    objs = []
    for src in sources:
        obj = BUILD / ("host_" + src.stem + ".o")
        objs.append(obj)
        if _newer(obj, [src] + headers):
            jobs.append([CXX, *flags, "-c", str(src), "-o", str(obj)])
    if jobs:
        with ThreadPoolExecutor(max_workers=min(8, len(jobs))) as ex:
            list(ex.map(_run, jobs))
    if _newer(out, objs):
        _run([CXX, "-shared", "-o", str(out), *map(str, objs), "-ldl"])
    if verbose:
        print(f"built {out}")
    return out


def build_all(verbose: bool = False) -> None:
    build_cuda(verbose)
    build_host(verbose)


if __name__ == "__main__":
    build_all(verbose=True)
    sys.exit(0)
