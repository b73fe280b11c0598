"""In-tree build of the native parts of femtovllm_b200.

Produces, next to this file:

* ``libfemtovllm_b200.so`` - every CUDA kernel plus the ``extern "C"`` ABI of
  ``include/femtovllm_b200.h``, compiled by nvcc for sm_100a only
  (``-gencode arch=compute_100a,code=sm_100a``), cudart linked statically;
* ``_C.so`` - the PyTorch extension (``csrc/torch_ext.cpp``) that mirrors the
  reference's ``femtovllm._C`` and calls the C ABI; linked against
  ``libfemtovllm_b200.so`` with an ``$ORIGIN`` rpath.

Run ``python -m femtovllm_b200._build`` (from ``nano-vllm-practice_b200/``) or
``__graft_entry__.build()``.  Objects go to ``nano-vllm-practice_b200/_build/``;
a source is recompiled only when it or a header is newer than its object.
"""

from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
import sysconfig
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
ROOT = PKG_DIR.parent  # nano-vllm-practice_b200/
REPO = ROOT.parent
CSRC = ROOT / "csrc"
INCLUDE = REPO / "include"
BUILD = ROOT / "_build"
LIB = PKG_DIR / "libfemtovllm_b200.so"
EXT = PKG_DIR / "_C.so"

CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = str(CUDA_HOME / "bin" / "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    f"-I{INCLUDE}",
    f"-I{CSRC}",
]
CU_SOURCES = [
    "capi.cu",
    "store_kvcache.cu",
    "qk_norm_rope.cu",
    "metadata.cu",
    "sampler.cu",
    "decode.cu",
    "decode_noalloc.cu",
    "prefill_simt.cu",
    "prefill_sm100.cu",
]


def _headers() -> list[Path]:
    return sorted(list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h")))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _run(cmd: list[str], verbose: bool) -> None:
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"build step failed ({res.returncode}):\n{' '.join(cmd)}\n{res.stdout}")
    if verbose and res.stdout.strip():
        print(res.stdout, flush=True)


def build_lib(verbose: bool = False, jobs: int | None = None) -> Path:
    """Compile the CUDA sources and link libfemtovllm_b200.so."""
    BUILD.mkdir(exist_ok=True)
    headers = _headers()
    sources = [s for s in CU_SOURCES if (CSRC / s).exists()]
    objs = []
    todo = []
    for s in sources:
        obj = BUILD / (Path(s).stem + ".o")
        objs.append(obj)
        if _stale(obj, [CSRC / s] + headers):
            todo.append([NVCC, *NVCC_FLAGS, "-c", str(CSRC / s), "-o", str(obj)])
    with cf.ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 4)) as ex:
        list(ex.map(lambda c: _run(c, verbose), todo))
    if todo or _stale(LIB, objs):
        tmp = BUILD / LIB.name
        _run([NVCC, *ARCH, "-shared", "-Xcompiler", "-fPIC", *map(str, objs), "-o", str(tmp)], verbose)
        shutil.copy2(tmp, LIB)
    return LIB


def build_ext(verbose: bool = False) -> Path:
    """Compile csrc/torch_ext.cpp into _C.so against the installed PyTorch."""
    import torch
    from torch.utils import cpp_extension

    src = CSRC / "torch_ext.cpp"
    deps = [src, LIB, INCLUDE / "femtovllm_b200.h", Path(__file__)]
    if not _stale(EXT, deps):
        return EXT
    BUILD.mkdir(exist_ok=True)
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    incs = [f"-I{p}" for p in cpp_extension.include_paths(device_type="cuda")]
    incs += [f"-I{sysconfig.get_paths()['include']}", f"-I{INCLUDE}", f"-I{CUDA_HOME / 'include'}"]
    libdirs = [f"-L{p}" for p in cpp_extension.library_paths(device_type="cuda")]
    tmp = BUILD / "_C.so"
    cmd = [
        "g++",
        "-O2",
        "-std=c++17",
        "-fPIC",
        "-shared",
        f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
        "-DTORCH_EXTENSION_NAME=_C",
        "-DTORCH_API_INCLUDE_EXTENSION_H",
        *incs,
        str(src),
        "-o",
        str(tmp),
        *libdirs,
        f"-L{PKG_DIR}",
        "-lfemtovllm_b200",
        "-lc10",
        "-lc10_cuda",
        "-ltorch",
        "-ltorch_cpu",
        "-ltorch_cuda",
        "-ltorch_python",
        "-Wl,-rpath,$ORIGIN",
        *[f"-Wl,-rpath,{p}" for p in cpp_extension.library_paths(device_type="cuda")],
    ]
    _run(cmd, verbose)
    shutil.copy2(tmp, EXT)
    return EXT


def build(verbose: bool = False) -> None:
    build_lib(verbose)
    build_ext(verbose)


if __name__ == "__main__":
    build(verbose="-v" in sys.argv)
    print(f"built {LIB} and {EXT}")
