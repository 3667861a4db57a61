"""Build the in-tree shared libraries of the paged KV-cache path.

* ``lib/libvasr_pa.so``  — the sm_100a CUDA kernels behind the C ABI of
  ``include/vasr_pa.h`` (nvcc, ``-gencode arch=compute_100a,code=sm_100a``,
  static cudart so the library has no runtime dependency besides the driver).
* ``lib/_vasr_host*.so`` — the C++ host mirror of the ``vasr-paged-attn``
  Rust API (metadata builders, block manager, graph buckets) as a pybind11
  module, used by the Python package and the tests.

Objects go to ``_build/``; each unit is rebuilt only when it or a header it
may include is newer than its object. Run ``python build.py`` or call
``build()``.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
import sysconfig
from pathlib import Path

PKG = Path(__file__).resolve().parent
REPO = PKG.parent
CSRC = PKG / "csrc"
HOST = CSRC / "host"
OBJ = PKG / "_build"
LIB = PKG / "lib"
INCLUDE = REPO / "include"

NVCC = os.environ.get("NVCC", shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc")
CUDA_HOME = Path(NVCC).resolve().parent.parent
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CUDA_UNITS = ["kv_ops.cu", "decode.cu", "prefill.cu", "capi.cu", "decode_noalloc.cu",
              "fused_rope.cu", "prefill_umma.cu", "decode_loop.cu"]
NVCC_FLAGS = ARCH + [
    "-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-O3",
    "--expt-relaxed-constexpr", "-I", str(INCLUDE),
]


def _newest_header_mtime() -> float:
    hdrs = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))
    hdrs += list(INCLUDE.glob("*.hpp")) + list(HOST.glob("*.hpp"))
    return max((h.stat().st_mtime for h in hdrs), default=0.0)


def _stale(target: Path, sources: list[Path], hdr_mtime: float) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(s.stat().st_mtime > t for s in sources) or hdr_mtime > t


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"command failed ({r.returncode}): {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")


def build_cuda(verbose: bool = False) -> Path:
    """Compile the CUDA units and link ``lib/libvasr_pa.so``."""
    OBJ.mkdir(exist_ok=True)
    LIB.mkdir(exist_ok=True)
    hdr = _newest_header_mtime()
    jobs = []
    for unit in CUDA_UNITS:
        src = CSRC / unit
        obj = OBJ / (src.stem + ".o")
        if _stale(obj, [src], hdr):
            cmd = [NVCC, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
            if verbose:
                cmd.insert(1, "-Xptxas=-v")
            jobs.append(cmd)
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        for f in [ex.submit(_run, j) for j in jobs]:
            f.result()
    out = LIB / "libvasr_pa.so"
    objs = [OBJ / (Path(u).stem + ".o") for u in CUDA_UNITS]
    if jobs or _stale(out, objs, 0.0):
        _run([NVCC, *ARCH, "-shared", "-Xcompiler", "-fPIC", *map(str, objs), "-o", str(out)])
    return out


def build_host() -> Path | None:
    """Compile the pybind11 module of the C++ host mirror (if its sources exist)."""
    srcs = sorted(HOST.glob("*.cpp")) if HOST.exists() else []
    if not srcs:
        return None
    import pybind11  # noqa: PLC0415

    LIB.mkdir(exist_ok=True)
    suffix = sysconfig.get_config_var("EXT_SUFFIX") or ".so"
    out = LIB / f"_vasr_host{suffix}"
    hdr = _newest_header_mtime()
    if not _stale(out, srcs, hdr):
        return out
    # The system g++ (the image's $CXX points at a toolchain without the
    # full runtime); static cudart like libvasr_pa.so; rpath to lib/.
    cmd = [
        shutil.which("g++") or "g++", "-O2", "-std=c++17", "-shared", "-fPIC", "-Wall",
        "-fvisibility=hidden",
        "-I", str(INCLUDE), "-I", str(HOST), "-I", pybind11.get_include(),
        "-I", sysconfig.get_paths()["include"], "-I", str(CUDA_HOME / "include"),
        *map(str, srcs), "-o", str(out),
        "-L", str(LIB), "-lvasr_pa", "-Wl,-rpath,$ORIGIN",
        str(CUDA_HOME / "lib64" / "libcudart_static.a"), "-ldl", "-lpthread", "-lrt",
    ]
    _run(cmd)
    return out


def build(verbose: bool = False) -> None:
    build_cuda(verbose=verbose)
    build_host()


if __name__ == "__main__":
    build(verbose="-v" in sys.argv)
    print("built:", *sorted(p.name for p in LIB.glob("*.so")))
