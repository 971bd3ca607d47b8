"""Builds libtsugumi_cuda.so in-tree for sm_100a.

Each .cu file under csrc/ is compiled with nvcc into csrc/../_build/*.o and
linked into tsugumi_b200/libtsugumi_cuda.so.  The CUDA runtime is linked
statically; the driver API (tensor-map encoding) is reached through
cudaGetDriverEntryPoint, so the library has no link-time dependency on
libcuda.  Run as ``python -m tsugumi_b200.build`` or through
``__graft_entry__.build()``.
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
BUILD = PKG / "_build"
LIB = PKG / "libtsugumi_cuda.so"
INCLUDE = PKG.parent / "include"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH_FLAGS + [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    f"-I{INCLUDE}",
]


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(path).exists():
        raise RuntimeError("nvcc not found")
    return path


def _defines() -> list[str]:
    """Extra -D flags from TSG_NVCC_DEFINES (an instrumentation build, e.g.
    "-DTSG_PHASE_STAMPS=1"); empty for the product."""
    return [d for d in os.environ.get("TSG_NVCC_DEFINES", "").split() if d.startswith("-D")]


def _compile(src: Path, verbose_ptxas: bool) -> Path:
    obj = BUILD / (src.stem + ".o")
    deps = [src] + sorted(CSRC.glob("*.cuh")) + [INCLUDE / "tsugumi_cuda.h"]
    stamp = BUILD / (src.stem + ".defines")
    defines = _defines()
    same_defines = stamp.exists() and stamp.read_text() == " ".join(defines)
    if (obj.exists() and same_defines and
            all(obj.stat().st_mtime >= d.stat().st_mtime for d in deps)):
        return obj
    cmd = [nvcc(), *NVCC_FLAGS, *defines, "-c", str(src), "-o", str(obj)]
    if verbose_ptxas:
        cmd += ["-Xptxas", "-v"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stderr}")
    stamp.write_text(" ".join(defines))
    if verbose_ptxas:
        sys.stderr.write(res.stderr)
    return obj


def build(verbose_ptxas: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose_ptxas), sources))
    newest = max(o.stat().st_mtime for o in objs)
    if LIB.exists() and LIB.stat().st_mtime >= newest:
        return LIB
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objs)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(verbose_ptxas="-v" in sys.argv))
