"""Build liblr_w8a8.so, the sm_100a C-ABI library of the W8A8 projection path.

The library is built in-tree (next to this file) so that it travels with the
source tree; there is no JIT cache. Usage: ``python -m lynnreal_omni_b200.build``.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
CSRC = PACKAGE / "csrc"
INCLUDE = PACKAGE.parent / "include"
LIBRARY = PACKAGE / "liblr_w8a8.so"
SOURCES = ["lr_host.cu", "lr_elementwise.cu", "lr_gemm_sm100.cu", "lr_flash.cu", "lr_attention.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3", "--expt-relaxed-constexpr",
         "-Xptxas", "-O3"]


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(path).exists():
        raise RuntimeError("nvcc not found: the sm_100a library cannot be built")
    return path


def _stale() -> bool:
    if not LIBRARY.exists():
        return True
    built = LIBRARY.stat().st_mtime
    deps = list(CSRC.glob("*")) + list(INCLUDE.glob("*.h")) + [Path(__file__)]
    return any(p.stat().st_mtime > built for p in deps)


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> Path:
    """Compile every CUDA source into the shared library (skipped if up to date)."""
    if not force and not ptxas_info and not _stale():
        return LIBRARY
    objs = []
    build_dir = PACKAGE / "_build"
    build_dir.mkdir(exist_ok=True)
    procs = []
    for src in SOURCES:
        obj = build_dir / (Path(src).stem + ".o")
        cmd = [nvcc(), *ARCH, *FLAGS, "-I", str(INCLUDE), "-c", str(CSRC / src), "-o", str(obj)]
        if ptxas_info:
            cmd += ["-Xptxas", "-v"]
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT,
                                            text=True)))
        objs.append(str(obj))
    failed = []
    for src, proc in procs:
        out, _ = proc.communicate()
        if verbose or ptxas_info or proc.returncode:
            sys.stdout.write(out)
        if proc.returncode:
            failed.append(src)
    if failed:
        raise RuntimeError("nvcc failed for: " + ", ".join(failed))
    tmp = LIBRARY.with_suffix(f".so.{os.getpid()}.tmp")
    link = [nvcc(), *ARCH, "-shared", "-Xcompiler", "-fPIC", *objs, "-o", str(tmp), "-lcuda"
            if False else "-lcudart_static"]
    subprocess.run(link, check=True)
    tmp.replace(LIBRARY)
    return LIBRARY


if __name__ == "__main__":
    path = build(force="--force" in sys.argv, verbose=True, ptxas_info="--ptxas" in sys.argv)
    print(path)
