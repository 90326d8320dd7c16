"""Build libgko_b200.so (all CUDA kernels + the C ABI) in-tree with nvcc for sm_100a.

Usage: python -m evocompile_b200.build [--force]
The library lands next to this file so that it travels with the source tree.
"""

from __future__ import annotations

import hashlib
import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
REPO = PKG.parent
LIB = PKG / "libgko_b200.so"
BUILD_DIR = REPO / "_build"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC",
              "-Xptxas", "-warn-spills"]


def nvcc() -> str:
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    return str(Path(cuda) / "bin" / "nvcc")


def sources() -> list[Path]:
    return sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cpp")))


def _digest() -> str:
    h = hashlib.sha256()
    for p in sorted(list(CSRC.glob("*")) + [REPO / "include" / "gko_b200.h"]):
        if p.is_file():
            h.update(p.name.encode())
            h.update(p.read_bytes())
    h.update(" ".join(ARCH + NVCC_FLAGS).encode())
    return h.hexdigest()[:16]


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile every translation unit under csrc/ and link libgko_b200.so. Returns its path."""
    stamp = PKG / ".libgko_b200.stamp"
    digest = _digest()
    if LIB.exists() and stamp.exists() and stamp.read_text().strip() == digest and not force:
        return LIB
    BUILD_DIR.mkdir(exist_ok=True)
    objs = []
    procs = []
    for src in sources():
        obj = BUILD_DIR / (src.name + ".o")
        cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-I", str(REPO / "include"), "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)))
        objs.append(obj)
    failed = []
    for src, pr in procs:
        out, _ = pr.communicate()
        text = out.decode(errors="replace")
        if pr.returncode != 0:
            failed.append(f"--- {src.name}\n{text}")
        elif verbose and text.strip():
            print(text)
    if failed:
        raise RuntimeError("nvcc failed:\n" + "\n".join(failed))
    tmp = LIB.with_suffix(".so.tmp")
    link = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-lcudart", "-lcuda"]
    # libcuda is resolved at run time from the driver; link against the stub when present.
    stub = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda")) / "lib64" / "stubs"
    if stub.is_dir():
        link[-1:-1] = ["-L", str(stub)]
    r = subprocess.run(link, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("link failed:\n" + r.stdout + r.stderr)
    os.replace(tmp, LIB)
    stamp.write_text(digest)
    return LIB


if __name__ == "__main__":
    p = build(force="--force" in sys.argv, verbose=True)
    print(p)
