"""Build libd3b200.so (the C-ABI CUDA library) in-tree for sm_100a.

    python -m drama3_offloading_b200.build [--verbose]

Compiles every ``csrc/*.cu`` with nvcc for ``-gencode arch=compute_100a,code=sm_100a``
into ``drama3_offloading_b200/libd3b200.so`` (static cudart, so the library does not
depend on which libcudart torch loads).  ``-Xptxas -v`` resource usage is written
next to it as ``libd3b200.ptxas.txt``.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
LIB = PKG / "libd3b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("CUDA_HOME", ""), "/usr/local/cuda"):
        p = Path(cand) / "bin" / "nvcc"
        if cand and p.exists():
            return str(p)
    found = shutil.which("nvcc")
    if not found:
        raise RuntimeError("nvcc not found (set CUDA_HOME)")
    return found


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    t = LIB.stat().st_mtime
    deps = list(CSRC.glob("*")) + [PKG.parent / "include" / "d3b200.h", Path(__file__)]
    return all(d.stat().st_mtime <= t for d in deps if d.exists())


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and up_to_date():
        return LIB
    srcs = [str(s) for s in sources()]
    cmd = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC",
           "-Xcompiler", "-fvisibility=hidden", "-cudart", "static", "-Xptxas", "-v",
           "-I", str(PKG.parent / "include"), "-o", str(LIB) + ".tmp", *srcs]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError(f"nvcc failed building {LIB.name} (exit {r.returncode})")
    os.replace(str(LIB) + ".tmp", LIB)
    (PKG / "libd3b200.ptxas.txt").write_text(r.stderr)
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))


if __name__ == "__main__":
    main()
