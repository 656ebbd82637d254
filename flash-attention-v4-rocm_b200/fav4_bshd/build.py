"""Build recipe for the in-tree CUDA libraries (sm_100a only).

    python -m fav4_bshd.build [--force]

Compiles csrc/fav4_bshd.cu -> build/libfav4_bshd.so (the C ABI of
include/fav4_bshd.h) and csrc/probe.cu -> build/libfav4_probe.so (test probes)
with nvcc for sm_100a, statically linked against the CUDA runtime. The ptxas
resource report (registers, spills, shared memory) of each build is written
next to the library as build/<lib>.ptxas.txt.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parents[1]
REPO_ROOT = PKG_ROOT.parent
CSRC = PKG_ROOT / "csrc"
INCLUDE = REPO_ROOT / "include"
BUILD = PKG_ROOT / "build"
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-shared", "-Xptxas", "-v",
          f"-I{INCLUDE}", f"-I{CSRC}"]
TARGETS = {
    "libfav4_bshd.so": ["fav4_bshd.cu"],
    "libfav4_probe.so": ["probe.cu"],
}


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _stale(out: Path, deps) -> bool:
    if not out.exists():
        return True
    t = out.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> list[Path]:
    BUILD.mkdir(parents=True, exist_ok=True)
    deps = list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))
    built = []
    for lib, srcs in TARGETS.items():
        out = BUILD / lib
        if force or _stale(out, deps):
            cmd = [nvcc(), *ARCH_FLAGS, *COMMON, "-o", str(out), *[str(CSRC / s) for s in srcs]]
            r = subprocess.run(cmd, capture_output=True, text=True)
            (BUILD / f"{lib}.ptxas.txt").write_text(r.stdout + r.stderr)
            if r.returncode != 0:
                sys.stderr.write(r.stdout + r.stderr)
                raise RuntimeError(f"nvcc failed for {lib}")
            if verbose:
                print(" ".join(cmd))
        built.append(out)
    return built


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    for p in build(force=a.force, verbose=True):
        print("built", p)


if __name__ == "__main__":
    main()
