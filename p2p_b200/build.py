"""Build recipe for libp2pattn.so (sm_100a only).

    python p2p_b200/build.py [--verbose-ptxas]

Compiles every p2p_b200/csrc/*.cu with nvcc for `arch=compute_100a,code=sm_100a` into
p2p_b200/_build/*.o (in parallel) and links p2p_b200/libp2pattn.so in-tree, with the CUDA
runtime linked statically so the library only needs the driver at run time; then builds the
plain C host program p2p_b200/host/p2p_decode_loop against it.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libp2pattn.so"
INCLUDE = PKG.parent / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC,-fvisibility=hidden", "-I", str(INCLUDE), "-I", str(CSRC),
    "-DP2P_BUILD_LIB",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise FileNotFoundError("nvcc not found")


def _compile(src: Path, verbose_ptxas: bool) -> tuple[Path, str]:
    obj = BUILD / (src.stem + ".o")
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    if verbose_ptxas:
        cmd += ["-Xptxas", "-v"]
    deps = [src, *CSRC.glob("*.cuh"), *CSRC.glob("*.h"), *INCLUDE.glob("*.h")]
    if not verbose_ptxas and obj.exists() and obj.stat().st_mtime > max(d.stat().st_mtime for d in deps):
        return obj, ""
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
    return obj, r.stdout + r.stderr


def build(verbose_ptxas: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        results = list(ex.map(lambda s: _compile(s, verbose_ptxas), srcs))
    for _, log in results:
        if log.strip():
            sys.stderr.write(log)
    objs = [o for o, _ in results]
    newest = max(o.stat().st_mtime for o in objs)
    if not LIB.exists() or LIB.stat().st_mtime < newest:
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs),
               "-ldl"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        tmp.replace(LIB)
    build_host_loop()
    return LIB


HOST_SRC = PKG / "host" / "decode_loop.c"
HOST_BIN = PKG / "host" / "p2p_decode_loop"


def build_host_loop() -> Path:
    """The plain C host program that drives the decode step through the C ABI (no Python):
    the end-to-end leg of bench.py runs it.  CUDA runtime linked statically, the library found
    beside it through the run path."""
    deps = [HOST_SRC, LIB, *INCLUDE.glob("*.h")]
    if HOST_BIN.exists() and HOST_BIN.stat().st_mtime > max(d.stat().st_mtime for d in deps):
        return HOST_BIN
    cuda = Path(nvcc()).resolve().parent.parent
    cmd = ["gcc", "-O2", "-std=c11", "-Wall", "-Wextra", "-I", str(INCLUDE),
           "-I", str(cuda / "include"), str(HOST_SRC), "-o", str(HOST_BIN),
           "-L", str(PKG), "-lp2pattn", "-L", str(cuda / "lib64"), "-lcudart_static",
           "-lpthread", "-ldl", "-lrt", "-lm", "-Wl,-rpath,$ORIGIN/.."]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"host program build failed:\n{r.stdout}\n{r.stderr}")
    return HOST_BIN


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose-ptxas", action="store_true")
    args = ap.parse_args()
    print(build(args.verbose_ptxas))
