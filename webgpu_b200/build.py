"""In-tree native build: the CUDA decoder library (sm_100a), the synthetic-weight
generator, and the CPU oracle used by the tests.

    python -m webgpu_b200.build            # everything
    python -m webgpu_b200.build --cuda     # only libwgd.so

Outputs stay inside the repository (webgpu_b200/_build/, oracle/_build/) so they
travel with the source tree to the GPU machine.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

from ._build_paths import BUILD_DIR, PACKAGE_DIR, REPO_DIR, synth_lib_path, wgd_lib_path

CSRC = os.path.join(PACKAGE_DIR, "csrc")
NVCC = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
                     "--expt-relaxed-constexpr", "-I", os.path.join(REPO_DIR, "include")]


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError(f"build step failed: {' '.join(cmd[:3])} ...")


def _stale(target: str, sources: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(s) > t for s in sources)


def build_cuda(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(os.path.join(BUILD_DIR, "obj"), exist_ok=True)
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    headers = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + [os.path.join(REPO_DIR, "include", "wgd.h")]
    objs, jobs = [], []
    for src in sources:
        obj = os.path.join(BUILD_DIR, "obj", os.path.basename(src) + ".o")
        objs.append(obj)
        if force or _stale(obj, [src] + headers):
            cmd = [NVCC, *NVCC_FLAGS, "-c", src, "-o", obj]
            if verbose:
                cmd.insert(1, "-Xptxas=-v")
            jobs.append(cmd)
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
            list(ex.map(_run, jobs))
    lib = wgd_lib_path()
    if force or jobs or _stale(lib, objs):
        _run([NVCC, *ARCH, "-shared", "-o", lib, *objs, "-lcudart"])
    return lib


def build_synth(force: bool = False) -> str:
    os.makedirs(BUILD_DIR, exist_ok=True)
    src = os.path.join(PACKAGE_DIR, "synth", "quantize.c")
    out = synth_lib_path()
    if force or _stale(out, [src]):
        _run(["gcc", "-O2", "-fopenmp", "-fPIC", "-shared", "-std=gnu11", "-o", out, src, "-lm"])
    return out


def build_oracle(force: bool = False) -> str:
    src = os.path.join(REPO_DIR, "oracle", "oracle.c")
    out = os.path.join(REPO_DIR, "oracle", "_build", "liboracle.so")
    if force or _stale(out, [src]):
        _run(["make", "-s", "-C", os.path.join(REPO_DIR, "oracle"), "CC=gcc"] + (["-B"] if force else []))
    return out


def build_all(force: bool = False) -> None:
    build_synth(force)
    build_oracle(force)
    build_cuda(force)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--cuda", action="store_true")
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    if a.cuda:
        print(build_cuda(a.force, a.verbose))
    else:
        build_all(a.force)
        print("built", wgd_lib_path())


if __name__ == "__main__":
    main()
