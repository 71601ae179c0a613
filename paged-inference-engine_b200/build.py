"""Build recipe for libpaged_attn_b200.so (sm_100a only) and its torch extension.

Compiles every ``csrc/*.cu`` with nvcc for ``-gencode arch=compute_100a,code=sm_100a``
in parallel and links them into ``pie_b200/libpaged_attn_b200.so`` next to the
Python bindings, so the library travels with the source tree.  Then compiles
``csrc/torch_ops.cpp`` (the torch.library registration of the C ABI) against
torch's headers into ``pie_b200/_pie_b200_torch.so``, linked to the library
through ``$ORIGIN``.  Incremental: a translation unit is rebuilt only when it or
a header is newer than its output.

Usage:  python build.py [--verbose] [--ptxas-info]
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
OUT_DIR = os.path.join(HERE, "pie_b200")
OBJ_DIR = os.path.join(HERE, "_build")
LIB_NAME = "libpaged_attn_b200.so"
EXT_NAME = "_pie_b200_torch.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libpaged_attn_b200.so")
    return cand


def _headers() -> list[str]:
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    hs += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith(".h")]
    return hs


def _compile(nvcc: str, src: str, obj: str, ptxas_info: bool) -> tuple[str, str]:
    cmd = [nvcc, *ARCH, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
           "-I", CSRC, "-I", INCLUDE, "-c", src, "-o", obj]
    if ptxas_info:
        cmd.insert(1, "-Xptxas=-v")
    extra = os.environ.get("PIE_B200_NVCC_FLAGS", "").split()
    cmd[1:1] = extra
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {os.path.basename(src)}:\n{r.stdout}\n{r.stderr}")
    return src, r.stdout + r.stderr


def build_torch_ext(lib: str, force: bool = False, verbose: bool = False) -> str:
    """g++ of csrc/torch_ops.cpp against torch (its headers and libraries) and the C-ABI library."""
    import torch
    import torch.utils.cpp_extension as ce

    src = os.path.join(CSRC, "torch_ops.cpp")
    out = os.path.join(OUT_DIR, EXT_NAME)
    newest = max([os.path.getmtime(src), os.path.getmtime(lib)] + [os.path.getmtime(h) for h in _headers()])
    if not force and os.path.exists(out) and os.path.getmtime(out) >= newest:
        return out
    cxx = shutil.which("g++") or "c++"
    incs = []
    for d in ce.include_paths(device_type="cuda") + [INCLUDE]:
        incs += ["-isystem" if d != INCLUDE else "-I", d]
    libdirs = [x for d in ce.library_paths(device_type="cuda") for x in ("-L", d)]
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = [cxx, "-O2", "-std=c++17", "-fPIC", "-shared", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           "-DTORCH_EXTENSION_NAME=_pie_b200_torch", *incs, src, "-o", out + ".tmp", "-L", OUT_DIR,
           "-lpaged_attn_b200", *libdirs, "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda",
           "-Wl,-rpath,$ORIGIN"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"g++ failed for torch_ops.cpp:\n{r.stdout}\n{r.stderr}")
    if verbose:
        print(f"[g++] torch_ops.cpp\n{r.stdout}{r.stderr}", file=sys.stderr)
    os.replace(out + ".tmp", out)
    return out


def build(verbose: bool = False, ptxas_info: bool = False, force: bool = False) -> str:
    """Compile (if stale) and link the library and the torch extension; returns the library's path."""
    nvcc = nvcc_path()
    os.makedirs(OBJ_DIR, exist_ok=True)
    srcs = sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))
    newest_header = max((os.path.getmtime(h) for h in _headers()), default=0.0)
    jobs = []
    objs = []
    for s in srcs:
        o = os.path.join(OBJ_DIR, os.path.basename(s)[:-3] + ".o")
        objs.append(o)
        stale = force or ptxas_info or bool(os.environ.get("PIE_B200_NVCC_FLAGS")) or not os.path.exists(o) or os.path.getmtime(o) < max(os.path.getmtime(s),
                                                                                           newest_header)
        if stale:
            jobs.append((s, o))
    lib = os.path.join(OUT_DIR, LIB_NAME)
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as ex:
            futs = [ex.submit(_compile, nvcc, s, o, ptxas_info) for s, o in jobs]
            for f in futs:
                src, log = f.result()
                if verbose or ptxas_info:
                    print(f"[nvcc] {os.path.basename(src)}\n{log}", file=sys.stderr)
    if jobs or not os.path.exists(lib):
        tmp = lib + ".tmp"
        cmd = [nvcc, *ARCH, "-shared", "-o", tmp, *objs, "-lcudart"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, lib)
    build_torch_ext(lib, force=force, verbose=verbose)
    return lib


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(verbose=a.verbose, ptxas_info=a.ptxas_info, force=a.force))
