"""Build libparis_moe.so in-tree with nvcc for sm_100a (no JIT cache).

    python paris-hackathon-2026-inference_b200/build.py [--verbose-ptxas]

libparis_moe.so has no torch dependency: it exports the C ABI of
include/paris_moe.h and is loaded with ctypes.  libparis_moe_torch.so
(csrc/torch_ops.cpp, g++ against the installed torch's headers) registers the
torch.ops.paris_moe operators over that ABI.
"""
from __future__ import annotations

import argparse
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
LIB = os.path.join(PKG, "libparis_moe.so")
OPS_LIB = os.path.join(PKG, "libparis_moe_torch.so")
OPS_SRC = os.path.join(CSRC, "torch_ops.cpp")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def headers():
    return sorted(glob.glob(os.path.join(CSRC, "*.cuh"))) + [
        os.path.join(ROOT, "include", "paris_moe.h")]


def needs_build() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    return any(os.path.getmtime(f) > t for f in sources() + headers())


def build(force: bool = False, verbose_ptxas: bool = False, jobs: int | None = None) -> str:
    build_lib(force, verbose_ptxas)
    build_ops(force)
    return LIB


def build_ops(force: bool = False) -> str:
    """The torch operator library, linked against libparis_moe.so and torch."""
    if (not force and os.path.exists(OPS_LIB) and
            os.path.getmtime(OPS_LIB) > max(os.path.getmtime(f) for f in
                                            [OPS_SRC, LIB, *headers()])):
        return OPS_LIB
    import torch
    from torch.utils import cpp_extension
    cuda_home = os.path.dirname(os.path.dirname(nvcc_path()))
    inc = cpp_extension.include_paths() + [os.path.join(cuda_home, "include"),
                                           os.path.join(ROOT, "include")]
    torch_lib = os.path.join(os.path.dirname(torch.__file__), "lib")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    tmp = OPS_LIB + ".tmp"
    cmd = (["g++", "-O2", "-std=c++17", "-fPIC", "-shared", f"-D_GLIBCXX_USE_CXX11_ABI={abi}"] +
           [f"-I{d}" for d in inc] + [OPS_SRC, "-o", tmp, f"-L{PKG}", "-lparis_moe",
                                      f"-L{torch_lib}", "-lc10", "-lc10_cuda", "-ltorch_cpu",
                                      "-ltorch", "-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{torch_lib}"])
    subprocess.check_call(cmd)
    os.replace(tmp, OPS_LIB)
    return OPS_LIB


def build_lib(force: bool = False, verbose_ptxas: bool = False) -> str:
    if not force and not needs_build():
        return LIB
    nvcc = nvcc_path()
    objdir = os.path.join(PKG, "_build")
    os.makedirs(objdir, exist_ok=True)
    common = [nvcc, "-O3", "-std=c++17", *ARCH, "-lineinfo", "-Xcompiler", "-fPIC",
              "-I", os.path.join(ROOT, "include"), "--expt-relaxed-constexpr"]
    if verbose_ptxas:
        common += ["-Xptxas", "-v"]
    objs = []
    procs = []
    for src in sources():
        obj = os.path.join(objdir, os.path.basename(src) + ".o")
        objs.append(obj)
        procs.append((src, subprocess.Popen(common + ["-c", src, "-o", obj],
                                            stdout=subprocess.PIPE, stderr=subprocess.STDOUT)))
    failed = []
    for src, p in procs:
        out = p.communicate()[0].decode()
        if out.strip():
            sys.stderr.write(out)
        if p.returncode != 0:
            failed.append(src)
    if failed:
        raise RuntimeError(f"nvcc failed for {failed}")
    tmp = LIB + ".tmp"
    subprocess.check_call([nvcc, *ARCH, "-shared", "-o", tmp, *objs, "-lcuda"])
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose-ptxas", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force or a.verbose_ptxas, verbose_ptxas=a.verbose_ptxas))
