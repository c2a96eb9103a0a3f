"""Build the sm_100a kernel library in-tree with nvcc.

``python -m suffixgpu_b200.build`` compiles every ``csrc/*.cu`` for
``sm_100a`` (``-gencode arch=compute_100a,code=sm_100a``) into
``suffixgpu_b200/libsuffixgpu_b200.so``. Objects are rebuilt only when a
source or header is newer. The library has no torch dependency: it exports
the C ABI declared in ``include/suffixgpu.h``. ``csrc/torch_ops.cpp`` (the
torch operator over that ABI for the per-step call) is compiled with the
host C++ compiler against torch's headers into
``suffixgpu_b200/libsuffixgpu_b200_torch.so``, linked to the kernel
library.
"""

from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
OBJ = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libsuffixgpu_b200.so")
TORCH_LIB = os.path.join(PKG, "libsuffixgpu_b200_torch.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
         "-fmad=false", "--expt-relaxed-constexpr",
         "-I" + os.path.join(ROOT, "include")]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"),
                 "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _newest_dep() -> float:
    deps = glob.glob(os.path.join(CSRC, "*.cuh")) + [
        os.path.join(ROOT, "include", "suffixgpu.h")]
    return max(os.path.getmtime(p) for p in deps)


def build(verbose: bool = False, extra_flags: list[str] | None = None) -> str:
    """Compile (incrementally) and link; returns the library path."""
    nvcc = _nvcc()
    os.makedirs(OBJ, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    dep_t = _newest_dep()
    flags = FLAGS + (extra_flags or [])
    jobs = []
    objs = []
    for src in srcs:
        obj = os.path.join(OBJ, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        if (not os.path.exists(obj)
                or os.path.getmtime(obj) < max(os.path.getmtime(src), dep_t)):
            jobs.append([nvcc, *ARCH, *flags, "-c", src, "-o", obj])

    def run(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed:\n{' '.join(cmd)}\n{r.stderr}")
        if verbose and r.stderr.strip():
            print(r.stderr, file=sys.stderr)
        return r

    with ThreadPoolExecutor(max_workers=min(8, max(1, len(jobs)))) as ex:
        list(ex.map(run, jobs))
    if jobs or not os.path.exists(LIB) or os.path.getmtime(LIB) < max(
            os.path.getmtime(o) for o in objs):
        run([nvcc, *ARCH, "-shared", "-o", LIB, *objs, "-lcudart"])
    build_torch_ops(verbose)
    return LIB


def _loaded_cxx_runtime() -> str | None:
    """Path of the C++ runtime (libstdc++) this process has loaded -- the
    one torch uses, which the operator library must share."""
    try:
        with open("/proc/self/maps") as f:
            for line in f:
                path = line.split()[-1]
                if os.path.basename(path).startswith("libstdc++.so"):
                    return path
    except OSError:
        pass
    return None


def build_torch_ops(verbose: bool = False) -> str:
    """Compile the torch operator (incrementally) against torch's headers
    and libraries, linked to the kernel library (found next to it)."""
    src = os.path.join(CSRC, "torch_ops.cpp")
    newest = max(os.path.getmtime(src), os.path.getmtime(LIB),
                 os.path.getmtime(os.path.join(ROOT, "include", "suffixgpu.h")))
    if os.path.exists(TORCH_LIB) and os.path.getmtime(TORCH_LIB) >= newest:
        return TORCH_LIB
    import torch
    import torch.utils.cpp_extension as ce
    cxx = os.environ.get("CXX") or shutil.which("g++") or "g++"
    cuda_inc = os.path.join(os.path.dirname(os.path.dirname(_nvcc())),
                            "include")
    cmd = [cxx, "-O2", "-std=c++17", "-fPIC", "-shared",
           f"-D_GLIBCXX_USE_CXX11_ABI={int(torch._C._GLIBCXX_USE_CXX11_ABI)}",
           src, "-o", TORCH_LIB, "-I" + cuda_inc]
    # Link against the process's own libstdc++ by path: a compiler whose
    # shared libstdc++ link is missing would otherwise fall back to the
    # static archive, and a second C++ runtime inside this library crashes
    # as soon as it formats a number into an error message.
    rt = _loaded_cxx_runtime()
    if rt:
        cmd.append(rt)
    cmd += ["-I" + p for p in ce.include_paths(device_type="cuda")]
    cmd += ["-L" + p for p in ce.library_paths(device_type="cuda")]
    cmd += ["-L" + PKG, "-lsuffixgpu_b200", "-Wl,-rpath,$ORIGIN",
            "-lc10", "-ltorch", "-ltorch_cpu", "-lc10_cuda", "-ltorch_cuda"]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"torch op build failed:\n{' '.join(cmd)}\n"
                           f"{r.stderr}")
    return TORCH_LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
