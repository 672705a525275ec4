"""Build libqfn.so (the sm_100a kernels + C ABI) in-tree with nvcc.

Usage: python build.py [--force]

The shared library (and the thin torch extension over it, libqfn_torch.so)
is written next to this file so that it travels with the source tree;
`_lib.py` loads it from there.  Rebuilds only when a source or
header is newer than the library (or with --force).
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(REPO, "include")
LIB = os.path.join(HERE, "libqfn.so")

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-shared",
         "--expt-relaxed-constexpr", "-I", INCLUDE, "-I", CSRC]


def sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def deps():
    out = sources()
    out += [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    out += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith(".h")]
    return out


def needs_build():
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    return any(os.path.getmtime(p) > t for p in deps())


TORCH_EXT_SRC = os.path.join(HERE, "torch_ext", "qfn_torch.cpp")
TORCH_EXT = os.path.join(HERE, "libqfn_torch.so")


def build_torch_ext(force=False):
    """The thin torch extension (torch.ops.qfn.*) over libqfn.so, compiled with
    g++ against the installed torch; linked to libqfn.so next to it."""
    deps_ = [TORCH_EXT_SRC, LIB, os.path.join(INCLUDE, "qfn.h")]
    if not force and os.path.exists(TORCH_EXT) and all(os.path.getmtime(p) <= os.path.getmtime(TORCH_EXT)
                                                       for p in deps_):
        return TORCH_EXT
    import torch
    import torch.utils.cpp_extension as ce
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    inc = [f"-I{p}" for p in ce.include_paths()] + ["-I/usr/local/cuda/include", f"-I{INCLUDE}"]
    libs = [f"-L{p}" for p in ce.library_paths()] + ["-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu"]
    tmp = TORCH_EXT + ".tmp"
    cmd = ["g++", "-O2", "-std=c++17", "-shared", "-fPIC", f"-D_GLIBCXX_USE_CXX11_ABI={abi}", *inc, TORCH_EXT_SRC,
           *libs, f"-L{HERE}", "-lqfn", "-Wl,-rpath,$ORIGIN", "-o", tmp]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"g++ (torch extension) failed ({r.returncode}):\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, TORCH_EXT)
    return TORCH_EXT


def build(force=False, verbose=False):
    """Compile every .cu under csrc/ into libqfn.so, then the torch extension
    over it (libqfn_torch.so); returns the library path."""
    if force or needs_build():
        _build_lib(verbose)
    build_torch_ext(force)
    return LIB


def _build_lib(verbose=False):
    tmp = LIB + ".tmp"
    cmd = [NVCC, *ARCH, *FLAGS, *sources(), "-o", tmp, "-lcuda", "-ldl"]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd))
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed ({r.returncode}):\n{r.stdout}\n{r.stderr}")
    if verbose:
        print(r.stdout + r.stderr)
    os.replace(tmp, LIB)


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
