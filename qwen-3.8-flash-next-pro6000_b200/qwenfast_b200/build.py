"""Build the native libraries in-tree: the CUDA kernels + C ABI with nvcc for sm_100a (``libqwenfast_b200.so``), and
the torch operator registration over that C ABI with g++ against torch's headers (``libqwenfast_b200_torch.so``:
``torch.ops.qwenfast_b200.*``).

``python -m qwenfast_b200.build`` (with the package directory on ``sys.path``) or ``build()`` from Python. The
libraries land next to this file; each is rebuilt only when a source or header it depends on changed.
"""
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
SRC_DIR = os.path.join(os.path.dirname(PKG_DIR), "csrc")
TORCH_SRC_DIR = os.path.join(os.path.dirname(PKG_DIR), "csrc_torch")
REPO_ROOT = os.path.dirname(os.path.dirname(PKG_DIR))
INCLUDE_DIR = os.path.join(REPO_ROOT, "include")
BUILD_DIR = os.path.join(REPO_ROOT, "_build")
LIB_PATH = os.path.join(PKG_DIR, "libqwenfast_b200.so")
TORCH_LIB_PATH = os.path.join(PKG_DIR, "libqwenfast_b200_torch.so")

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH_FLAGS + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-O3",
                           "--expt-relaxed-constexpr", "-I" + INCLUDE_DIR, "-I" + SRC_DIR]


def _nvcc():
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    path = os.path.join(home, "bin", "nvcc")
    return path if os.path.exists(path) else "nvcc"


def sources():
    return sorted(os.path.join(SRC_DIR, f) for f in os.listdir(SRC_DIR) if f.endswith(".cu"))


def _deps():
    hdrs = [os.path.join(SRC_DIR, f) for f in os.listdir(SRC_DIR) if f.endswith((".cuh", ".h"))]
    hdrs += [os.path.join(INCLUDE_DIR, f) for f in os.listdir(INCLUDE_DIR) if f.endswith(".h")]
    return hdrs


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False, extra_flags=None) -> str:
    """Compile every ``csrc/*.cu`` for sm_100a and link ``libqwenfast_b200.so``. Returns the library path."""
    os.makedirs(BUILD_DIR, exist_ok=True)
    hdrs = _deps()
    flags = NVCC_FLAGS + list(extra_flags or [])
    objs, jobs = [], []
    for src in sources():
        obj = os.path.join(BUILD_DIR, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        if force or _stale(obj, [src] + hdrs):
            jobs.append([_nvcc()] + flags + ["-c", src, "-o", obj])

    def run(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("nvcc failed:\n" + " ".join(cmd) + "\n" + r.stdout + r.stderr)
        if verbose and (r.stdout or r.stderr):
            print(r.stdout + r.stderr, flush=True)

    with ThreadPoolExecutor(max_workers=min(8, max(1, len(jobs)))) as ex:
        list(ex.map(run, jobs))
    if force or jobs or _stale(LIB_PATH, objs):
        run([_nvcc()] + ARCH_FLAGS + ["-shared", "-Xcompiler", "-fPIC", "-o", LIB_PATH] + objs + ["-lcudart"])
    build_torch_ops(force=force, verbose=verbose)
    return LIB_PATH


def build_torch_ops(force: bool = False, verbose: bool = False) -> str:
    """g++ the TORCH_LIBRARY registration (``csrc_torch/torch_ops.cpp``) against torch's headers into
    ``libqwenfast_b200_torch.so``, linked to ``libqwenfast_b200.so`` (found next to it through $ORIGIN) and torch."""
    import torch
    from torch.utils import cpp_extension as ce
    srcs = sorted(os.path.join(TORCH_SRC_DIR, f) for f in os.listdir(TORCH_SRC_DIR) if f.endswith(".cpp"))
    deps = srcs + [os.path.join(INCLUDE_DIR, f) for f in os.listdir(INCLUDE_DIR) if f.endswith(".h")] + [LIB_PATH]
    if not force and not _stale(TORCH_LIB_PATH, deps):
        return TORCH_LIB_PATH
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    tlib = ce.library_paths()[0]
    cmd = (["g++", "-O2", "-std=c++17", "-fPIC", "-shared",
            f"-D_GLIBCXX_USE_CXX11_ABI={int(torch._C._GLIBCXX_USE_CXX11_ABI)}"]
           + [f"-I{p}" for p in ce.include_paths()] + [f"-I{os.path.join(home, 'include')}", f"-I{INCLUDE_DIR}"]
           + srcs + ["-o", TORCH_LIB_PATH, f"-L{PKG_DIR}", "-lqwenfast_b200", "-Wl,-rpath,$ORIGIN",
                     f"-L{tlib}", f"-Wl,-rpath,{tlib}", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-lc10", "-lc10_cuda",
                     f"-L{os.path.join(home, 'lib64')}", "-lcudart"])
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("g++ failed:\n" + " ".join(cmd) + "\n" + r.stdout + r.stderr)
    return TORCH_LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
