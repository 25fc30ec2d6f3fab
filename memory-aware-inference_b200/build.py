"""Build libsi_cuda.so (sm_100a) in-tree from csrc/ with nvcc.

Usage: python memory-aware-inference_b200/build.py [--force]
Objects go to memory-aware-inference_b200/_build/, the library to
memory-aware-inference_b200/libsi_cuda.so and the si-bench command line next
to it (all git-ignored; they travel with the repository snapshot to the GPU box).
"""
import concurrent.futures as cf
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libsi_cuda.so")
CLI = os.path.join(HERE, "si-bench")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nccl_dirs():
    import importlib.util
    spec = importlib.util.find_spec("nvidia.nccl")
    if spec and spec.submodule_search_locations:
        base = list(spec.submodule_search_locations)[0]
        inc, lib = os.path.join(base, "include"), os.path.join(base, "lib")
        if os.path.exists(os.path.join(inc, "nccl.h")):
            return inc, lib
    return "/usr/include", "/usr/lib/x86_64-linux-gnu"


def _flags():
    inc, _ = _nccl_dirs()
    return ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-I", os.path.join(REPO, "include"),
                   "-I", inc, "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills"]


def _deps():
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + \
        [os.path.join(REPO, "include", "si_cuda.h")]


def _compile(src, force, verbose):
    obj = os.path.join(BUILD, os.path.basename(src) + ".o")
    newest = max([os.path.getmtime(src)] + [os.path.getmtime(d) for d in _deps()])
    if not force and os.path.exists(obj) and os.path.getmtime(obj) >= newest:
        return obj, ""
    cmd = [NVCC] + _flags() + (["-Xptxas", "-v"] if verbose else []) + ["-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stderr}")
    return obj, r.stderr


def build(force=False, verbose=False):
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        results = list(ex.map(lambda s: _compile(s, force, verbose), srcs))
    objs = [o for o, _ in results]
    if verbose:
        for _, log in results:
            if log:
                print(log)
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        _, libdir = _nccl_dirs()
        cmd = [NVCC] + ARCH + ["-shared", "-o", LIB] + objs + ["-L", libdir, "-l:libnccl.so.2",
                                                            "-Xlinker", "-rpath," + libdir]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stderr}")
    build_cli(force)
    return LIB


def build_cli(force=False):
    """The command-line programs (cli/*.cpp: si-bench, si-gguf-inspect): host
    C++ over the C ABI, linked against libsi_cuda.so beside them."""
    _, libdir = _nccl_dirs()
    for name, src in (("si-bench", "si_bench.cpp"), ("si-gguf-inspect", "si_gguf_inspect.cpp")):
        out = os.path.join(HERE, name)
        src = os.path.join(HERE, "cli", src)
        deps = [src, LIB, os.path.join(REPO, "include", "si_cuda.h")]
        if not force and os.path.exists(out) and os.path.getmtime(out) >= max(os.path.getmtime(d) for d in deps):
            continue
        cmd = ["g++", "-O2", "-std=c++17", "-Wall", "-I", os.path.join(REPO, "include"), src, "-o", out, "-L", HERE,
               "-l:libsi_cuda.so", "-Wl,-rpath,$ORIGIN", "-Wl,-rpath-link," + libdir]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"{name} build failed:\n{r.stderr}")
    return CLI


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
