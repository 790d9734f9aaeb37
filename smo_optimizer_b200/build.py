"""Build recipe of the CUDA library (``libsmo_b200.so``) and the host
extension (``_smo_host``), both in-tree.

    python -m smo_optimizer_b200.build [--verbose]

Compiles every ``csrc/*.cu`` for sm_100a with nvcc into one shared library
with the C ABI of include/smo_b200.h.  Needs nvcc only (no GPU): it
cross-compiles.  ``-fmad=false`` keeps every multiply and add separately
rounded unless the source asks for a fused multiply-add explicitly; the fp32
op order must match the reference bit for bit.

``csrc/smo_host.cpp`` (the per-step host work of the optimizer classes) is a
CPython extension compiled with g++ against the installed torch's headers and
libraries; it calls the CUDA library through a function pointer handed over
by the binding, so both use the one library ctypes loaded.
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
INCLUDE = os.path.join(ROOT, "include")
LIB_PATH = os.path.join(PKG, "libsmo_b200.so")

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-fmad=false", "-Xcompiler", "-fPIC,-O2",
              "-Xcompiler", "-fvisibility=hidden"]


def nvcc_path() -> str:
    cand = os.environ.get("CUDA_HOME") or "/usr/local/cuda"
    p = os.path.join(cand, "bin", "nvcc")
    if os.path.exists(p):
        return p
    found = shutil.which("nvcc")
    if not found:
        raise RuntimeError("nvcc not found: the CUDA library cannot be built")
    return found


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def deps():
    return sources() + sorted(glob.glob(os.path.join(CSRC, "*.cuh"))) + [os.path.join(INCLUDE, "smo_b200.h")]


def up_to_date() -> bool:
    if not os.path.exists(LIB_PATH):
        return False
    t = os.path.getmtime(LIB_PATH)
    return all(os.path.getmtime(d) <= t for d in deps())


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and up_to_date():
        return LIB_PATH
    import tempfile
    from concurrent.futures import ThreadPoolExecutor

    nvcc = nvcc_path()
    flags = [*ARCH_FLAGS, *NVCC_FLAGS, "-I", INCLUDE]
    if verbose:
        flags.insert(0, "-Xptxas=-v")
    with tempfile.TemporaryDirectory() as tmpdir:
        # one nvcc per source file, in parallel, then one link
        def compile_one(src):
            obj = os.path.join(tmpdir, os.path.basename(src) + ".o")
            cmd = [nvcc, *flags, "-c", src, "-o", obj]
            if verbose:
                print(" ".join(cmd))
            return obj, subprocess.run(cmd, capture_output=True, text=True)

        with ThreadPoolExecutor(max_workers=max(1, min(len(sources()), os.cpu_count() or 1))) as pool:
            results = list(pool.map(compile_one, sources()))
        for obj, res in results:
            if verbose or res.returncode != 0:
                sys.stderr.write(res.stdout + res.stderr)
            if res.returncode != 0:
                raise RuntimeError("nvcc failed to build libsmo_b200.so")
        tmp = LIB_PATH + ".tmp"
        res = subprocess.run([nvcc, *ARCH_FLAGS, "-shared", "-o", tmp, *[o for o, _ in results]],
                             capture_output=True, text=True)
        if res.returncode != 0:
            sys.stderr.write(res.stdout + res.stderr)
            raise RuntimeError("nvcc failed to link libsmo_b200.so")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


HOST_SRC = os.path.join(CSRC, "smo_host.cpp")


def host_ext_path() -> str:
    import sysconfig
    return os.path.join(PKG, "_smo_host" + sysconfig.get_config_var("EXT_SUFFIX"))


def build_host(force: bool = False, verbose: bool = False) -> str:
    """g++ build of the _smo_host extension (no GPU, no nvcc needed)."""
    import sysconfig

    import torch

    out = host_ext_path()
    srcs = [HOST_SRC, os.path.join(INCLUDE, "smo_b200.h")]
    if not force and os.path.exists(out) and all(os.path.getmtime(d) <= os.path.getmtime(out) for d in srcs):
        return out
    cuda_home = os.path.dirname(os.path.dirname(nvcc_path()))
    torch_dir = os.path.dirname(os.path.abspath(torch.__file__))
    incs = [os.path.join(torch_dir, "include"), os.path.join(torch_dir, "include", "torch", "csrc", "api", "include"),
            sysconfig.get_paths()["include"], os.path.join(cuda_home, "include"), INCLUDE]
    libdirs = [os.path.join(torch_dir, "lib")]
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = [shutil.which("g++") or "g++", "-O2", "-std=c++17", "-shared", "-fPIC", "-fvisibility=hidden",
           f"-D_GLIBCXX_USE_CXX11_ABI={abi}", *[f"-I{d}" for d in incs], HOST_SRC, "-o", out + ".tmp",
           *[f"-L{d}" for d in libdirs], *[f"-Wl,-rpath,{d}" for d in libdirs],
           "-lc10", "-lc10_cuda", "-ltorch_cpu", "-ltorch_python"]
    if verbose:
        print(" ".join(cmd))
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError("g++ failed to build the _smo_host extension")
    os.replace(out + ".tmp", out)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--force", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force or args.verbose, verbose=args.verbose))
    print(build_host(force=args.force, verbose=args.verbose))


if __name__ == "__main__":
    main()
