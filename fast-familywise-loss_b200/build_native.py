"""Builds the native parts in-tree (the built files travel with the source tree).

    python build_native.py     # both targets, skipped when up to date
    python build_native.py --force

Targets
  fwloss_b200/libfwloss_b200.so   the C-ABI library (include/fwloss_b200.h):
                                  all CUDA kernels, compiled for sm_100a only.
  fw_radix_cuda<EXT_SUFFIX>       the drop-in Python module `fw_radix_cuda`
                                  (csrc/fw_torch_binding.cpp), a host-only C++
                                  torch extension linked against the library.
"""
import os
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(ROOT, "include")
PKG = os.path.join(HERE, "fwloss_b200")
LIB = os.path.join(PKG, "libfwloss_b200.so")
BUILD_DIR = os.path.join(HERE, "_build")  # object files (git-ignored)
EXT = os.path.join(HERE, "fw_radix_cuda" + sysconfig.get_config_var("EXT_SUFFIX"))

NVCC_ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")


def _nvcc():
    p = os.path.join(CUDA_HOME, "bin", "nvcc")
    return p if os.path.exists(p) else "nvcc"


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _cuda_sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cu", ".cuh")))


def _compile_one(src, obj, verbose):
    cmd = [_nvcc(), *NVCC_ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
           "-Xcompiler", "-fvisibility=hidden", "-c", "-o", obj, src]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    return subprocess.run(cmd, capture_output=True, text=True)


def build_lib(force=False, verbose=False):
    """Every .cu file of csrc/ is one translation unit (compiled in parallel
    into BUILD_DIR), linked into one shared library."""
    from concurrent.futures import ThreadPoolExecutor

    headers = [p for p in _cuda_sources() if p.endswith(".cuh")] + [os.path.join(INCLUDE, "fwloss_b200.h")]
    units = [p for p in _cuda_sources() if p.endswith(".cu")]
    if not force and not _stale(LIB, headers + units):
        return LIB
    os.makedirs(BUILD_DIR, exist_ok=True)
    objs = [os.path.join(BUILD_DIR, os.path.basename(u)[:-3] + ".o") for u in units]
    todo = [(u, o) for u, o in zip(units, objs) if force or _stale(o, [u] + headers)]
    with ThreadPoolExecutor(max_workers=max(1, min(len(todo), os.cpu_count() or 1))) as ex:
        results = list(ex.map(lambda uo: (uo[0], _compile_one(uo[0], uo[1], verbose)), todo))
    for u, r in results:
        if verbose or r.returncode != 0:
            sys.stderr.write(r.stdout + r.stderr)
        if r.returncode != 0:
            raise subprocess.CalledProcessError(r.returncode, f"nvcc {u}")
    subprocess.run([_nvcc(), *NVCC_ARCH, "-shared", "-Xcompiler", "-fPIC", "-o", LIB + ".tmp", *objs], check=True)
    os.replace(LIB + ".tmp", LIB)
    return LIB


def build_ext(force=False):
    src = os.path.join(CSRC, "fw_torch_binding.cpp")
    deps = [src, os.path.join(INCLUDE, "fwloss_b200.h"), LIB]
    if not force and not _stale(EXT, deps):
        return EXT
    import torch
    from torch.utils import cpp_extension as ce

    incs = ce.include_paths(device_type="cuda") + [sysconfig.get_paths()["include"], INCLUDE,
                                                   os.path.join(CUDA_HOME, "include")]
    libdirs = ce.library_paths(device_type="cuda")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", src, "-o", EXT + ".tmp",
           "-DTORCH_EXTENSION_NAME=fw_radix_cuda", "-DTORCH_API_INCLUDE_EXTENSION_H",
           f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-Wno-deprecated-declarations"]
    cmd += [f"-I{p}" for p in incs]
    cmd += [f"-L{p}" for p in libdirs] + [f"-Wl,-rpath,{p}" for p in libdirs]
    cmd += [f"-L{PKG}", "-lfwloss_b200", "-Wl,-rpath,$ORIGIN/fwloss_b200",
            "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-ltorch_python"]
    subprocess.run(cmd, check=True)
    os.replace(EXT + ".tmp", EXT)
    return EXT


def build(force=False, verbose=False):
    build_lib(force, verbose)
    build_ext(force)


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
    print(EXT)
