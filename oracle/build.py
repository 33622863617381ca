"""Builds the oracle side -- TEST INFRASTRUCTURE ONLY.

  oracle/_build/libfw_oracle.so      the C restatement (oracle/fw_oracle.c)
  oracle/_ref/fw_cpu_ref_<isa>*.so   the reference's own CPU extension,
                                     compiled from its single source file
                                     src/cpu/fw_cpu.cpp where it lies in the
                                     reference checkout (read-only; nothing is
                                     copied), one build per ISA level so the
                                     file runs on any x86-64 host:
                                       avx512: -march=x86-64-v4
                                       avx2:   -march=x86-64-v3
                                     Flags otherwise as the reference's loader
                                     (src/cpu/fwcpp.py:12-16): -O3 -fopenmp
                                     -fno-math-errno.

  oracle/_ref/fw_radix_cuda_ref*.so  the reference's own CUDA extension
                                     (src/cuda/fw_radix_argmax.cu and
                                     src/cuda/binding.cpp, the two sources its
                                     setup.py:7-13 builds), compiled for
                                     sm_100a where they lie, as module
                                     fw_radix_cuda_ref: the GPU baseline that
                                     the benchmark times next to ours and a
                                     parity check of kappa.

The reference build needs the reference checkout: the directory named by the
environment variable FW_REF_PATH, or else a checkout named `reference` beside
this repository (REF_PATH below); where it is absent (e.g. on a GPU box) the
prebuilt files travel with the tree and this step is skipped.
"""
import os
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
BUILD = os.path.join(HERE, "_build")
REF_OUT = os.path.join(HERE, "_ref")
ORACLE_SO = os.path.join(BUILD, "libfw_oracle.so")
REF_PATH = os.environ.get("FW_REF_PATH") or os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")
REF_SRC = os.path.join(REF_PATH, "src", "cpu", "fw_cpu.cpp")
ISAS = {"avx512": "-march=x86-64-v4", "avx2": "-march=x86-64-v3"}
SUFFIX = sysconfig.get_config_var("EXT_SUFFIX")


def ref_module_path(isa):
    return os.path.join(REF_OUT, f"fw_cpu_ref_{isa}{SUFFIX}")


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    return any(os.path.getmtime(d) > os.path.getmtime(target) for d in deps if os.path.exists(d))


def build_oracle(force=False):
    os.makedirs(BUILD, exist_ok=True)
    src = os.path.join(HERE, "fw_oracle.c")
    if force or _stale(ORACLE_SO, [src]):
        subprocess.run(["gcc", "-O2", "-fopenmp", "-fPIC", "-shared", src, "-o", ORACLE_SO + ".tmp", "-lm"],
                       check=True)
        os.replace(ORACLE_SO + ".tmp", ORACLE_SO)
    return ORACLE_SO


def build_ref(force=False):
    if not os.path.exists(REF_SRC):
        return []
    import torch
    from torch.utils import cpp_extension as ce

    os.makedirs(REF_OUT, exist_ok=True)
    incs = ce.include_paths() + [sysconfig.get_paths()["include"]]
    libdirs = ce.library_paths()
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    out = []
    for isa, march in ISAS.items():
        target = ref_module_path(isa)
        out.append(target)
        if not force and not _stale(target, [REF_SRC]):
            continue
        cmd = ["/usr/bin/g++", "-O3", "-fopenmp", "-fno-math-errno", march, "-std=c++17", "-fPIC",
               "-shared", REF_SRC, "-o", target + ".tmp",
               f"-DTORCH_EXTENSION_NAME=fw_cpu_ref_{isa}", "-DTORCH_API_INCLUDE_EXTENSION_H",
               f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-Wno-deprecated-declarations"]
        cmd += [f"-I{p}" for p in incs] + [f"-L{p}" for p in libdirs]
        cmd += [f"-Wl,-rpath,{p}" for p in libdirs]
        cmd += ["-lc10", "-ltorch", "-ltorch_cpu", "-ltorch_python", "-fopenmp"]
        subprocess.run(cmd, check=True)
        os.replace(target + ".tmp", target)
    return out


REF_CUDA_SRCS = [os.path.join(REF_PATH, "src", "cuda", f) for f in ("fw_radix_argmax.cu", "binding.cpp")]


def ref_cuda_module_path():
    return os.path.join(REF_OUT, f"fw_radix_cuda_ref{SUFFIX}")


def build_ref_cuda(force=False):
    """nvcc / g++ on the reference's two CUDA-extension sources, with the
    defines torch's CUDAExtension passes (the reference's setup.py adds no
    flags of its own), for sm_100a."""
    if not all(os.path.exists(p) for p in REF_CUDA_SRCS):
        return None
    target = ref_cuda_module_path()
    if not force and not _stale(target, REF_CUDA_SRCS):
        return target
    import torch
    from torch.utils import cpp_extension as ce

    os.makedirs(REF_OUT, exist_ok=True)
    os.makedirs(BUILD, exist_ok=True)
    incs = ce.include_paths(device_type="cuda") + [sysconfig.get_paths()["include"]]
    libdirs = ce.library_paths(device_type="cuda")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    defs = ["-DTORCH_EXTENSION_NAME=fw_radix_cuda_ref", "-DTORCH_API_INCLUDE_EXTENSION_H",
            f"-D_GLIBCXX_USE_CXX11_ABI={abi}"]
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    nvcc = os.path.join(cuda_home, "bin", "nvcc")
    cu_obj = os.path.join(BUILD, "fw_radix_argmax_ref.o")
    cpp_obj = os.path.join(BUILD, "binding_ref.o")
    cmd = [nvcc, "-c", REF_CUDA_SRCS[0], "-o", cu_obj, "-gencode", "arch=compute_100a,code=sm_100a", "-O3",
           "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr", "-D__CUDA_NO_HALF_OPERATORS__",
           "-D__CUDA_NO_HALF_CONVERSIONS__", "-D__CUDA_NO_BFLOAT16_CONVERSIONS__",
           "-D__CUDA_NO_HALF2_OPERATORS__", "-w"] + defs + [f"-I{p}" for p in incs]
    subprocess.run(cmd, check=True)
    cmd = ["g++", "-c", REF_CUDA_SRCS[1], "-o", cpp_obj, "-O2", "-std=c++17", "-fPIC",
           "-Wno-deprecated-declarations"] + defs + [f"-I{p}" for p in incs + [os.path.join(cuda_home, "include")]]
    subprocess.run(cmd, check=True)
    cmd = ["g++", "-shared", cu_obj, cpp_obj, "-o", target + ".tmp"]
    cmd += [f"-L{p}" for p in libdirs + [os.path.join(cuda_home, "lib64")]]
    cmd += [f"-Wl,-rpath,{p}" for p in libdirs]
    cmd += ["-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-ltorch_python", "-lcudart"]
    subprocess.run(cmd, check=True)
    os.replace(target + ".tmp", target)
    return target


def build(force=False):
    build_oracle(force)
    build_ref(force)
    build_ref_cuda(force)


if __name__ == "__main__":
    build(force="--force" in sys.argv)
    print(ORACLE_SO)
    for isa in ISAS:
        print(ref_module_path(isa), os.path.exists(ref_module_path(isa)))
    print(ref_cuda_module_path(), os.path.exists(ref_cuda_module_path()))
