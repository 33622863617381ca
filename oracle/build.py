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

The reference build needs the checkout (FW_REF_PATH, default
/root/reference); where it is absent (e.g. on a GPU box) the prebuilt files
travel with the tree and this step is skipped.
"""
import os
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
BUILD = os.path.join(HERE, "_build")
REF_OUT = os.path.join(HERE, "_ref")
ORACLE_SO = os.path.join(BUILD, "libfw_oracle.so")
REF_PATH = os.environ.get("FW_REF_PATH", "/root/reference")
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


def build(force=False):
    build_oracle(force)
    build_ref(force)


if __name__ == "__main__":
    build(force="--force" in sys.argv)
    print(ORACLE_SO)
    for isa in ISAS:
        print(ref_module_path(isa), os.path.exists(ref_module_path(isa)))
