"""Build the in-tree CUDA library `concord_b200/_lib/libconcord_b200.so`.

    python -m concord_b200.build

Compiles every .cu file under concord_b200/csrc for sm_100a with nvcc and
links one shared library with a plain C ABI (include/concord_b200.h).  The
step kernels are built with -fmad=false: the reference's arithmetic rounds
every fp32 multiply and add separately, and bit-exact words depend on the
compiler not fusing them.  Also builds the host copy of the correctly
rounded log2/exp2 (libcrmath_check.so) that the CPU tests check.
"""
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIBDIR = os.path.join(HERE, "_lib")
OUT = os.path.join(LIBDIR, "libconcord_b200.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVFLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-fmad=false", "-Xcompiler", "-fPIC",
                  "-Xcompiler", "-ffp-contract=off", "--expt-relaxed-constexpr"]


def _cutlass_root():
    """CUTLASS/CuTe headers (a vendored header tree shipped inside flashinfer)."""
    env = os.environ.get("CUTLASS_DIR")
    if env:
        return env
    import importlib.util
    spec = importlib.util.find_spec("flashinfer")
    if spec is None or not spec.submodule_search_locations:
        raise RuntimeError("CUTLASS headers not found: set CUTLASS_DIR")
    return os.path.join(list(spec.submodule_search_locations)[0], "data", "cutlass")


def _flags_for(cu):
    if os.path.basename(cu) in ("gemm.cu", "convgemm.cu"):
        root = _cutlass_root()
        # tensor-core GEMMs: contraction order is the hardware's; no -fmad=false needed
        return ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
                       "-I" + os.path.join(root, "include"),
                       "-I" + os.path.join(root, "tools", "util", "include"),
                       "-DNDEBUG", "-Xcompiler", "-Wno-psabi", "-diag-suppress", "20012"]
    return NVFLAGS


def _newer(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose=False, force=False):
    os.makedirs(LIBDIR, exist_ok=True)
    objdir = os.path.join(LIBDIR, "obj")
    os.makedirs(objdir, exist_ok=True)
    headers = glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh")) + \
        [os.path.join(HERE, "..", "include", "concord_b200.h")]
    objs = []
    for cu in sorted(glob.glob(os.path.join(CSRC, "*.cu"))):
        obj = os.path.join(objdir, os.path.basename(cu) + ".o")
        objs.append(obj)
        if force or _newer(obj, [cu] + headers):
            cmd = [NVCC] + _flags_for(cu) + ["-c", cu, "-o", obj]
            if verbose:
                print(" ".join(cmd), flush=True)
            subprocess.check_call(cmd)
    if force or _newer(OUT, objs):
        subprocess.check_call([NVCC] + ARCH + ["-shared", "-o", OUT] + objs + ["-lcudart"])
    chk = os.path.join(LIBDIR, "libcrmath_check.so")
    src = os.path.join(CSRC, "crmath_check.cpp")
    if force or _newer(chk, [src, os.path.join(CSRC, "crmath.h")]):
        subprocess.check_call(["g++", "-O2", "-fPIC", "-ffp-contract=off", "-shared", "-o", chk, src])
    return OUT


if __name__ == "__main__":
    print(build(verbose=True, force="--force" in sys.argv))
