"""Build libxq4.so (the sm_100a kernels + C ABI) in-tree with nvcc.

The library is compiled for sm_100a only (B200).  NCCL is bound at run time
(dlopen), so only its header is needed here.
"""
import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
OUT = PKG / "libxq4.so"
BUILD = PKG / "_build"

CU_SOURCES = ["api.cu", "gemv.cu", "gemv_w4a8.cu", "gemm_tc.cu", "dequant.cu", "comm.cu", "attn.cu"]
CPP_SOURCES = ["repack.cpp"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nccl_include():
    try:
        import nvidia.nccl  # noqa: F401
        inc = Path(list(nvidia.nccl.__path__)[0]) / "include"
        if (inc / "nccl.h").exists():
            return str(inc)
    except Exception:
        pass
    return "/usr/include"


def _nvcc():
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    p = Path(cuda) / "bin" / "nvcc"
    return str(p) if p.exists() else "nvcc"


def _stale(obj, deps):
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(verbose=False, force=False):
    BUILD.mkdir(exist_ok=True)
    headers = list(CSRC.glob("*.h")) + list(CSRC.glob("*.cuh")) + [ROOT / "include" / "xq4.h"]
    nvcc = _nvcc()
    common = ["-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-I", str(CSRC), "-I", str(ROOT / "include"),
              "-I", _nccl_include()]
    objs = []
    for src in CU_SOURCES:
        s = CSRC / src
        o = BUILD / (src + ".o")
        objs.append(o)
        if force or _stale(o, [s] + headers):
            cmd = [nvcc, *ARCH, "-lineinfo", *common, "-c", str(s), "-o", str(o)]
            if verbose:
                cmd.insert(1, "-Xptxas=-v")
            _run(cmd, verbose)
    for src in CPP_SOURCES:
        s = CSRC / src
        o = BUILD / (src + ".o")
        objs.append(o)
        if force or _stale(o, [s] + headers):
            _run(["g++", "-O3", "-std=c++17", "-fPIC", "-pthread", "-I", str(CSRC), "-I",
                  str(ROOT / "include"), "-c", str(s), "-o", str(o)], verbose)
    if force or _stale(OUT, objs):
        _run([nvcc, *ARCH, "-shared", "-o", str(OUT), *map(str, objs), "-lcudart", "-ldl", "-lpthread"],
             verbose)
    return OUT


def _run(cmd, verbose):
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if verbose or r.returncode:
        sys.stdout.write(r.stdout)
        sys.stderr.write(r.stderr)
    if r.returncode:
        raise RuntimeError(f"build step failed: {' '.join(cmd[:3])} ... (exit {r.returncode})")


if __name__ == "__main__":
    build(verbose="-v" in sys.argv, force="-f" in sys.argv)
    print(OUT)
