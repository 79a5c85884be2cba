"""Build libsquirrel_cuda.so in-tree (squirrel-rs_b200/lib/) for sm_100a.

CUDA sources: nvcc -gencode arch=compute_100a,code=sm_100a -O3 -lineinfo.
Host sources: g++ -O2 -ffp-contract=off (host float math, e.g. the RoPE table
and inv_freq, must round like the reference's Rust, which never contracts).
The CUDA runtime is linked statically, so the library needs only the driver.
"""
import concurrent.futures as cf
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIB_DIR = os.path.join(HERE, "lib")
OBJ_DIR = os.path.join(HERE, "lib", "obj")
LIB = os.path.join(LIB_DIR, "libsquirrel_cuda.so")
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA, "bin", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def sources():
    cu = sorted(os.path.join(HERE, "csrc", f) for f in os.listdir(os.path.join(HERE, "csrc")) if f.endswith(".cu"))
    cpp = sorted(os.path.join(HERE, "host", f) for f in os.listdir(os.path.join(HERE, "host")) if f.endswith(".cpp"))
    return cu, cpp


def nccl_include():
    """Directory of nccl.h (types only: libnccl is opened at run time, not linked)."""
    for d in ("/usr/include", os.path.join(CUDA, "include")):
        if os.path.exists(os.path.join(d, "nccl.h")):
            return d
    try:
        import nvidia.nccl
        return os.path.join(os.path.dirname(nvidia.nccl.__file__), "include")
    except Exception:
        return "/usr/include"


def headers():
    out = [os.path.join(ROOT, "include", "squirrel_cuda.h")]
    for d in ("csrc", "host"):
        out += [os.path.join(HERE, d, f) for f in os.listdir(os.path.join(HERE, d)) if f.endswith((".cuh", ".h"))]
    return out


def _compile(src):
    obj = os.path.join(OBJ_DIR, os.path.basename(src) + ".o")
    newest = max([os.path.getmtime(src)] + [os.path.getmtime(h) for h in headers()])
    if os.path.exists(obj) and os.path.getmtime(obj) >= newest:
        return obj
    if src.endswith(".cu"):
        cmd = [NVCC] + ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xptxas", "-v",
                               "--expt-relaxed-constexpr", "-c", src, "-o", obj]
    else:
        cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-ffp-contract=off", "-fno-fast-math", "-I" + os.path.join(CUDA, "include"),
               "-I" + nccl_include(),
               "-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"compile failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    with open(obj + ".log", "w") as f:
        f.write(r.stderr)
    return obj


def build(force: bool = False) -> str:
    os.makedirs(OBJ_DIR, exist_ok=True)
    cu, cpp = sources()
    if force:
        for f in os.listdir(OBJ_DIR):
            os.remove(os.path.join(OBJ_DIR, f))
    with cf.ThreadPoolExecutor(max_workers=8) as ex:
        objs = list(ex.map(_compile, cu + cpp))
    if not force and os.path.exists(LIB) and all(os.path.getmtime(LIB) >= os.path.getmtime(o) for o in objs):
        return LIB
    cmd = [NVCC] + ARCH + ["-shared", "-cudart", "static", "-o", LIB] + objs + ["-lpthread", "-ldl", "-lrt"]  # no -lnccl
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
