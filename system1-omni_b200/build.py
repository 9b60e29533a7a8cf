"""Build the native libraries of this package in-tree (no GPU needed: nvcc cross-compiles).

  libqwen3_5_cuda.so -- the cs1_* C ABI (csrc/*.cu), sm_100a kernels
  libs1_model.so     -- the C++ prefill host (host/*.cpp): configuration, weight arena,
                        packed / shared-prefix forward, scorer head, CUDA graphs; it
                        dlopens a cs1_* library at run time, like the reference's loader

    python system1-omni_b200/build.py [--jobs N] [--force]
"""
import argparse
import concurrent.futures as cf
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
HOST = os.path.join(PKG, "host")
OUT = os.path.join(PKG, "lib")
OBJ = os.path.join(PKG, "_build")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CUDA_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
              "--expt-relaxed-constexpr", "-I", os.path.join(ROOT, "include")]

CU_SOURCES = ["runtime.cu", "norm.cu", "elementwise.cu", "gemm.cu", "attention.cu", "gdn.cu",
              "head.cu", "gdn_noalloc.cu", "gdn_fused.cu"]
CPP_SOURCES = ["model.cpp", "checkpoint.cpp", "tokenizer.cpp", "processing.cpp"]


def _newer(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def _headers(d):
    return [os.path.join(d, f) for f in os.listdir(d) if f.endswith((".h", ".cuh", ".hpp"))] + \
        [os.path.join(ROOT, "include", f) for f in os.listdir(os.path.join(ROOT, "include"))]


def compile_cu(src, force, tuning=False):
    obj = os.path.join(OBJ, os.path.basename(src) + ".o")
    if not force and not _newer(obj, [src] + _headers(CSRC)):
        return obj, None
    cmd = [NVCC, *ARCH, *CUDA_FLAGS, *(["-DS1_TUNING"] if tuning else []), "-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode:
        return obj, r.stderr + r.stdout
    return obj, None


def build(jobs=8, force=False, verbose=False, tuning=False):
    """tuning: compile with -DS1_TUNING (kernel-choice overrides read from the environment,
    for calibration runs only); forces a full rebuild, as does the next product build."""
    stamp = os.path.join(OBJ, "tuning.stamp")
    if tuning != os.path.exists(stamp):
        force = True
    os.makedirs(OUT, exist_ok=True)
    os.makedirs(OBJ, exist_ok=True)
    srcs = [os.path.join(CSRC, s) for s in CU_SOURCES]
    errors = []
    objs = []
    with cf.ThreadPoolExecutor(jobs) as ex:
        for obj, err in ex.map(lambda s: compile_cu(s, force, tuning), srcs):
            objs.append(obj)
            if err:
                errors.append(err)
    if errors:
        raise RuntimeError("nvcc failed:\n" + "\n".join(errors))
    if tuning:
        open(stamp, "w").close()
    elif os.path.exists(stamp):
        os.remove(stamp)
    lib = os.path.join(OUT, "libqwen3_5_cuda.so")
    if force or _newer(lib, objs):
        cmd = [NVCC, *ARCH, "-shared", "-Xcompiler", "-fPIC", "-o", lib, *objs, "-lcudart_static", "-lrt",
               "-ldl", "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode:
            raise RuntimeError("link failed:\n" + r.stderr + r.stdout)
    model = os.path.join(OUT, "libs1_model.so")
    cpp = [os.path.join(HOST, s) for s in CPP_SOURCES]
    if force or _newer(model, cpp + _headers(HOST)):
        cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-fvisibility=hidden", "-I",
               os.path.join(ROOT, "include"), "-I", "/usr/local/cuda/include", "-o", model, *cpp, "-ldl",
               "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode:
            raise RuntimeError("g++ failed:\n" + r.stderr + r.stdout)
    if verbose:
        print("built", lib, model)
    return lib, model


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--jobs", type=int, default=8)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--tuning", action="store_true", help="kernel-choice overrides from the environment")
    a = ap.parse_args()
    try:
        build(a.jobs, a.force, verbose=True, tuning=a.tuning)
    except RuntimeError as e:
        print(e, file=sys.stderr)
        sys.exit(1)
