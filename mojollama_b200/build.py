"""Build the in-tree native libraries (no JIT cache, no pip install).

    python -m mojollama_b200.build            # incremental
    python -m mojollama_b200.build --clean

Outputs in mojollama_b200/lib/:
  libmojollama_b200.so   all CUDA kernels (sm_100a) + the mlq_* C-ABI
  combined_engine.so     reference-named drop-ins for combined_engine.so
  quant_kernels_omp.so   (same symbols; the reference loads it as a fallback)
  cengine_batch_instr.so (same symbols; the reference loads it for ssm/batch_forward)
  simd_ops.so            reference-named drop-ins for simd_ops.so
  gqa_attention.so       reference-named drop-in for gqa_attention.so
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

PKG = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(PKG, "csrc")
LIB = os.path.join(PKG, "lib")
OBJ = os.path.join(os.path.dirname(PKG), "_build", "obj")
INCLUDE = os.path.join(os.path.dirname(PKG), "include")

NVCC = os.environ.get("NVCC", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVFLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
                  "-I" + INCLUDE, "--expt-relaxed-constexpr"]
CC = os.environ.get("CC_HOST", "gcc")
CFLAGS = ["-O2", "-fPIC", "-shared", "-I" + INCLUDE, "-Wall", "-Wno-unused-function"]

# reference library name -> shim source
ALIASES = {
    "combined_engine.so": "abi/engine_abi.c",
    "quant_kernels_omp.so": "abi/engine_abi.c",
    "cengine_batch_instr.so": "abi/engine_abi.c",
    "simd_ops.so": "abi/simd_abi.c",
    "gqa_attention.so": "abi/gqa_abi.c",
}


def _run(cmd):
    r = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if r.returncode != 0:
        sys.stderr.write(" ".join(cmd) + "\n" + r.stdout)
        raise RuntimeError(f"build step failed: {cmd[0]} ({r.returncode})")
    return r.stdout


def _stale(out, deps):
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose: bool = False, jobs: int = 0) -> str:
    os.makedirs(OBJ, exist_ok=True)
    os.makedirs(LIB, exist_ok=True)
    headers = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + \
        glob.glob(os.path.join(INCLUDE, "*.h"))
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    objs = []
    todo = []
    for s in sources:
        o = os.path.join(OBJ, os.path.basename(s)[:-3] + ".o")
        objs.append(o)
        if _stale(o, [s] + headers):
            todo.append((s, o))

    def compile_one(so):
        s, o = so
        out = _run([NVCC] + NVFLAGS + ["-Xptxas", "-v", "-c", s, "-o", o])
        if verbose:
            print(out)
        return s

    if todo:
        with ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 4)) as ex:
            for s in ex.map(compile_one, todo):
                print(f"  nvcc {os.path.relpath(s, PKG)}", flush=True)
    core = os.path.join(LIB, "libmojollama_b200.so")
    if _stale(core, objs):
        _run([NVCC] + ARCH + ["-shared", "-o", core] + objs + ["-lcudart", "-lcuda", "-lcublas"])
        print(f"  link {os.path.relpath(core, PKG)}", flush=True)
    for name, src in ALIASES.items():
        out = os.path.join(LIB, name)
        srcp = os.path.join(CSRC, src)
        if _stale(out, [srcp, core] + headers):
            _run([CC] + CFLAGS + ["-o", out, srcp, "-L" + LIB, "-lmojollama_b200",
                                  "-Wl,-rpath,$ORIGIN", "-Wl,--no-as-needed"])
            print(f"  cc   {os.path.relpath(out, PKG)}", flush=True)
    return LIB


def clean() -> None:
    shutil.rmtree(OBJ, ignore_errors=True)
    shutil.rmtree(LIB, ignore_errors=True)


if __name__ == "__main__":
    if "--clean" in sys.argv:
        clean()
    build(verbose="-v" in sys.argv)
