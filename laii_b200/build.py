"""Build the native libraries in-tree (laii_b200/_lib/).

  liblfm_gpu_moe.so  CUDA kernels + C-ABI (include/lfm_gpu_moe.h), sm_100a only
  liblfm_synth.so    host seeded-input generator (C)

nvcc flags: -gencode arch=compute_100a,code=sm_100a; -fmad=false and
-ftz=true so device fp32 follows the reference's evaluation order under
FTZ/DAZ (every FMA in the kernels is explicit); the CUDA runtime is linked
statically so the library does not depend on which libcudart a host process
already loaded.  Run:  python -m laii_b200.build
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
LIB = os.path.join(PKG, "_lib")
BUILD = os.path.join(PKG, "_build")

GPU_SO = os.path.join(LIB, "liblfm_gpu_moe.so")
SYNTH_SO = os.path.join(LIB, "liblfm_synth.so")

CU_SOURCES = ["lfm_gpu_moe.cu", "k_route.cu", "k_gemv.cu", "k_layer.cu", "k_gemm.cu", "k_umma.cu", "k_expert.cu", "k_ep.cu", "k_q6k.cu", "k_synth.cu", "lfm_gguf.cpp"]
HEADERS = ["lfm_formats.h", "lfm_synth_core.h", "moe_internal.h", "moe_device.cuh"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-fmad=false", "-ftz=true", "-prec-div=true", "-prec-sqrt=true",
    "-Xcompiler", "-fPIC,-fvisibility=hidden",
    "-I" + CSRC, "-I" + os.path.join(ROOT, "include"),
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the CUDA library cannot be built")


def _newest(paths):
    return max(os.path.getmtime(p) for p in paths)


def _stale(target: str, deps) -> bool:
    return not os.path.exists(target) or os.path.getmtime(target) < _newest(deps)


def _run(cmd):
    r = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if r.returncode != 0:
        raise RuntimeError("build failed:\n" + " ".join(cmd) + "\n" + r.stdout)
    return r.stdout


class _BuildLock:
    """Exclusive lock over the build folder, so that several processes started together (one per
    GPU) build once: the others wait, then find the library fresh."""

    def __enter__(self):
        import fcntl
        os.makedirs(LIB, exist_ok=True)
        self.f = open(os.path.join(LIB, ".build.lock"), "w")
        fcntl.flock(self.f, fcntl.LOCK_EX)
        return self

    def __exit__(self, *exc):
        import fcntl
        fcntl.flock(self.f, fcntl.LOCK_UN)
        self.f.close()


def build_synth(force: bool = False) -> str:
    src = os.path.join(CSRC, "lfm_synth.c")
    deps = [src] + [os.path.join(CSRC, h) for h in ("lfm_formats.h", "lfm_synth_core.h")]
    if not (force or _stale(SYNTH_SO, deps)):
        return SYNTH_SO
    with _BuildLock():
        if force or _stale(SYNTH_SO, deps):
            cc = os.environ.get("CC", "gcc")
            tmp = f"{SYNTH_SO}.{os.getpid()}.tmp"
            _run([cc, "-std=c11", "-O2", "-fPIC", "-shared", "-fvisibility=hidden", "-o", tmp, src,
                  "-lm", "-lpthread"])
            os.replace(tmp, SYNTH_SO)
    return SYNTH_SO


def build_gpu(force: bool = False, verbose_ptxas: bool = False) -> str:
    srcs = [os.path.join(CSRC, s) for s in CU_SOURCES]
    deps = srcs + [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(ROOT, "include", "lfm_gpu_moe.h"),
                                                              os.path.abspath(__file__)]
    if not (force or _stale(GPU_SO, deps)):
        return GPU_SO
    with _BuildLock():
        if force or _stale(GPU_SO, deps):
            _build_gpu_locked(srcs, verbose_ptxas)
    return GPU_SO


def _build_gpu_locked(srcs, verbose_ptxas: bool) -> None:
    os.makedirs(BUILD, exist_ok=True)
    nvcc = _nvcc()
    extra = ["-Xptxas", "-v"] if verbose_ptxas else []

    def compile_one(src):
        obj = os.path.join(BUILD, os.path.basename(src) + ".o")
        out = _run([nvcc, *NVCC_FLAGS, *extra, "-c", src, "-o", obj])
        return obj, out

    with ThreadPoolExecutor(max_workers=len(srcs)) as ex:
        results = list(ex.map(compile_one, srcs))
    if verbose_ptxas:
        for _, out in results:
            sys.stdout.write(out)
    objs = [o for o, _ in results]
    tmp = f"{GPU_SO}.{os.getpid()}.tmp"
    _run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-cudart", "static", "-o", tmp, *objs,
          "-Xlinker", "--exclude-libs,ALL"])
    os.replace(tmp, GPU_SO)


def build_all(force: bool = False) -> None:
    build_synth(force)
    build_gpu(force)


if __name__ == "__main__":
    build_all(force="--force" in sys.argv)
    if "--ptxas" in sys.argv:
        build_gpu(force=True, verbose_ptxas=True)
    print("built", GPU_SO, SYNTH_SO)
