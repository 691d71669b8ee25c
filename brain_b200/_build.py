"""Native build of the brain_b200 libraries (sm_100a CUDA kernels and the C++ runtime).

Every CUDA source is compiled with ``nvcc -gencode arch=compute_100a,code=sm_100a`` into an
object under ``_build/`` at the repository root and linked into a shared library inside
``brain_b200/lib/``. The libraries expose a plain ``extern "C"`` ABI that ``brain_b200._native``
binds through ctypes, so no PyTorch headers are compiled and the build takes seconds per file.
Builds are incremental (object newer than its source and every header) and run in parallel.

Usage: ``python -m brain_b200._build [--force] [--jobs N]``.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
import sysconfig

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
LIBDIR = os.path.join(PKG, "lib")
OBJDIR = os.path.join(ROOT, "_build", "obj")

NVCC = os.environ.get("BRAIN_NVCC", shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc")
CUDA_HOME = os.path.dirname(os.path.dirname(os.path.realpath(NVCC)))
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC",
    "-Xcompiler", "-fvisibility=hidden", "-DNDEBUG", "-Xptxas", "-warn-spills",
]
CXX_FLAGS = ["-O3", "-std=c++17", "-fPIC", "-fvisibility=hidden", "-pthread", "-Wall", "-Wno-unused-function"]

# library name -> list of sources (relative to csrc/). Every CUDA library links host_utils.cu.
LIBRARIES = {
    "brain_kernels": [
        "host_utils.cu", "gemm.cu", "norms.cu", "elementwise.cu", "cross_entropy.cu", "optim.cu",
        "attention.cu", "attention_tc.cu", "attention_bwd_tc.cu", "attention_decode.cu", "decode_tp.cu", "fp8.cu",
        "linalg.cu",
    ],
    "brain_comm": ["host_utils.cu", "comm.cu"],
}
# Host-only C++ libraries (g++): the checkpoint codec, the native token loader, the BPE encoder and the
# float64 CPU oracle kernels.
CXX_LIBRARIES = {
    "brain_runtime": ["codec.cpp", "loader.cpp", "bpe.cpp", "oracle.cpp"],
}


def _headers():
    return [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h", ".hpp"))]


def _needs_build(out: str, deps: list[str]) -> bool:
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("build failed:\n" + " ".join(cmd) + "\n" + r.stdout + r.stderr)
    msg = (r.stdout + r.stderr).strip()
    if msg and os.environ.get("BRAIN_BUILD_VERBOSE"):
        print(msg)


def _compile_cu(src: str, force: bool) -> str:
    obj = os.path.join(OBJDIR, os.path.basename(src) + ".o")
    if force or _needs_build(obj, [src] + _headers()):
        _run([NVCC] + NVCC_FLAGS + ["-I", CSRC, "-c", src, "-o", obj])
    return obj


def _compile_cpp(src: str, force: bool) -> str:
    obj = os.path.join(OBJDIR, os.path.basename(src) + ".o")
    if force or _needs_build(obj, [src] + _headers()):
        _run(["g++"] + CXX_FLAGS + ["-I", CSRC, "-I", os.path.join(CUDA_HOME, "include"), "-c", src, "-o", obj])
    return obj


def build(force: bool = False, jobs: int | None = None, only: list[str] | None = None) -> list[str]:
    """Compile every native library; returns the list of produced .so paths."""
    os.makedirs(OBJDIR, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    jobs = jobs or max(1, (os.cpu_count() or 4))
    libs = {k: v for k, v in LIBRARIES.items() if not only or k in only}
    cxx_libs = {k: v for k, v in CXX_LIBRARIES.items() if not only or k in only}
    cu_srcs = sorted({os.path.join(CSRC, s) for v in libs.values() for s in v})
    cpp_srcs = sorted({os.path.join(CSRC, s) for v in cxx_libs.values() for s in v})
    with cf.ThreadPoolExecutor(jobs) as ex:
        futs = {ex.submit(_compile_cu, s, force): s for s in cu_srcs}
        futs.update({ex.submit(_compile_cpp, s, force): s for s in cpp_srcs})
        errors = []
        for f in cf.as_completed(futs):
            try:
                f.result()
            except Exception as e:  # collect all failures before raising
                errors.append(str(e))
        if errors:
            raise RuntimeError("\n\n".join(errors))
    outs = []
    for name, srcs in libs.items():
        objs = [os.path.join(OBJDIR, os.path.basename(s) + ".o") for s in srcs]
        so = os.path.join(LIBDIR, f"lib{name}.so")
        if force or _needs_build(so, objs):
            _run([NVCC] + ARCH + ["-shared", "-Xcompiler", "-fPIC", "-o", so] + objs + ["-lcudart"])
        outs.append(so)
    for name, srcs in cxx_libs.items():
        objs = [os.path.join(OBJDIR, os.path.basename(s) + ".o") for s in srcs]
        so = os.path.join(LIBDIR, f"lib{name}.so")
        if force or _needs_build(so, objs):
            _run(["g++", "-shared", "-fPIC", "-pthread", "-o", so] + objs)
        outs.append(so)
    return outs


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    ap.add_argument("--only", nargs="*", default=None)
    a = ap.parse_args(argv)
    for so in build(force=a.force, jobs=a.jobs, only=a.only):
        print(so)


if __name__ == "__main__":
    sys.exit(main())
