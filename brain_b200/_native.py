"""ctypes bindings to the in-tree native libraries (``brain_b200/lib/*.so``).

The CUDA kernels and the C++ runtime export a plain C ABI (``extern "C"``). Each entry point
returns an ``int`` status (0 = success, otherwise a ``cudaError_t`` or a negative runtime code);
:func:`call` raises :class:`NativeError` on failure. Pointers are passed as integers
(``tensor.data_ptr()``) and the CUDA stream as the raw ``cudaStream_t`` of the current PyTorch
stream, so kernels order correctly with PyTorch work and can be captured in CUDA graphs.

When a CUDA tensor reaches an op whose library is missing, the op raises
:class:`NativeMissing` instead of silently falling back: on a GPU the native path is the product.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

LIBDIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "lib")

_P = ctypes.c_void_p
_I = ctypes.c_int
_L = ctypes.c_int64
_F = ctypes.c_float
_D = ctypes.c_double
_CODES = {"p": _P, "i": _I, "l": _L, "f": _F, "d": _D, "s": _P}

# name -> (library, argument codes). 's' marks the trailing cudaStream_t.
SIGNATURES: dict[str, tuple[str, str]] = {
    "brain_error_string": ("brain_kernels", "i"),
    "brain_gemm_bf16": ("brain_kernels", "pliplipliiiififpplis"),
    "brain_status_gemm": ("brain_kernels", "pi"),
    "brain_gemm_set_pair_mode": ("brain_kernels", "i"),
    "brain_gemm_set_push_stage": ("brain_kernels", "i"),
    "brain_gemm_bf16_rope": ("brain_kernels", "plplpliiipiiiis"),
    "brain_gemm_bf16_ws": ("brain_kernels", "pliplipliiiififpplpls"),
    "brain_gemm_splitk_plan": ("brain_kernels", "iiip"),
}

_lock = threading.Lock()
_libs: dict[str, ctypes.CDLL] = {}
_fns: dict[str, ctypes._CFuncPtr] = {}


class NativeMissing(RuntimeError):
    """A native library needed by a CUDA op is not built."""


class NativeError(RuntimeError):
    """A native entry point returned a non-zero status."""


def lib_path(name: str) -> str:
    return os.path.join(LIBDIR, f"lib{name}.so")


def load(name: str) -> ctypes.CDLL:
    with _lock:
        lib = _libs.get(name)
        if lib is not None:
            return lib
        path = lib_path(name)
        if not os.path.exists(path):
            raise NativeMissing(f"native library {path} is not built; run `python -m brain_b200._build`")
        lib = ctypes.CDLL(path, mode=ctypes.RTLD_GLOBAL)
        _libs[name] = lib
        return lib


def available(name: str = "brain_kernels") -> bool:
    try:
        load(name)
        return True
    except (NativeMissing, OSError):
        return False


# entry points whose C return type is int64_t (all others return int status codes)
RETURNS_I64: set[str] = set()


def fn(name: str):
    f = _fns.get(name)
    if f is not None:
        return f
    libname, codes = SIGNATURES[name]
    lib = load(libname)
    f = getattr(lib, name)
    f.argtypes = [_CODES[c] for c in codes]
    f.restype = ctypes.c_char_p if name == "brain_error_string" else (_L if name in RETURNS_I64 else _I)
    _fns[name] = f
    return f


def stream_ptr(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


# Kernels launched by one call of each multi-kernel entry point (default 1); used to count this
# library's launches inside a timed region (``launch_counter``).
KERNELS_PER_CALL = {
    "brain_norm_bwd": 2, "brain_attn_bwd": 4, "brain_sumsq": 2, "brain_error_string": 0,
    "brain_norm_bwd_partials": 0, "brain_gemm_splitk_plan": 0, "brain_gemm_bf16_ws": 2,
    "brain_colsum_partials": 0, "brain_colsum_bf16": 2,
}
_launches = {"on": False, "n": 0}


class launch_counter:
    """Context manager counting native kernel launches issued through :func:`call`."""

    def __enter__(self):
        _launches["on"], _launches["n"] = True, 0
        return self

    def __exit__(self, *exc):
        _launches["on"] = False

    @property
    def count(self) -> int:
        return _launches["n"]


_nvtx = {"on": os.environ.get("BRAIN_NVTX", "0") == "1"}


def set_nvtx(on: bool) -> None:
    """NVTX range (the entry point's name) around every native call, for Nsight timelines; also
    enabled by ``BRAIN_NVTX=1``. Off by default (a range push / pop costs host time per call)."""
    _nvtx["on"] = bool(on)


def call(name: str, *args) -> int:
    if _launches["on"]:
        _launches["n"] += KERNELS_PER_CALL.get(name, 1)
    if _nvtx["on"]:
        torch.cuda.nvtx.range_push(name)
        try:
            rc = fn(name)(*args)
        finally:
            torch.cuda.nvtx.range_pop()
    else:
        rc = fn(name)(*args)
    if rc != 0:
        try:
            msg = fn("brain_error_string")(rc).decode()
        except Exception:  # pragma: no cover - diagnostic only
            msg = "?"
        raise NativeError(f"{name} failed with status {rc} ({msg})")
    return rc


def status(lib_tag: str, clear: bool = True) -> tuple[int, int]:
    """Read the device status word of one kernel translation unit: (code, where)."""
    where = ctypes.c_int(0)
    code = fn(f"brain_status_{lib_tag}")(ctypes.byref(where), 1 if clear else 0)
    return code, where.value


def register(signatures: dict[str, tuple[str, str]]) -> None:
    """Add entry-point signatures (used by the op modules next to their wrappers)."""
    SIGNATURES.update(signatures)


def require_cuda_lib(t: torch.Tensor, name: str = "brain_kernels") -> None:
    """Raise loudly when a CUDA tensor would need a native library that is not built."""
    if t.is_cuda and not available(name):
        raise NativeMissing(f"CUDA tensor given but {lib_path(name)} is missing")
