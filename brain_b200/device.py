"""Devices, device properties, a device guard, a compute-backend interface and the BLAS level-1/2/3
routines under the reference's names.

Reference: crates/brain-core/src/device.rs (``DeviceType`` tags Cpu / Cuda / Vulkan / Metal / Tpu with
``is_accelerator`` / ``has_unified_memory`` / ``supports_p2p`` :55-140; ``Device`` constructors,
predicates, ``parse``, ``properties`` :226-670; ``DeviceList`` :790-940; ``DeviceProperties``
:1007-1160; the ``Backend`` trait :1571-1600; ``DeviceGuard``), crates/brain-core/src/tensor/blas.rs
(axpy / dot / scal / nrm2 / asum / iamax / rot / swap / copy :14-135, gemv :139, ger :196,
gemm(trans_a, trans_b, alpha, beta) :227-300) and tensor/quant.rs:9-80 (``QuantizedTensor``).

Only CPU and CUDA can hold tensors here; Vulkan, Metal and TPU remain tags (as in the reference,
where they are tags only) and report unavailable. CUDA properties come from the driver through
torch. ``CudaBackend.matmul`` and ``blas.gemm`` on bf16 CUDA tensors run the framework's tcgen05 GEMM.
"""
from __future__ import annotations

import enum
from dataclasses import dataclass

import torch


class DeviceType(enum.Enum):
    CPU = "Cpu"
    CUDA = "Cuda"
    VULKAN = "Vulkan"
    METAL = "Metal"
    TPU = "Tpu"

    def name_str(self) -> str:
        return self.value

    def is_accelerator(self) -> bool:
        return self != DeviceType.CPU

    def has_unified_memory(self) -> bool:
        return self in (DeviceType.CPU, DeviceType.METAL)

    def supports_p2p(self) -> bool:
        return self == DeviceType.CUDA


@dataclass(frozen=True)
class DeviceProperties:
    name: str
    total_memory: int
    multiprocessor_count: int
    compute_capability: str
    clock_mhz: float | None = None
    memory_bandwidth_gbs: float | None = None
    l2_cache_bytes: int | None = None


@dataclass(frozen=True)
class Device:
    type: DeviceType = DeviceType.CPU
    index: int = 0

    @classmethod
    def cpu(cls) -> "Device":
        return cls(DeviceType.CPU, 0)

    @classmethod
    def cuda(cls, index: int = 0) -> "Device":
        return cls(DeviceType.CUDA, index)

    @classmethod
    def vulkan(cls, index: int = 0) -> "Device":
        return cls(DeviceType.VULKAN, index)

    @classmethod
    def metal(cls, index: int = 0) -> "Device":
        return cls(DeviceType.METAL, index)

    @classmethod
    def tpu(cls, index: int = 0) -> "Device":
        return cls(DeviceType.TPU, index)

    @classmethod
    def parse(cls, s: str) -> "Device":
        """"cpu", "cuda", "cuda:3", "vulkan:1", ... (case-insensitive)."""
        kind, _, idx = s.strip().lower().partition(":")
        types = {t.value.lower(): t for t in DeviceType}
        if kind not in types:
            raise ValueError(f"unknown device '{s}'")
        if idx and not idx.isdigit():
            raise ValueError(f"bad device index in '{s}'")
        return cls(types[kind], int(idx) if idx else 0)

    @classmethod
    def from_torch(cls, d) -> "Device":
        d = torch.device(d)
        return cls.cuda(d.index or 0) if d.type == "cuda" else cls.cpu()

    def to_torch(self) -> torch.device:
        if self.type == DeviceType.CPU:
            return torch.device("cpu")
        if self.type == DeviceType.CUDA:
            return torch.device("cuda", self.index)
        raise RuntimeError(f"{self.name()} is a device tag only; tensors live on CPU or CUDA")

    def is_cpu(self):
        return self.type == DeviceType.CPU

    def is_cuda(self):
        return self.type == DeviceType.CUDA

    def is_accelerator(self):
        return self.type.is_accelerator()

    def device_type(self):
        return self.type

    def name(self) -> str:
        return "cpu" if self.is_cpu() else f"{self.type.value.lower()}:{self.index}"

    def short_name(self) -> str:
        return self.type.value.lower()

    def is_available(self) -> bool:
        if self.is_cpu():
            return True
        return self.is_cuda() and torch.cuda.is_available() and self.index < torch.cuda.device_count()

    def synchronize(self) -> None:
        if self.is_cuda():
            torch.cuda.synchronize(self.index)

    def properties(self) -> DeviceProperties | None:
        if not (self.is_cuda() and self.is_available()):
            return None
        p = torch.cuda.get_device_properties(self.index)
        return DeviceProperties(p.name, p.total_memory, p.multi_processor_count, f"{p.major}.{p.minor}",
                                l2_cache_bytes=getattr(p, "L2_cache_size", None))

    def total_memory(self):
        p = self.properties()
        return p.total_memory if p else None

    def memory_available(self):
        if self.is_cuda() and self.is_available():
            return torch.cuda.mem_get_info(self.index)[0]
        return None

    def compute_capability(self):
        p = self.properties()
        return p.compute_capability if p else None

    def num_sm(self):
        p = self.properties()
        return p.multiprocessor_count if p else None

    def has_unified_memory(self):
        return self.type.has_unified_memory()

    def supports_bf16(self) -> bool:
        return self.is_cpu() or (self.is_cuda() and self.is_available() and torch.cuda.is_bf16_supported())

    def supports_f16(self) -> bool:
        return self.is_cpu() or self.is_cuda()

    def supports_f64(self) -> bool:
        return self.type in (DeviceType.CPU, DeviceType.CUDA)

    def supports_tensor_cores(self) -> bool:
        cc = self.compute_capability()
        return cc is not None and int(cc.split(".")[0]) >= 7

    def supports_p2p_with(self, other: "Device") -> bool:
        if not (self.is_cuda() and other.is_cuda()) or self == other:
            return False
        if not (self.is_available() and other.is_available()):
            return False
        return bool(torch.cuda.can_device_access_peer(self.index, other.index))

    def can_access(self, other: "Device") -> bool:
        return self == other or (self.has_unified_memory() and other.has_unified_memory()) or self.supports_p2p_with(other)

    def unique_id(self) -> str:
        return f"{self.type.value}-{self.index}"

    def __str__(self):
        return self.name()


class DeviceList:
    def __init__(self, devices=None):
        self.devices = list(devices) if devices is not None else self.enumerate()

    @staticmethod
    def enumerate() -> list[Device]:
        out = [Device.cpu()]
        if torch.cuda.is_available():
            out += [Device.cuda(i) for i in range(torch.cuda.device_count())]
        return out

    def cpu(self):
        return next((d for d in self.devices if d.is_cpu()), None)

    def cuda_devices(self):
        return [d for d in self.devices if d.is_cuda()]

    def accelerators(self):
        return [d for d in self.devices if d.is_accelerator()]

    def __len__(self):
        return len(self.devices)

    def __iter__(self):
        return iter(self.devices)

    def get(self, i):
        return self.devices[i] if 0 <= i < len(self.devices) else None

    def contains(self, d):
        return d in self.devices

    def cuda_count(self):
        return len(self.cuda_devices())

    def first_cuda(self):
        c = self.cuda_devices()
        return c[0] if c else None

    def first_accelerator(self):
        a = self.accelerators()
        return a[0] if a else None

    def total_memory_all(self):
        mems = [d.total_memory() for d in self.cuda_devices()]
        return sum(m for m in mems if m) or None

    def summary(self) -> str:
        return ", ".join(d.name() for d in self.devices)


class DeviceGuard:
    """Makes ``device`` current for a ``with`` block and restores the previous CUDA device after."""

    def __init__(self, device):
        self.device = device if isinstance(device, Device) else Device.from_torch(device)
        self._prev = None

    def __enter__(self):
        if self.device.is_cuda():
            self._prev = torch.cuda.current_device()
            torch.cuda.set_device(self.device.index)
        return self.device

    def __exit__(self, *exc):
        if self._prev is not None:
            torch.cuda.set_device(self._prev)
        return False


class Backend:
    """Compute-backend interface (matmul / add / mul / sum / relu / softmax)."""

    device: Device

    def matmul(self, a, b):
        raise NotImplementedError

    def add(self, a, b):
        return a + b

    def mul(self, a, b):
        return a * b

    def sum(self, a):
        return a.sum()

    def relu(self, a):
        return torch.relu(a)

    def softmax(self, a, dim: int = -1):
        return torch.softmax(a, dim)


class CpuBackend(Backend):
    def __init__(self):
        self.device = Device.cpu()

    def matmul(self, a, b):
        return torch.matmul(a, b)


class CudaBackend(Backend):
    """bf16 2-D matmuls run the framework's tcgen05 GEMM; other dtypes use torch."""

    def __init__(self, index: int = 0):
        self.device = Device.cuda(index)

    def matmul(self, a, b):
        if a.dtype == torch.bfloat16 and b.dtype == torch.bfloat16 and a.dim() == 2 and b.dim() == 2:
            from . import ops
            return ops.gemm(a, b)
        return torch.matmul(a, b)

    def softmax(self, a, dim: int = -1):
        return torch.softmax(a, dim)


def backend_for(device) -> Backend:
    d = device if isinstance(device, Device) else Device.from_torch(device)
    return CudaBackend(d.index) if d.is_cuda() else CpuBackend()


# ------------------------------------------------------------------ BLAS
class blas:  # noqa: N801  (namespace with the reference's routine names)
    @staticmethod
    def axpy(alpha, x, y):
        """y <- alpha x + y (in place); returns y."""
        return y.add_(x, alpha=alpha)

    @staticmethod
    def dot(x, y):
        return torch.dot(x.reshape(-1), y.reshape(-1))

    @staticmethod
    def scal(alpha, x):
        return x.mul_(alpha)

    @staticmethod
    def nrm2(x):
        return torch.linalg.vector_norm(x.reshape(-1).float())

    @staticmethod
    def asum(x):
        return x.abs().sum()

    @staticmethod
    def iamax(x) -> int:
        return int(x.reshape(-1).abs().argmax())

    @staticmethod
    def rot(x, y, c: float, s: float):
        """Givens rotation: (x, y) <- (c x + s y, c y − s x), in place."""
        xn = c * x + s * y
        y.mul_(c).sub_(s * x)
        x.copy_(xn)
        return x, y

    @staticmethod
    def swap(x, y):
        t = x.clone()
        x.copy_(y)
        y.copy_(t)
        return x, y

    @staticmethod
    def copy(x, y):
        return y.copy_(x)

    @staticmethod
    def gemv(alpha, a, x, beta, y, trans: bool = False):
        """y <- alpha op(A) x + beta y."""
        m = a.t() if trans else a
        return y.mul_(beta).add_(torch.mv(m, x), alpha=alpha)

    @staticmethod
    def ger(alpha, x, y, a):
        """A <- alpha x yᵀ + A."""
        return a.add_(torch.outer(x, y), alpha=alpha)

    @staticmethod
    def gemm(a, b, c=None, alpha: float = 1.0, beta: float = 0.0, trans_a: bool = False, trans_b: bool = False):
        """C <- alpha op(A) op(B) + beta C (a new C when none is given). bf16 CUDA operands run the
        tcgen05 GEMM with alpha / beta applied in its epilogue."""
        if a.is_cuda and a.dtype == torch.bfloat16 and b.dtype == torch.bfloat16:
            from . import ops
            if c is None or beta == 0.0:
                return ops.gemm(a, b, trans_a, trans_b, alpha=alpha, out=c, out_dtype=c.dtype if c is not None else torch.bfloat16)
            return ops.gemm(a, b, trans_a, trans_b, alpha=alpha, beta=beta, out=c, out_dtype=c.dtype)
        oa = a.t() if trans_a else a
        ob = b.t() if trans_b else b
        prod = alpha * (oa @ ob)
        if c is None:
            return prod
        return c.mul_(beta).add_(prod)


# ------------------------------------------------------------------ quantised tensor
@dataclass
class QuantizedTensor:
    """Per-tensor affine int8: x ≈ (q − zero_point) · scale."""
    data: torch.Tensor
    scale: float
    zero_point: int

    @classmethod
    def quantize(cls, x: torch.Tensor, symmetric: bool = False) -> "QuantizedTensor":
        lo, hi = float(x.min()), float(x.max())
        if symmetric:
            amax = max(abs(lo), abs(hi), 1e-12)
            scale, zp = amax / 127.0, 0
        else:
            lo, hi = min(lo, 0.0), max(hi, 0.0)
            scale = max(hi - lo, 1e-12) / 255.0
            zp = int(round(-128 - lo / scale))
        q = torch.clamp(torch.round(x / scale) + zp, -128, 127).to(torch.int8)
        return cls(q, scale, zp)

    def dequantize(self) -> torch.Tensor:
        return (self.data.float() - self.zero_point) * self.scale

    @property
    def shape(self):
        return self.data.shape
