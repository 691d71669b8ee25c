"""Readers and writers for the reference's checkpoint formats, plus a large-model binary container.

Compatible formats (byte layouts shared with the reference so files move both ways):
  * ``serialize_tensor`` / ``deserialize_tensor``: per-tensor binary v2 (and v1 read)
    (crates/brain-core/src/serialization.rs:53-77, 190-390). The magic is ``b"BRAIN   "`` (three
    spaces) as in the code; the payload is always f64 little-endian, the dtype byte is a tag.
  * ``TensorArchive``: ``b"BRAIN_ARCHIVE\\0"`` + count + (name, size, tensor) entries (serialization.rs:414-553).
    Entries are written in sorted name order (the reference uses HashMap order, so any order is read).
  * ``BrainModelFile`` (``.bn``): ``b"BRAIN_BN"``, version 1, name, metadata, 3-D node coordinates,
    the archive, and a trailing CRC32 over every preceding byte (serialization.rs:574-760).
  * ``ModelState`` text ``BRAIN_STATE_V1`` (crates/brain-train/src/lib.rs:929-1075): ``meta|k|v`` lines
    then ``tensor|name|AxB|v,v,...`` lines with Rust f64 Display values; meta keys are written sorted.

New for large models: ``save_brain_v2`` / ``load_brain_v2`` (``b"BRAINCK2"``) keep tensors in their
native dtype (bf16/f32/fp8/int), one CRC32 per tensor, a JSON header with metadata, 64-byte aligned
payloads in deterministic order, and per-rank shard files for sharded optimizer state.
CRC32 and the float text encoding run in the C++ codec (``csrc/codec.cpp``).
"""
from __future__ import annotations

import ctypes
import json
import os
import struct
from dataclasses import dataclass, field

import numpy as np
import torch

from .. import _native

_native.register({
    "brain_crc32": ("brain_runtime", "pl"),
    "brain_crc32_update": ("brain_runtime", "ipl"),
    "brain_format_f64": ("brain_runtime", "plpl"),
    "brain_parse_f64": ("brain_runtime", "plpl"),
})

MAGIC_HEADER = b"BRAIN   "
ARCHIVE_MAGIC = b"BRAIN_ARCHIVE\x00"
BN_MAGIC = b"BRAIN_BN"
CKPT_V2_MAGIC = b"BRAINCK2"
FORMAT_VERSION_V1, FORMAT_VERSION_V2 = 1, 2
ENDIAN_LITTLE, ENDIAN_BIG = 0, 1
DTYPE_CODES = {"f64": 0, "f32": 1, "f16": 2, "bf16": 3, "i64": 4, "i32": 5, "i16": 6, "i8": 7, "u8": 8,
               "bool": 9}
CODE_DTYPES = {v: k for k, v in DTYPE_CODES.items()}
_TORCH_TAG = {torch.float64: "f64", torch.float32: "f32", torch.float16: "f16", torch.bfloat16: "bf16",
              torch.int64: "i64", torch.int32: "i32", torch.int16: "i16", torch.int8: "i8", torch.uint8: "u8",
              torch.bool: "bool"}
_TAG_TORCH = {v: k for k, v in _TORCH_TAG.items()}
_EXTRA_TAGS = {"fp8e4m3": torch.float8_e4m3fn, "fp8e5m2": torch.float8_e5m2}


class CheckpointError(ValueError):
    pass


# ------------------------------------------------------------------ native helpers
def _fix_sigs():
    for n in ("brain_crc32", "brain_crc32_update"):
        f = _native.fn(n)
        f.restype = ctypes.c_uint32
        if n == "brain_crc32_update":
            f.argtypes = [ctypes.c_uint32, ctypes.c_void_p, ctypes.c_int64]
    for n in ("brain_format_f64", "brain_parse_f64"):
        _native.fn(n).restype = ctypes.c_int64


_sigs_done = False


def _native_ready() -> bool:
    global _sigs_done
    if not _native.available("brain_runtime"):
        return False
    if not _sigs_done:
        _fix_sigs()
        _sigs_done = True
    return True


def _buf_ptr(b) -> tuple[int, int]:
    if isinstance(b, np.ndarray):
        return b.ctypes.data, b.nbytes
    mv = memoryview(b)
    arr = np.frombuffer(mv, dtype=np.uint8)
    return arr.ctypes.data, arr.nbytes


def crc32(data, state: int | None = None) -> int:
    """IEEE CRC32 (reflected 0xEDB88320, init/final xor 0xFFFFFFFF) of bytes / buffer / ndarray."""
    if _native_ready():
        arr = data if isinstance(data, np.ndarray) else np.frombuffer(memoryview(data), dtype=np.uint8)
        arr = np.ascontiguousarray(arr)
        p, n = arr.ctypes.data, arr.nbytes
        if state is None:
            return int(_native.fn("brain_crc32")(p, n))
        return int(_native.fn("brain_crc32_update")(state, p, n))
    import zlib
    raw = bytes(memoryview(data).cast("B")) if not isinstance(data, np.ndarray) else data.tobytes()
    if state is None:
        return zlib.crc32(raw) & 0xFFFFFFFF
    return (zlib.crc32(raw, state ^ 0xFFFFFFFF) ^ 0xFFFFFFFF) & 0xFFFFFFFF


def format_f64(values: np.ndarray) -> str:
    """Comma-joined Rust ``f64::to_string`` of each value (shortest round-trip, no exponent)."""
    v = np.ascontiguousarray(values, dtype=np.float64).reshape(-1)
    if v.size == 0:
        return ""
    if _native_ready():
        cap = 350 * v.size + 16
        out = ctypes.create_string_buffer(cap)
        n = _native.fn("brain_format_f64")(v.ctypes.data, v.size, out, cap)
        if n < 0:
            raise CheckpointError("format buffer too small")
        return out.raw[:n].decode("ascii")
    return ",".join(_rust_display(float(x)) for x in v)


def parse_f64(text: str) -> np.ndarray:
    if not text:
        return np.zeros(0, dtype=np.float64)
    raw = text.encode("ascii")
    if _native_ready():
        maxn = raw.count(b",") + 1
        out = np.empty(maxn, dtype=np.float64)
        n = _native.fn("brain_parse_f64")(raw, len(raw), out.ctypes.data, maxn)
        if n < 0:
            raise CheckpointError(f"bad float token #{-1 - n}")
        return out[:n]
    return np.array([_rust_parse(t) for t in text.split(",")], dtype=np.float64)


def _rust_display(x: float) -> str:
    import math
    if math.isnan(x):
        return "NaN"
    if math.isinf(x):
        return "inf" if x > 0 else "-inf"
    if x == 0.0:
        return "-0" if math.copysign(1.0, x) < 0 else "0"
    r = repr(x)
    if "e" not in r and "E" not in r:
        return r[:-2] if r.endswith(".0") else r
    from decimal import Decimal
    s = format(Decimal(r), "f")
    return s


def _rust_parse(t: str) -> float:
    if t == "NaN":
        return float("nan")
    if t in ("inf", "+inf", "infinity"):
        return float("inf")
    if t in ("-inf", "-infinity"):
        return float("-inf")
    if not t or any(c not in "0123456789.eE+-" for c in t):
        raise CheckpointError(f"bad float token {t!r}")
    return float(t)


# ------------------------------------------------------------------ per-tensor v2
def _tag(t: torch.Tensor) -> str:
    return _TORCH_TAG.get(t.dtype, "f64")


def serialize_tensor(t: torch.Tensor, dtype_tag: str | None = None) -> bytes:
    tag = dtype_tag or _tag(t)
    payload = t.detach().to("cpu", torch.float64).contiguous().numpy().astype("<f8").tobytes()
    hdr = bytearray(MAGIC_HEADER)
    hdr += struct.pack("<I", FORMAT_VERSION_V2)
    hdr += bytes([ENDIAN_LITTLE, DTYPE_CODES.get(tag, 0), 0, 0])
    hdr += struct.pack("<I", t.dim())
    for d in t.shape:
        hdr += struct.pack("<Q", d)
    hdr += struct.pack("<I", crc32(payload))
    hdr += struct.pack("<Q", len(payload))
    return bytes(hdr) + payload


def deserialize_tensor(b: bytes, return_tag: bool = False):
    if len(b) < 16:
        raise CheckpointError("Buffer too short for tensor header")
    if b[:8] != MAGIC_HEADER:
        raise CheckpointError("Invalid magic header signature")
    version = struct.unpack_from("<I", b, 8)[0]
    if version == FORMAT_VERSION_V1:
        tag = CODE_DTYPES.get(b[12])
        if tag is None:
            raise CheckpointError(f"Unknown dtype serialization code: {b[12]}")
        ndim = struct.unpack_from("<I", b, 13)[0]
        end = 17 + 8 * ndim
        if len(b) < end:
            raise CheckpointError("V1 shape buffer truncated")
        shape = list(struct.unpack_from(f"<{ndim}Q", b, 17))
        n = int(np.prod(shape)) if shape else 1
        if len(b) < end + 8 * n:
            raise CheckpointError("V1 payload truncated")
        data = np.frombuffer(b, dtype="<f8", count=n, offset=end)
    elif version == FORMAT_VERSION_V2:
        big = b[12] == ENDIAN_BIG
        tag = CODE_DTYPES.get(b[13])
        if tag is None:
            raise CheckpointError(f"Unknown dtype serialization code: {b[13]}")
        ndim = struct.unpack_from("<I", b, 16)[0]
        end = 20 + 8 * ndim
        if len(b) < end + 12:
            raise CheckpointError("Buffer too short for tensor shape and checksum header")
        shape = list(struct.unpack_from(f"<{ndim}Q", b, 20))
        crc_expect = struct.unpack_from("<I", b, end)[0]
        plen = struct.unpack_from("<Q", b, end + 4)[0]
        start = end + 12
        if len(b) < start + plen:
            raise CheckpointError("Truncated payload buffer")
        payload = memoryview(b)[start:start + plen]
        got = crc32(payload)
        if got != crc_expect:
            raise CheckpointError(f"CRC32 mismatch: expected 0x{crc_expect:08X}, got 0x{got:08X}")
        n = int(np.prod(shape)) if shape else 1
        if plen != 8 * n:
            raise CheckpointError(f"Payload size {plen} does not match numel * 8 ({8 * n})")
        data = np.frombuffer(payload, dtype=">f8" if big else "<f8", count=n)
    else:
        raise CheckpointError(f"Unsupported format version: {version}")
    t = torch.from_numpy(np.array(data, dtype=np.float64)).reshape(shape)
    return (t, tag) if return_tag else t


def save(t: torch.Tensor, path: str) -> None:
    with open(path, "wb") as f:
        f.write(serialize_tensor(t))


def load(path: str) -> torch.Tensor:
    with open(path, "rb") as f:
        return deserialize_tensor(f.read())


# ------------------------------------------------------------------ TensorArchive
class TensorArchive:
    def __init__(self):
        self.tensors: dict[str, torch.Tensor] = {}

    def add(self, name: str, t: torch.Tensor) -> None:
        self.tensors[name] = t

    def get(self, name: str):
        return self.tensors.get(name)

    def remove(self, name: str):
        return self.tensors.pop(name, None)

    def __len__(self):
        return len(self.tensors)

    def is_empty(self) -> bool:
        return not self.tensors

    def items(self):
        return self.tensors.items()

    def serialize(self) -> bytes:
        out = bytearray(ARCHIVE_MAGIC)
        out += struct.pack("<I", len(self.tensors))
        for name in sorted(self.tensors):
            nb = name.encode()
            tb = serialize_tensor(self.tensors[name])
            out += struct.pack("<I", len(nb)) + nb + struct.pack("<Q", len(tb)) + tb
        return bytes(out)

    @staticmethod
    def deserialize(b: bytes) -> "TensorArchive":
        if len(b) < 18:
            raise CheckpointError("Archive header too short")
        if b[:14] != ARCHIVE_MAGIC:
            raise CheckpointError("Invalid archive magic")
        n = struct.unpack_from("<I", b, 14)[0]
        off = 18
        a = TensorArchive()
        for _ in range(n):
            if off + 4 > len(b):
                raise CheckpointError("Truncated archive entry")
            nl = struct.unpack_from("<I", b, off)[0]
            off += 4
            if off + nl > len(b):
                raise CheckpointError("Truncated archive name")
            name = b[off:off + nl].decode()
            off += nl
            if off + 8 > len(b):
                raise CheckpointError("Truncated tensor size in archive")
            tl = struct.unpack_from("<Q", b, off)[0]
            off += 8
            if off + tl > len(b):
                raise CheckpointError("Truncated tensor buffer in archive")
            a.add(name, deserialize_tensor(b[off:off + tl]))
            off += tl
        return a

    def save_file(self, path: str) -> None:
        with open(path, "wb") as f:
            f.write(self.serialize())

    @staticmethod
    def load_file(path: str) -> "TensorArchive":
        with open(path, "rb") as f:
            return TensorArchive.deserialize(f.read())


# ------------------------------------------------------------------ .bn BrainModelFile
@dataclass
class NodeCoord3D:
    x: int
    y: int
    z: int


@dataclass
class BrainModelFile:
    name: str
    metadata: dict = field(default_factory=dict)
    node_coords: dict = field(default_factory=dict)
    archive: TensorArchive = field(default_factory=TensorArchive)

    def with_meta(self, k: str, v: str) -> "BrainModelFile":
        self.metadata[k] = v
        return self

    def add_tensor(self, name: str, t: torch.Tensor, coord: NodeCoord3D | None = None) -> None:
        if coord is not None:
            self.node_coords[name] = coord
        self.archive.add(name, t)

    def to_bytes(self) -> bytes:
        out = bytearray(BN_MAGIC) + struct.pack("<I", 1)
        nb = self.name.encode()
        out += struct.pack("<I", len(nb)) + nb
        out += struct.pack("<I", len(self.metadata))
        for k in sorted(self.metadata):
            kb, vb = k.encode(), str(self.metadata[k]).encode()
            out += struct.pack("<I", len(kb)) + kb + struct.pack("<I", len(vb)) + vb
        out += struct.pack("<I", len(self.node_coords))
        for k in sorted(self.node_coords):
            c = self.node_coords[k]
            kb = k.encode()
            out += struct.pack("<I", len(kb)) + kb + struct.pack("<QQQ", c.x, c.y, c.z)
        ab = self.archive.serialize()
        out += struct.pack("<Q", len(ab)) + ab
        out += struct.pack("<I", crc32(bytes(out)))
        return bytes(out)

    @staticmethod
    def from_bytes(b: bytes) -> "BrainModelFile":
        if len(b) < 16:
            raise CheckpointError(".bn file buffer too short")
        if b[:8] != BN_MAGIC:
            raise CheckpointError("Invalid .bn magic header")
        expect = struct.unpack_from("<I", b, len(b) - 4)[0]
        got = crc32(memoryview(b)[:len(b) - 4])
        if got != expect:
            raise CheckpointError(f".bn CRC32 mismatch: expected 0x{expect:08X}, got 0x{got:08X}")
        off = 8
        ver = struct.unpack_from("<I", b, off)[0]
        off += 4
        if ver != 1:
            raise CheckpointError(f"Unsupported .bn format version: {ver}")

        def rd_str():
            nonlocal off
            n = struct.unpack_from("<I", b, off)[0]
            off += 4
            s = b[off:off + n].decode()
            off += n
            return s

        name = rd_str()
        meta = {}
        cnt = struct.unpack_from("<I", b, off)[0]
        off += 4
        for _ in range(cnt):
            k = rd_str()
            meta[k] = rd_str()
        cnt = struct.unpack_from("<I", b, off)[0]
        off += 4
        coords = {}
        for _ in range(cnt):
            k = rd_str()
            x, y, z = struct.unpack_from("<QQQ", b, off)
            off += 24
            coords[k] = NodeCoord3D(x, y, z)
        al = struct.unpack_from("<Q", b, off)[0]
        off += 8
        arch = TensorArchive.deserialize(b[off:off + al])
        return BrainModelFile(name, meta, coords, arch)

    def save_file(self, path: str) -> None:
        with open(path, "wb") as f:
            f.write(self.to_bytes())

    @staticmethod
    def load_file(path: str) -> "BrainModelFile":
        with open(path, "rb") as f:
            return BrainModelFile.from_bytes(f.read())


# ------------------------------------------------------------------ BRAIN_STATE_V1 text
@dataclass
class NamedTensor:
    name: str
    tensor: torch.Tensor


@dataclass
class ModelState:
    tensors: list = field(default_factory=list)
    metadata: dict = field(default_factory=dict)

    @staticmethod
    def from_module(module: torch.nn.Module, metadata: dict | None = None) -> "ModelState":
        ts = [NamedTensor(n, p.detach()) for n, p in module.named_parameters()]
        return ModelState(ts, dict(metadata or {}))

    def to_brain_bytes(self) -> bytes:
        lines = ["BRAIN_STATE_V1"]
        for k in sorted(self.metadata):
            k_s, v_s = str(k), str(self.metadata[k])
            if "|" in k_s or "\n" in k_s or "|" in v_s or "\n" in v_s:
                raise CheckpointError("metadata must not contain '|' or newlines")
            lines.append(f"meta|{k_s}|{v_s}")
        for nt in self.tensors:
            if "|" in nt.name:
                raise CheckpointError("tensor names must not contain '|'")
            shape = "x".join(str(d) for d in nt.tensor.shape)
            vals = format_f64(nt.tensor.detach().to("cpu", torch.float64).numpy())
            lines.append(f"tensor|{nt.name}|{shape}|{vals}")
        return ("\n".join(lines) + "\n").encode()

    to_bn_bytes = to_brain_bytes
    to_bytes = to_brain_bytes

    @staticmethod
    def from_brain_bytes(b: bytes) -> "ModelState":
        try:
            text = b.decode("utf-8")
        except UnicodeDecodeError as e:
            raise CheckpointError(str(e))
        lines = text.splitlines()
        if not lines or lines[0] != "BRAIN_STATE_V1":
            raise CheckpointError("missing BRAIN_STATE_V1 header")
        st = ModelState()
        for line in lines[1:]:
            parts = line.split("|")
            if len(parts) == 3 and parts[0] == "meta":
                st.metadata[parts[1]] = parts[2]
            elif len(parts) == 4 and parts[0] == "tensor":
                _, name, shape, vals = parts
                try:
                    dims = [int(x) for x in shape.split("x")] if shape else []
                except ValueError as e:
                    raise CheckpointError(str(e))
                data = parse_f64(vals)
                n = int(np.prod(dims)) if dims else 1
                if data.size != n and not (data.size == 0 and n == 0):
                    raise CheckpointError(f"tensor {name}: {data.size} values for shape {dims}")
                st.tensors.append(NamedTensor(name, torch.from_numpy(data.copy()).reshape(dims)))
            else:
                raise CheckpointError(f"invalid state line: {line[:80]}")
        return st

    from_bn_bytes = from_brain_bytes
    from_bytes = from_brain_bytes

    def save_file(self, path: str) -> None:
        d = os.path.dirname(path)
        if d:
            os.makedirs(d, exist_ok=True)
        with open(path, "wb") as f:
            f.write(self.to_brain_bytes())

    @staticmethod
    def load_file(path: str) -> "ModelState":
        with open(path, "rb") as f:
            return ModelState.from_brain_bytes(f.read())

    def parameters(self) -> list:
        return [nt.tensor for nt in self.tensors]

    def load_into(self, module: torch.nn.Module, strict: bool = True) -> None:
        params = dict(module.named_parameters())
        seen = set()
        with torch.no_grad():
            for nt in self.tensors:
                p = params.get(nt.name)
                if p is None:
                    if strict:
                        raise CheckpointError(f"unexpected tensor {nt.name}")
                    continue
                p.copy_(nt.tensor.to(p.dtype).reshape(p.shape))
                seen.add(nt.name)
        if strict and seen != set(params):
            raise CheckpointError(f"missing tensors: {sorted(set(params) - seen)[:5]}")


# ------------------------------------------------------------------ binary .brain v2 (large models)
def _tensor_tag(t: torch.Tensor) -> str:
    for k, v in _EXTRA_TAGS.items():
        if t.dtype == v:
            return k
    return _TORCH_TAG[t.dtype]


def _tag_dtype(tag: str) -> torch.dtype:
    return _EXTRA_TAGS.get(tag) or _TAG_TORCH[tag]


def save_brain_v2(path: str, tensors: dict, metadata: dict | None = None) -> None:
    """Write named tensors in native dtype: magic, u32 version, u64 header length, JSON header
    (metadata + per-tensor name/dtype/shape/offset/nbytes/crc32), payloads aligned to 64 bytes,
    and a final u32 CRC32 of the header. Order is sorted by name, so output is deterministic."""
    entries = []
    off = 0
    blobs = []
    for name in sorted(tensors):
        t = tensors[name].detach()
        host = t.to("cpu").contiguous()
        raw = host.view(torch.uint8).numpy() if host.numel() else np.zeros(0, dtype=np.uint8)
        raw = raw.reshape(-1)
        off = -(-off // 64) * 64
        entries.append({"name": name, "dtype": _tensor_tag(t), "shape": list(t.shape), "offset": off,
                        "nbytes": int(raw.nbytes), "crc32": crc32(raw)})
        blobs.append((off, raw))
        off += raw.nbytes
    header = json.dumps({"metadata": metadata or {}, "tensors": entries}, sort_keys=True).encode()
    base = 8 + 4 + 8 + len(header) + 4
    base = -(-base // 64) * 64
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        f.write(CKPT_V2_MAGIC + struct.pack("<I", 2) + struct.pack("<Q", len(header)) + header)
        f.write(struct.pack("<I", crc32(header)))
        f.write(b"\0" * (base - f.tell()))
        for o, raw in blobs:
            f.seek(base + o)
            f.write(raw.tobytes())
    os.replace(tmp, path)


def load_brain_v2(path: str, device="cpu", verify: bool = True) -> tuple[dict, dict]:
    with open(path, "rb") as f:
        data = f.read()
    if data[:8] != CKPT_V2_MAGIC:
        raise CheckpointError("not a BRAINCK2 file")
    ver = struct.unpack_from("<I", data, 8)[0]
    if ver != 2:
        raise CheckpointError(f"unsupported BRAINCK2 version {ver}")
    hl = struct.unpack_from("<Q", data, 12)[0]
    header = data[20:20 + hl]
    hcrc = struct.unpack_from("<I", data, 20 + hl)[0]
    if crc32(header) != hcrc:
        raise CheckpointError("BRAINCK2 header CRC32 mismatch")
    meta = json.loads(header)
    base = -(-(20 + hl + 4) // 64) * 64
    out = {}
    for e in meta["tensors"]:
        raw = np.frombuffer(data, dtype=np.uint8, count=e["nbytes"], offset=base + e["offset"])
        if verify and crc32(raw) != e["crc32"]:
            raise CheckpointError(f"CRC32 mismatch in tensor {e['name']}")
        dt = _tag_dtype(e["dtype"])
        t = torch.from_numpy(raw.copy()).view(dt).reshape(e["shape"])
        out[e["name"]] = t.to(device)
    return out, meta["metadata"]
