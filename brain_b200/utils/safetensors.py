"""safetensors reader / writer (interop with the Hugging Face format; reference brain-export
crates/brain-export/src/safetensors.rs:27-195).

Layout: u64 little-endian header length, a JSON header mapping names to {dtype, shape,
data_offsets} plus an optional ``__metadata__`` string map, then the raw little-endian tensor bytes.
"""
from __future__ import annotations

import json
import struct

import numpy as np
import torch

_DT = {torch.float64: "F64", torch.float32: "F32", torch.float16: "F16", torch.bfloat16: "BF16", torch.int64: "I64",
       torch.int32: "I32", torch.int16: "I16", torch.int8: "I8", torch.uint8: "U8", torch.bool: "BOOL",
       torch.float8_e4m3fn: "F8_E4M3", torch.float8_e5m2: "F8_E5M2"}
_TD = {v: k for k, v in _DT.items()}


def save_safetensors(path: str, tensors: dict, metadata: dict | None = None) -> None:
    header, blobs, off = {}, [], 0
    for name in sorted(tensors):
        t = tensors[name].detach().to("cpu").contiguous()
        raw = t.view(torch.uint8).numpy().tobytes() if t.numel() else b""
        header[name] = {"dtype": _DT[t.dtype], "shape": list(t.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    hb = json.dumps(header, separators=(",", ":")).encode()
    hb += b" " * ((8 - len(hb) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hb)) + hb)
        for b in blobs:
            f.write(b)


def load_safetensors(path: str, device="cpu") -> tuple[dict, dict]:
    with open(path, "rb") as f:
        data = f.read()
    n = struct.unpack_from("<Q", data, 0)[0]
    header = json.loads(data[8:8 + n])
    meta = header.pop("__metadata__", {})
    base = 8 + n
    out = {}
    for name, e in header.items():
        s, t = e["data_offsets"]
        raw = np.frombuffer(data, dtype=np.uint8, count=t - s, offset=base + s).copy()
        out[name] = torch.from_numpy(raw).view(_TD[e["dtype"]]).reshape(e["shape"]).to(device)
    return out, meta
