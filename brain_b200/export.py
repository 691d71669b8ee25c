"""Model export: format options, per-format op-support tables, ONNX / WebNN / Core ML / TFLite
exporters for the graph IR, an uncompressed ZIP packer, quantised-weight export, ``.bn`` <->
safetensors conversion and numerical verification.

Reference: crates/brain-export (core.rs:7-45 ``ExportFormat`` / ``ExportOptions`` / ``ExportError``;
ops_supported.rs; onnx/ops.rs, tflite/ops.rs, coreml/ops.rs, webnn/ops.rs op tables; zip.rs:8-70;
verify.rs:9; export_all.rs:10-40; quant_export.rs:7-30; convert.rs:10-80). The reference's TFLite,
Core ML and WebNN exporters write nothing; here WebNN writes a JSON graph descriptor (operands,
operations, base64 constants), Core ML writes a package (ZIP) holding a MIL-style program text and a
weight blob, and TFLite writes a JSON model description keyed by TFLite builtin operator names (the
binary flatbuffer is not produced). ONNX is the binary ModelProto of ``brain_b200.onnx``.
"""
from __future__ import annotations

import base64
import enum
import io
import json
import os
import struct
import zipfile
from dataclasses import dataclass, field

import torch

from . import onnx as _onnx
from .graph import GraphInterpreter, GraphIr


class ExportFormat(enum.Enum):
    ONNX = "onnx"
    TFLITE = "tflite"
    COREML = "coreml"
    WEBNN = "webnn"


@dataclass
class ExportOptions:
    format: ExportFormat = ExportFormat.ONNX
    opset_version: int = _onnx.OPSET
    quantize: bool = False
    verify: bool = True


class ExportError(RuntimeError):
    pass


# graph op -> target op name (None: not expressible in that format)
OP_TABLES = {
    ExportFormat.ONNX: {**_onnx._STD, **{k: f"{_onnx.CUSTOM_DOMAIN}.{k}" for k in _onnx._CUSTOM}},
    ExportFormat.TFLITE: {"add": "ADD", "sub": "SUB", "mul": "MUL", "div": "DIV", "relu": "RELU", "tanh": "TANH",
                          "sigmoid": "LOGISTIC", "exp": "EXP", "log": "LOG", "neg": "NEG", "sqrt": "SQRT",
                          "rsqrt": "RSQRT", "abs": "ABS", "maximum": "MAXIMUM", "minimum": "MINIMUM", "pow": "POW",
                          "matmul": "BATCH_MATMUL", "linear": "FULLY_CONNECTED", "softmax": "SOFTMAX",
                          "log_softmax": "LOG_SOFTMAX", "reshape": "RESHAPE", "transpose": "TRANSPOSE",
                          "concat": "CONCATENATION", "sum": "SUM", "mean": "MEAN", "gelu": "GELU",
                          "identity": None, "layer_norm": None, "rms_norm": None, "swiglu": None, "silu": None,
                          "constant_scale": "MUL"},
    ExportFormat.COREML: {"add": "add", "sub": "sub", "mul": "mul", "div": "real_div", "relu": "relu",
                          "tanh": "tanh", "sigmoid": "sigmoid", "exp": "exp", "log": "log", "neg": "mul",
                          "sqrt": "sqrt", "rsqrt": "rsqrt", "abs": "abs", "maximum": "maximum", "minimum": "minimum",
                          "pow": "pow", "matmul": "matmul", "linear": "linear", "softmax": "softmax",
                          "log_softmax": "log_softmax", "reshape": "reshape", "transpose": "transpose",
                          "concat": "concat", "sum": "reduce_sum", "mean": "reduce_mean", "gelu": "gelu",
                          "layer_norm": "layer_norm", "silu": "silu", "identity": "identity", "rms_norm": None,
                          "swiglu": None, "constant_scale": "mul"},
    ExportFormat.WEBNN: {"add": "add", "sub": "sub", "mul": "mul", "div": "div", "relu": "relu", "tanh": "tanh",
                         "sigmoid": "sigmoid", "exp": "exp", "log": "log", "neg": "neg", "sqrt": "sqrt",
                         "rsqrt": None, "abs": "abs", "maximum": "max", "minimum": "min", "pow": "pow",
                         "matmul": "matmul", "linear": "gemm", "softmax": "softmax", "log_softmax": None,
                         "reshape": "reshape", "transpose": "transpose", "concat": "concat", "sum": "reduceSum",
                         "mean": "reduceMean", "gelu": "gelu", "layer_norm": "layerNormalization",
                         "identity": "identity", "rms_norm": None, "swiglu": None, "silu": None,
                         "constant_scale": "mul"},
}


@dataclass
class SupportedOpsReport:
    format: ExportFormat
    supported: list = field(default_factory=list)
    unsupported: list = field(default_factory=list)

    def ok(self) -> bool:
        return not self.unsupported


def supported_ops_report(g: GraphIr, fmt: ExportFormat) -> SupportedOpsReport:
    rep = SupportedOpsReport(fmt)
    table = OP_TABLES[fmt]
    for n in g.nodes:
        (rep.supported if table.get(n.op) else rep.unsupported).append(n.op)
    return rep


def _require(g: GraphIr, fmt: ExportFormat) -> None:
    rep = supported_ops_report(g, fmt)
    if not rep.ok():
        raise ExportError(f"{fmt.value}: unsupported ops {sorted(set(rep.unsupported))}")


def _raw(t: torch.Tensor) -> bytes:
    t = t.detach().cpu().contiguous().reshape(-1)
    return t.view(torch.uint8).numpy().tobytes() if t.numel() else b""


def _b64(t: torch.Tensor) -> str:
    return base64.b64encode(_raw(t)).decode()


def export_webnn(g: GraphIr) -> str:
    """WebNN-style graph descriptor: inputs / constants (base64 little-endian) / operations / outputs."""
    _require(g, ExportFormat.WEBNN)
    table = OP_TABLES[ExportFormat.WEBNN]
    name = lambda vid: f"v{vid}"  # noqa: E731
    desc = {"inputs": [{"name": name(i), "dataType": g.values[i].dtype, "shape": list(g.values[i].shape or ())}
                       for i in g.inputs],
            "constants": [{"name": name(v), "dataType": str(x.constant.dtype).replace("torch.", ""),
                           "shape": list(x.constant.shape), "data": _b64(x.constant)}
                          for v, x in g.values.items() if x.constant is not None],
            "operations": [], "outputs": [name(o) for o in g.outputs]}
    for n in g.nodes:
        op, opts = table[n.op], dict(n.attrs)
        if n.op == "linear":
            opts = {"bTranspose": True}
        desc["operations"].append({"op": op, "inputs": [name(i) for i in n.inputs],
                                   "outputs": [name(o) for o in n.outputs], "options": opts})
    return json.dumps(desc, sort_keys=True)


def export_tflite_json(g: GraphIr) -> str:
    _require(g, ExportFormat.TFLITE)
    table = OP_TABLES[ExportFormat.TFLITE]
    codes = sorted({table[n.op] for n in g.nodes})
    tensors = {vid: i for i, vid in enumerate(g.values)}
    buffers = [""] + [_b64(v.constant) for v in g.values.values() if v.constant is not None]
    bidx, k = {}, 1
    for vid, v in g.values.items():
        if v.constant is not None:
            bidx[vid] = k
            k += 1
    model = {"version": 3, "operator_codes": [{"builtin_code": c} for c in codes],
             "subgraphs": [{"tensors": [{"name": v.name, "shape": list(v.shape or ()), "type": v.dtype.upper(),
                                         "buffer": bidx.get(vid, 0)} for vid, v in g.values.items()],
                            "inputs": [tensors[i] for i in g.inputs], "outputs": [tensors[o] for o in g.outputs],
                            "operators": [{"opcode_index": codes.index(table[n.op]),
                                           "inputs": [tensors[i] for i in n.inputs],
                                           "outputs": [tensors[o] for o in n.outputs]} for n in g.nodes]}],
             "buffers": [{"data": b} for b in buffers]}
    return json.dumps(model)


def export_coreml_package(g: GraphIr) -> bytes:
    """ZIP with ``model.mil`` (one ``%out = op(inputs)`` line per node, constants referenced by blob
    offset), ``weights.bin`` (concatenated little-endian constants) and ``manifest.json``."""
    _require(g, ExportFormat.COREML)
    table = OP_TABLES[ExportFormat.COREML]
    blob, offsets = bytearray(), {}
    for vid, v in g.values.items():
        if v.constant is not None:
            offsets[vid] = len(blob)
            blob += _raw(v.constant)
    lines = ["program(1.0)", "func main(" + ", ".join(f"%v{i}: tensor<{g.values[i].dtype}, {list(g.values[i].shape or ())}>"
                                                  for i in g.inputs) + ") {"]
    for vid, off in offsets.items():
        v = g.values[vid]
        lines.append(f"  %v{vid} = const(blob=weights.bin, offset={off}, dtype={v.dtype}, shape={list(v.shape)})")
    for n in g.nodes:
        args = ", ".join(f"%v{i}" for i in n.inputs)
        attrs = "".join(f", {k}={v}" for k, v in sorted(n.attrs.items()))
        lines.append(f"  %v{n.outputs[0]} = {table[n.op]}({args}{attrs})")
    lines.append("} -> (" + ", ".join(f"%v{o}" for o in g.outputs) + ")")
    return create_zip_archive([("model.mil", "\n".join(lines).encode()), ("weights.bin", bytes(blob)),
                               ("manifest.json", json.dumps({"name": g.name, "format": "brain-mil-1"}).encode())])


def create_zip_archive(files) -> bytes:
    """Stored (uncompressed) ZIP of (name, bytes) pairs."""
    buf = io.BytesIO()
    with zipfile.ZipFile(buf, "w", compression=zipfile.ZIP_STORED) as z:
        for name, data in files:
            z.writestr(zipfile.ZipInfo(name, date_time=(1980, 1, 1, 0, 0, 0)), data)
    return buf.getvalue()


def verify_export(actual: torch.Tensor, expected: torch.Tensor, tol: float) -> None:
    if actual.shape != expected.shape:
        raise ExportError(f"shape mismatch {tuple(actual.shape)} vs {tuple(expected.shape)}")
    err = float((actual.double() - expected.double()).abs().max()) if actual.numel() else 0.0
    if err > tol:
        raise ExportError(f"verification failed: max abs error {err:.3g} > {tol:.3g}")


@dataclass
class ExportSummary:
    files: dict = field(default_factory=dict)
    skipped: dict = field(default_factory=dict)


def export_all(g: GraphIr, out_dir: str, example_inputs=None, tol: float = 1e-5) -> ExportSummary:
    """Writes every format the graph's ops allow; with ``example_inputs`` the ONNX file is re-imported
    and checked against the interpreter."""
    os.makedirs(out_dir, exist_ok=True)
    s = ExportSummary()
    writers = {ExportFormat.ONNX: ("model.onnx", lambda: _onnx.export_onnx(g)),
               ExportFormat.WEBNN: ("model.webnn.json", lambda: export_webnn(g).encode()),
               ExportFormat.TFLITE: ("model.tflite.json", lambda: export_tflite_json(g).encode()),
               ExportFormat.COREML: ("model.mlpackage.zip", lambda: export_coreml_package(g))}
    for fmt, (fname, fn) in writers.items():
        try:
            data = fn()
        except ExportError as e:
            s.skipped[fmt.value] = str(e)
            continue
        path = os.path.join(out_dir, fname)
        with open(path, "wb") as f:
            f.write(data)
        s.files[fmt.value] = path
    if example_inputs is not None and "onnx" in s.files:
        with open(s.files["onnx"], "rb") as f:
            back = _onnx.import_onnx(f.read())
        for a, b in zip(GraphInterpreter().run(back, list(example_inputs)), GraphInterpreter().run(g, list(example_inputs))):
            verify_export(a, b, tol)
    return s


@dataclass
class QuantExportConfig:
    per_channel: bool = True
    bit_width: int = 8


def export_quantized_safetensors(tensors: dict, path: str, config: QuantExportConfig | None = None) -> dict:
    """2-D float tensors -> symmetric int8 (per output channel or per tensor) with f32 scales stored as
    ``<name>.scale``; other tensors are stored as they are. Returns the max reconstruction error."""
    from .quantization import QuantDType, QuantScheme, quantize_tensor
    from .utils.safetensors import save_safetensors

    c = config or QuantExportConfig()
    if c.bit_width != 8:
        raise ExportError("only 8-bit export is supported")
    out, err = {}, {}
    for k, t in tensors.items():
        if t.is_floating_point() and t.dim() == 2:
            scheme = QuantScheme.PER_CHANNEL if c.per_channel else QuantScheme.PER_TENSOR
            q, scale, _ = quantize_tensor(t, QuantDType.INT8, True, scheme, 0)
            out[k] = q.to(torch.int8).reshape(t.shape)
            out[k + ".scale"] = scale.float().reshape(-1)
            recon = out[k].float() * (out[k + ".scale"][:, None] if c.per_channel else out[k + ".scale"])
            err[k] = float((recon - t.float()).abs().max())
        else:
            out[k] = t
    save_safetensors(path, out, {"format": "brain-int8", "per_channel": str(c.per_channel)})
    return err


@dataclass
class ConversionReport:
    num_tensors: int
    format_from: str
    format_to: str


def convert_bn_to_safetensors(bn_path: str, st_path: str) -> ConversionReport:
    from .checkpoint.formats import BrainModelFile
    from .utils.safetensors import save_safetensors

    m = BrainModelFile.load_file(bn_path)
    tensors = dict(m.archive.items())
    save_safetensors(st_path, tensors, {"name": m.name, **{f"meta.{k}": v for k, v in m.metadata.items()}})
    return ConversionReport(len(tensors), "bn", "safetensors")


def convert_safetensors_to_bn(st_path: str, bn_path: str, name: str = "model") -> ConversionReport:
    from .checkpoint.formats import BrainModelFile
    from .utils.safetensors import load_safetensors

    tensors, meta = load_safetensors(st_path)
    m = BrainModelFile(meta.get("name", name) if meta else name)
    for k, v in (meta or {}).items():
        if k.startswith("meta."):
            m.with_meta(k[5:], v)
    for k, t in tensors.items():
        m.add_tensor(k, t)
    m.save_file(bn_path)
    return ConversionReport(len(tensors), "safetensors", "bn")


# ------------------------------------------------------------------ exporter objects and the builder
# crates/brain-export/src: onnx/mod.rs, tflite/mod.rs, coreml/mod.rs, webnn/mod.rs (one exporter per
# format), builder.rs (ExportBuilder), model/mod.rs (ModelExporter), ops.rs (is_op_supported),
# common/dtype_map.rs (map_dtype_to_onnx / map_dtype_to_tflite), name_gen.rs (sanitize_name),
# utils.rs (align4, encode_uleb128), safetensors.rs (SafetensorsArchive).

class _Exporter:
    FORMAT: ExportFormat

    def export(self, g: GraphIr):
        raise NotImplementedError

    def save(self, g: GraphIr, path: str) -> str:
        data = self.export(g)
        mode = "wb" if isinstance(data, (bytes, bytearray)) else "w"
        with open(path, mode) as f:
            f.write(data)
        return path

    def supports(self, g: GraphIr) -> bool:
        return all(n.op in OP_TABLES[self.FORMAT] for n in g.nodes)


class OnnxExporter(_Exporter):
    FORMAT = ExportFormat.ONNX

    def export(self, g):
        return _onnx.export_onnx(g)

    def supports(self, g):
        return True


class TfliteExporter(_Exporter):
    FORMAT = ExportFormat.TFLITE

    def export(self, g):
        return export_tflite_json(g)


class CoreMlExporter(_Exporter):
    FORMAT = ExportFormat.COREML

    def export(self, g):
        return export_coreml_package(g)


class WebnnExporter(_Exporter):
    FORMAT = ExportFormat.WEBNN

    def export(self, g):
        return export_webnn(g)


_EXPORTERS = {ExportFormat.ONNX: OnnxExporter, ExportFormat.TFLITE: TfliteExporter,
              ExportFormat.COREML: CoreMlExporter, ExportFormat.WEBNN: WebnnExporter}


def is_op_supported(op: str, fmt: ExportFormat) -> bool:
    return fmt == ExportFormat.ONNX or op in OP_TABLES[fmt]


class ExportBuilder:
    """``ExportBuilder(graph).format("webnn").build().save(path)``: picks the exporter for a format."""

    def __init__(self, g: GraphIr):
        self.g, self.fmt = g, ExportFormat.ONNX

    def format(self, fmt) -> "ExportBuilder":
        self.fmt = ExportFormat(fmt) if not isinstance(fmt, ExportFormat) else fmt
        return self

    def build(self) -> _Exporter:
        ex = _EXPORTERS[self.fmt]()
        if not ex.supports(self.g):
            bad = sorted({n.op for n in self.g.nodes if not is_op_supported(n.op, self.fmt)})
            raise ExportError(f"{self.fmt.value} cannot express: {', '.join(bad)}")
        return ex


def export_model(g: GraphIr, fmt, path: str) -> str:
    return ExportBuilder(g).format(fmt).build().save(g, path)


_ONNX_DTYPES = {torch.float32: 1, torch.uint8: 2, torch.int8: 3, torch.int16: 5, torch.int32: 6, torch.int64: 7,
                torch.bool: 9, torch.float16: 10, torch.float64: 11, torch.bfloat16: 16,
                torch.float8_e4m3fn: 17, torch.float8_e5m2: 19}
_TFLITE_DTYPES = {torch.float32: 0, torch.float16: 1, torch.int32: 2, torch.uint8: 3, torch.int64: 4, torch.bool: 6,
                  torch.int16: 7, torch.int8: 9, torch.float64: 10}


def map_dtype_to_onnx(dtype: torch.dtype) -> int:
    return _ONNX_DTYPES[dtype]


def map_dtype_to_tflite(dtype: torch.dtype) -> int:
    return _TFLITE_DTYPES[dtype]


def sanitize_name(name: str) -> str:
    import re
    s = re.sub(r"[^0-9A-Za-z_]", "_", name)
    return s if s and not s[0].isdigit() else "_" + s


def align4(n: int) -> int:
    return (n + 3) & ~3


def encode_uleb128(v: int) -> bytes:
    out = bytearray()
    while True:
        b = v & 0x7F
        v >>= 7
        out.append(b | (0x80 if v else 0))
        if not v:
            return bytes(out)


class SafetensorsArchive:
    """Named tensors written to / read from one ``.safetensors`` file."""

    def __init__(self, tensors: dict | None = None, metadata: dict | None = None):
        self.tensors, self.metadata = dict(tensors or {}), dict(metadata or {})

    def add(self, name: str, t: torch.Tensor) -> "SafetensorsArchive":
        self.tensors[name] = t
        return self

    def save(self, path: str) -> None:
        from .utils.safetensors import save_safetensors
        save_safetensors(path, self.tensors, {k: str(v) for k, v in self.metadata.items()})

    @classmethod
    def load(cls, path: str) -> "SafetensorsArchive":
        from .utils.safetensors import load_safetensors
        t, m = load_safetensors(path)
        return cls(t, m)
