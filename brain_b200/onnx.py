"""ONNX export and import of the graph IR with a self-contained protobuf codec (no ``onnx`` package).

Reference: crates/brain-onnx (hand-written protobuf decoder/encoder proto/*.rs, import
import/onnx2graph.rs, export graph2onnx.rs, checker eval/checker.rs) and the ONNX mapping tables of
crates/brain-export (onnx/ops.rs).

The wire format is the public protobuf encoding (varint / 64-bit / length-delimited / 32-bit fields)
and the message layouts are those of the public ``onnx.proto`` (ModelProto, GraphProto, NodeProto,
AttributeProto, TensorProto, ValueInfoProto); both have to be alike for other ONNX tools to read the
files. Ops with an ONNX standard equivalent map to it (opset 20); the framework's fused ops
(``rms_norm``, ``swiglu``, ``silu``, ``constant_scale``) use the ``ai.brain`` domain.
"""
from __future__ import annotations

import struct

import torch

from .graph import GraphError, GraphIr

OPSET = 20
CUSTOM_DOMAIN = "ai.brain"

_ONNX_DTYPE = {torch.float32: 1, torch.uint8: 2, torch.int8: 3, torch.int16: 5, torch.int32: 6, torch.int64: 7,
               torch.bool: 9, torch.float16: 10, torch.float64: 11, torch.bfloat16: 16}
_TORCH_DTYPE = {v: k for k, v in _ONNX_DTYPE.items()}

_STD = {"relu": "Relu", "tanh": "Tanh", "sigmoid": "Sigmoid", "exp": "Exp", "log": "Log", "neg": "Neg",
        "sqrt": "Sqrt", "abs": "Abs", "add": "Add", "sub": "Sub", "mul": "Mul", "div": "Div", "pow": "Pow",
        "maximum": "Max", "minimum": "Min", "matmul": "MatMul", "softmax": "Softmax", "log_softmax": "LogSoftmax",
        "concat": "Concat", "identity": "Identity", "gelu": "Gelu", "layer_norm": "LayerNormalization",
        "linear": "Gemm", "transpose": "Transpose", "reshape": "Reshape", "sum": "ReduceSum", "mean": "ReduceMean",
        "rsqrt": "Reciprocal"}
_CUSTOM = {"rms_norm", "swiglu", "silu", "constant_scale"}


# ------------------------------------------------------------------ protobuf wire format
def _varint(n: int) -> bytes:
    n &= (1 << 64) - 1
    out = bytearray()
    while True:
        b = n & 0x7F
        n >>= 7
        if n:
            out.append(b | 0x80)
        else:
            out.append(b)
            return bytes(out)


def _key(field: int, wire: int) -> bytes:
    return _varint((field << 3) | wire)


def _f_varint(field: int, v: int) -> bytes:
    return _key(field, 0) + _varint(v)


def _f_bytes(field: int, b: bytes) -> bytes:
    return _key(field, 2) + _varint(len(b)) + b


def _f_str(field: int, s: str) -> bytes:
    return _f_bytes(field, s.encode())


def _f_float(field: int, f: float) -> bytes:
    return _key(field, 5) + struct.pack("<f", f)


def _read_varint(b: bytes, p: int):
    n = shift = 0
    while True:
        c = b[p]
        p += 1
        n |= (c & 0x7F) << shift
        if not c & 0x80:
            return n, p
        shift += 7


def parse(b: bytes) -> dict[int, list]:
    """Decodes one message into {field: [raw values]} (ints for varint / fixed, bytes otherwise)."""
    out: dict[int, list] = {}
    p = 0
    while p < len(b):
        k, p = _read_varint(b, p)
        field, wire = k >> 3, k & 7
        if wire == 0:
            v, p = _read_varint(b, p)
        elif wire == 1:
            v = b[p:p + 8]
            p += 8
        elif wire == 2:
            n, p = _read_varint(b, p)
            v = b[p:p + n]
            p += n
        elif wire == 5:
            v = b[p:p + 4]
            p += 4
        else:
            raise GraphError(f"unsupported protobuf wire type {wire}")
        out.setdefault(field, []).append(v)
    return out


def _signed(n: int) -> int:
    return n - (1 << 64) if n >= 1 << 63 else n


# ------------------------------------------------------------------ message builders
def _tensor_proto(name: str, t: torch.Tensor) -> bytes:
    t = t.detach().cpu().contiguous()
    body = b"".join(_f_varint(1, d) for d in t.shape)
    body += _f_varint(2, _ONNX_DTYPE[t.dtype]) + _f_str(8, name)
    raw = t.view(torch.int16).numpy().tobytes() if t.dtype == torch.bfloat16 else t.numpy().tobytes()
    return body + _f_bytes(9, raw)


def _value_info(name: str, shape, dtype: str) -> bytes:
    dims = b"".join(_f_bytes(1, _f_varint(1, int(d))) for d in (shape or ()))
    tensor_type = _f_varint(1, _ONNX_DTYPE[getattr(torch, dtype)]) + _f_bytes(2, dims)
    return _f_str(1, name) + _f_bytes(2, _f_bytes(1, tensor_type))


def _attr(name: str, v) -> bytes:
    b = _f_str(1, name)
    if isinstance(v, bool) or isinstance(v, int):
        return b + _f_varint(3, int(v)) + _f_varint(20, 2)
    if isinstance(v, float):
        return b + _f_float(2, v) + _f_varint(20, 1)
    if isinstance(v, str):
        return b + _f_bytes(4, v.encode()) + _f_varint(20, 3)
    if isinstance(v, (list, tuple)) and all(isinstance(x, int) for x in v):
        return b + b"".join(_f_varint(8, x) for x in v) + _f_varint(20, 7)
    raise GraphError(f"unsupported attribute {name}={v!r}")


def _node(op_type: str, inputs, outputs, name: str, attrs: dict, domain: str = "") -> bytes:
    b = b"".join(_f_str(1, i) for i in inputs) + b"".join(_f_str(2, o) for o in outputs)
    b += _f_str(3, name) + _f_str(4, op_type)
    b += b"".join(_f_bytes(5, _attr(k, v)) for k, v in sorted(attrs.items()))
    if domain:
        b += _f_str(7, domain)
    return b


def export_onnx(g: GraphIr, path: str | None = None) -> bytes:
    """Serialises the graph as an ONNX ModelProto. Constants become initializers."""
    names = {vid: f"v{vid}_{v.name}".replace(" ", "_") for vid, v in g.values.items()}
    nodes, extra_init = [], []
    for n in g.nodes:
        ins, outs = [names[i] for i in n.inputs], [names[o] for o in n.outputs]
        a = dict(n.attrs)
        if n.op in _CUSTOM:
            nodes.append(_node(n.op, ins, outs, f"n{n.id}", {k: v for k, v in a.items()}, CUSTOM_DOMAIN))
            continue
        op = _STD.get(n.op)
        if op is None:
            raise GraphError(f"no ONNX mapping for {n.op}")
        attrs = {}
        if n.op == "linear":
            attrs = {"transB": 1}
        elif n.op in ("softmax", "log_softmax"):
            attrs = {"axis": int(a.get("dim", -1))}
        elif n.op == "concat":
            attrs = {"axis": int(a.get("dim", -1))}
        elif n.op == "gelu":
            attrs = {"approximate": a.get("approximate", "tanh")}
        elif n.op == "layer_norm":
            attrs = {"axis": -1, "epsilon": float(a.get("eps", 1e-5))}
        elif n.op == "transpose":
            rank = len(g.values[n.inputs[0]].shape or ())
            if rank == 0:
                raise GraphError("transpose export needs a known input rank")
            perm = list(range(rank))
            d0, d1 = a.get("dim0", -2) % rank, a.get("dim1", -1) % rank
            perm[d0], perm[d1] = perm[d1], perm[d0]
            attrs = {"perm": perm}
        elif n.op == "reshape":
            sname = f"{outs[0]}_shape"
            extra_init.append(_tensor_proto(sname, torch.tensor(list(a["shape"]), dtype=torch.int64)))
            ins = ins + [sname]
        elif n.op in ("sum", "mean"):
            attrs = {"keepdims": int(bool(a.get("keepdim", False)))}
            if "dim" in a:
                dims = a["dim"] if isinstance(a["dim"], (list, tuple)) else [a["dim"]]
                aname = f"{outs[0]}_axes"
                extra_init.append(_tensor_proto(aname, torch.tensor(list(dims), dtype=torch.int64)))
                ins = ins + [aname]
        elif n.op == "rsqrt":
            # Reciprocal(Sqrt(x)): emit the Sqrt as its own node
            mid = f"{outs[0]}_sqrt"
            nodes.append(_node("Sqrt", ins, [mid], f"n{n.id}_sqrt", {}))
            ins = [mid]
        nodes.append(_node(op, ins, outs, f"n{n.id}", attrs))
    graph = b"".join(_f_bytes(1, x) for x in nodes) + _f_str(2, g.name)
    inits = [_tensor_proto(names[vid], v.constant) for vid, v in g.values.items() if v.constant is not None]
    graph += b"".join(_f_bytes(5, x) for x in inits + extra_init)
    graph += b"".join(_f_bytes(11, _value_info(names[i], g.values[i].shape, g.values[i].dtype)) for i in g.inputs)
    graph += b"".join(_f_bytes(12, _value_info(names[o], g.values[o].shape, g.values[o].dtype or "float32"))
                      for o in g.outputs)
    model = _f_varint(1, 9) + _f_str(2, "brain_b200") + _f_str(3, "1")
    model += _f_bytes(7, graph)
    model += _f_bytes(8, _f_str(1, "") + _f_varint(2, OPSET)) + _f_bytes(8, _f_str(1, CUSTOM_DOMAIN) + _f_varint(2, 1))
    if path:
        with open(path, "wb") as f:
            f.write(model)
    return model


# ------------------------------------------------------------------ import
def _decode_tensor(b: bytes):
    m = parse(b)
    dims = [_signed(d) for d in m.get(1, [])]
    dt = _TORCH_DTYPE[m[2][0]]
    name = m[8][0].decode() if 8 in m else ""
    if 9 in m:
        raw = m[9][0]
        if dt == torch.bfloat16:
            t = torch.frombuffer(bytearray(raw), dtype=torch.int16).view(torch.bfloat16)
        else:
            t = torch.frombuffer(bytearray(raw), dtype=dt) if raw else torch.zeros(0, dtype=dt)
    elif 4 in m:
        t = torch.tensor([struct.unpack("<f", x)[0] for x in m[4]], dtype=torch.float32)
    elif 7 in m:
        t = torch.tensor([_signed(x) for x in m[7]], dtype=torch.int64)
    else:
        t = torch.zeros(0, dtype=dt)
    return name, t.reshape(dims).clone()


def _decode_attr(b: bytes):
    m = parse(b)
    name, typ = m[1][0].decode(), m.get(20, [0])[0]
    if typ == 1:
        return name, struct.unpack("<f", m[2][0])[0]
    if typ == 2:
        return name, _signed(m[3][0])
    if typ == 3:
        return name, m[4][0].decode()
    if typ == 7:
        vals = []
        for x in m.get(8, []):
            if isinstance(x, (bytes, bytearray)):  # packed encoding
                p = 0
                while p < len(x):
                    v, p = _read_varint(x, p)
                    vals.append(_signed(v))
            else:
                vals.append(_signed(x))
        return name, vals
    raise GraphError(f"unsupported attribute type {typ} for {name}")


def _decode_value_info(b: bytes):
    m = parse(b)
    name = m[1][0].decode()
    shape, dtype = None, "float32"
    if 2 in m:
        tt = parse(parse(m[2][0])[1][0])
        dtype = str(_TORCH_DTYPE[tt[1][0]]).replace("torch.", "")
        if 2 in tt:
            shape = tuple(_signed(parse(d).get(1, [0])[0]) for d in parse(tt[2][0]).get(1, []))
    return name, shape, dtype


def import_onnx(data: bytes) -> GraphIr:
    model = parse(data)
    gm = parse(model[7][0])
    g = GraphIr(gm[2][0].decode() if 2 in gm else "onnx")
    ids: dict[str, int] = {}
    consts = {}
    for b in gm.get(5, []):
        name, t = _decode_tensor(b)
        consts[name] = t
    for b in gm.get(11, []):
        name, shape, dtype = _decode_value_info(b)
        if name not in consts:
            ids[name] = g.add_input(name, shape, dtype)
    rev = {v: k for k, v in _STD.items()}

    def val(name):
        if name not in ids:
            if name in consts:
                ids[name] = g.constant(name, consts[name])
            else:
                raise GraphError(f"value {name} used before definition")
        return ids[name]

    pending_sqrt = {}
    for b in gm.get(1, []):
        m = parse(b)
        ins = [x.decode() for x in m.get(1, [])]
        outs = [x.decode() for x in m.get(2, [])]
        op_type = m[4][0].decode()
        domain = m[7][0].decode() if 7 in m else ""
        attrs = dict(_decode_attr(x) for x in m.get(5, []))
        if domain == CUSTOM_DOMAIN:
            if op_type not in _CUSTOM:
                raise GraphError(f"unknown {CUSTOM_DOMAIN} op {op_type}")
            ids[outs[0]] = g.add_node(op_type, [val(i) for i in ins], attrs, name=outs[0])
            continue
        if op_type == "Sqrt":
            pending_sqrt[outs[0]] = ins[0]
            continue
        if op_type == "Reciprocal" and ins[0] in pending_sqrt:
            ids[outs[0]] = g.add_node("rsqrt", [val(pending_sqrt.pop(ins[0]))], name=outs[0])
            continue
        op = rev.get(op_type)
        if op is None:
            raise GraphError(f"unsupported ONNX op {op_type}")
        a = {}
        if op in ("softmax", "log_softmax", "concat"):
            a["dim"] = attrs.get("axis", -1)
        elif op == "layer_norm":
            a["eps"] = attrs.get("epsilon", 1e-5)
        elif op == "gelu":
            a["approximate"] = attrs.get("approximate", "none")
        elif op == "linear":
            if attrs.get("transB", 0) != 1 or attrs.get("transA", 0):
                raise GraphError("only Gemm with transB=1 is supported")
        elif op == "transpose":
            perm = attrs["perm"]
            moved = [i for i, p in enumerate(perm) if p != i]
            if len(moved) not in (0, 2):
                raise GraphError("only two-axis transposes are supported")
            a = {"dim0": moved[0], "dim1": moved[1]} if moved else {"dim0": 0, "dim1": 0}
        elif op == "reshape":
            a["shape"] = consts[ins[1]].tolist()
            ins = ins[:1]
        elif op in ("sum", "mean"):
            a["keepdim"] = bool(attrs.get("keepdims", 1))
            if len(ins) > 1:
                dims = consts[ins[1]].tolist()
                a["dim"] = dims[0] if len(dims) == 1 else dims
                ins = ins[:1]
        ids[outs[0]] = g.add_node(op, [val(i) for i in ins], a, name=outs[0])
    for b in gm.get(12, []):
        name, _, _ = _decode_value_info(b)
        g.mark_output(ids[name])
    return g


def check_model(data: bytes) -> list[str]:
    """Structural checks: a graph, an opset import, every node input defined before use."""
    errs = []
    model = parse(data)
    if 7 not in model:
        return ["no graph"]
    if 8 not in model:
        errs.append("no opset_import")
    gm = parse(model[7][0])
    defined = {_decode_tensor(b)[0] for b in gm.get(5, [])} | {_decode_value_info(b)[0] for b in gm.get(11, [])}
    for b in gm.get(1, []):
        m = parse(b)
        for i in m.get(1, []):
            if i.decode() and i.decode() not in defined:
                errs.append(f"node {m.get(3, [b'?'])[0].decode()} uses undefined {i.decode()}")
        defined.update(x.decode() for x in m.get(2, []))
    for b in gm.get(12, []):
        if _decode_value_info(b)[0] not in defined:
            errs.append("graph output never produced")
    return errs


# ------------------------------------------------------------------ the reference's ONNX entry points
# crates/brain-onnx/src: impl_.rs (load_onnx, import_and_optimize), ir2graph.rs / graph2onnx.rs (lowering to
# and from the graph IR), eval/mod.rs (evaluate_onnx_model), optimize/onnx_passes.rs (fold_constant_nodes,
# fuse_matmul_add), tools.rs (onnx_summary), model_zoo.rs (create_mlp_zoo_model), utils.rs (varints,
# little-endian reads, CRC-32), version.rs (default_opset, is_valid_opset).
DEFAULT_OPSET = 17


def default_opset() -> int:
    return DEFAULT_OPSET


def is_valid_opset(v: int) -> bool:
    return 1 <= int(v) <= 23


def encode_varint(v: int) -> bytes:
    return _varint(v)


def decode_varint(b: bytes, pos: int = 0) -> tuple[int, int]:
    """(value, position after it) of the protobuf varint starting at ``pos``."""
    out, shift = 0, 0
    while True:
        c = b[pos]
        pos += 1
        out |= (c & 0x7F) << shift
        shift += 7
        if not c & 0x80:
            return out, pos


def read_f32_le(b: bytes, offset: int = 0) -> float:
    return struct.unpack_from("<f", b, offset)[0]


def read_f64_le(b: bytes, offset: int = 0) -> float:
    return struct.unpack_from("<d", b, offset)[0]


def compute_crc32(b: bytes) -> int:
    import zlib
    return zlib.crc32(b) & 0xFFFFFFFF


def load_onnx(path: str) -> GraphIr:
    with open(path, "rb") as f:
        return import_onnx(f.read())


lower_to_graph_ir = import_onnx


def lower_from_graph_ir(g: GraphIr) -> bytes:
    return export_onnx(g)


def fold_constant_nodes(g: GraphIr) -> bool:
    from .graph import fold_constants
    return fold_constants(g)


def fuse_matmul_add(g: GraphIr) -> int:
    """matmul(x, W) followed by add(., b) with a constant 1-D b becomes linear(x, W^T, b). Returns the count."""
    from .graph import _rename
    cons = g.consumers()
    n_f = 0
    for n in list(g.nodes):
        if n.op != "matmul" or len(cons.get(n.outputs[0], [])) != 1:
            continue
        add = cons[n.outputs[0]][0]
        if add.op != "add" or n.outputs[0] in g.outputs:
            continue
        other = add.inputs[1] if add.inputs[0] == n.outputs[0] else add.inputs[0]
        w, b = g.values[n.inputs[1]].constant, g.values[other].constant
        if w is None or b is None or w.dim() != 2 or b.dim() != 1 or b.shape[0] != w.shape[1]:
            continue
        wt = g.constant(f"{g.values[n.inputs[1]].name}_t", w.t().contiguous())
        lin_out = g.add_node("linear", [n.inputs[0], wt, other])
        lin = g.nodes.pop()  # the node just appended goes where the add was
        g.nodes.insert(g.nodes.index(add), lin)
        g.nodes.remove(add)
        g.nodes.remove(n)
        _rename(g, add.outputs[0], lin_out)
        n_f += 1
    return n_f


def import_and_optimize(data: bytes, level: int = 2) -> GraphIr:
    from .graph import optimize
    g = import_onnx(data)
    fuse_matmul_add(g)
    optimize(g, level)
    return g


def evaluate_onnx_model(data: bytes, inputs) -> list:
    """Run an ONNX model through the graph interpreter (the framework's kernels for bf16 CUDA inputs)."""
    from .graph import GraphInterpreter
    return GraphInterpreter().run(import_onnx(data), list(inputs))


def onnx_summary(data: bytes) -> dict:
    g = import_onnx(data)
    ops: dict[str, int] = {}
    for n in g.nodes:
        ops[n.op] = ops.get(n.op, 0) + 1
    params = sum(v.constant.numel() for v in g.values.values() if v.constant is not None)
    return {"name": g.name, "nodes": len(g.nodes), "inputs": len(g.inputs), "outputs": len(g.outputs),
            "parameters": int(params), "ops": dict(sorted(ops.items())), "problems": check_model(data)}


def create_mlp_zoo_model(dims=(4, 8, 2), seed: int = 0) -> bytes:
    from .graph_tools import build_mlp_graph
    return export_onnx(build_mlp_graph(list(dims), seed=seed))
