"""The ctypes signature table must match every exported C prototype in csrc/ (parsed from source)."""
import os
import re

import brain_b200.ops  # noqa: F401  (registers op signatures)
import brain_b200.parallel.symm  # noqa: F401
import brain_b200.parallel.tensor_parallel  # noqa: F401
import brain_b200.models.llama_tp  # noqa: F401
import brain_b200.parallel.overlap  # noqa: F401
import brain_b200.checkpoint  # noqa: F401
import brain_b200.data  # noqa: F401
import brain_b200.oracle  # noqa: F401
from brain_b200 import _native

CSRC = os.path.join(os.path.dirname(_native.__file__), "csrc")


def _code(param: str) -> str:
    param = param.strip()
    if "cudaStream_t" in param:
        return "s"
    if "*" in param:
        return "p"
    toks = param.replace("const", "").split()
    ty = " ".join(toks[:-1])
    return {"int64_t": "l", "int": "i", "float": "f", "double": "d", "uint64_t": "l", "uint32_t": "i"}[ty]


def _prototypes():
    protos = {}
    for fn in os.listdir(CSRC):
        if not fn.endswith((".cu", ".cpp")):
            continue
        src = open(os.path.join(CSRC, fn)).read()
        for m in re.finditer(r"BRAIN_API\s+[\w\s\*]+?\s(\w+)\(([^)]*)\)\s*\{", src):
            name, params = m.group(1), m.group(2)
            params = [p for p in params.replace("\n", " ").split(",") if p.strip() and p.strip() != "void"]
            protos[name] = "".join(_code(p) for p in params)
    return protos


def test_signatures_match_sources():
    protos = _prototypes()
    missing, wrong = [], []
    for name, (_, codes) in _native.SIGNATURES.items():
        if name.startswith("brain_status_"):
            continue
        if name not in protos:
            missing.append(name)
        elif protos[name] != codes:
            wrong.append((name, codes, protos[name]))
    assert not missing, f"bound but not exported: {missing}"
    assert not wrong, "signature mismatch (name, bound, source): " + repr(wrong)
