"""Build a linear layer as a graph, export it to ONNX, check and re-import it, and evaluate both
(the reference's examples/onnx_export.rs). Run from the repository root with it on ``PYTHONPATH``."""
import torch

from brain_b200 import graph as G
from brain_b200 import onnx as O


def main(path: str = "linear_layer.onnx"):
    g = G.GraphIr("linear_layer")
    x = g.add_input("X", (1, 2))
    w = g.constant("W", torch.tensor([[0.5, -1.0], [2.0, 0.25]]))
    b = g.constant("B", torch.tensor([0.1, -0.2]))
    g.mark_output(g.add_node("relu", [g.add_node("linear", [x, w, b], name="Y0")], name="Y"))
    G.infer_shapes(g)
    data = O.export_onnx(g, path)
    print("checker:", O.check_model(data) or "ok", f"({len(data)} bytes)")
    back = O.import_onnx(data)
    xin = torch.tensor([[1.0, 2.0]])
    y0, y1 = G.GraphInterpreter().run(g, [xin])[0], G.GraphInterpreter().run(back, [xin])[0]
    print("graph:", y0.tolist(), " re-imported:", y1.tolist())
    return y0, y1


if __name__ == "__main__":
    main()
