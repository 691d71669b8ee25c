"""Int8 weight quantisation and magnitude pruning of a linear layer (the reference's
examples/quantize_linear.rs): compare the float output with the dequantised-weight output, then
prune half of the weights. Run from the repository root with it on ``PYTHONPATH``."""
import torch

from brain_b200.nn.pruning import PruningMask
from brain_b200.quantization import QuantDType, dequantize_tensor, quantize_tensor


def main():
    w = torch.tensor([[0.12, -0.45, 0.78, -0.23], [0.91, -0.05, 0.33, -0.88]])
    x = torch.tensor([[1.0, 0.5, -0.5, 2.0]])
    q, scale, zp = quantize_tensor(w, QuantDType.INT8)
    wq = dequantize_tensor(q, scale, zp, w.shape)
    y, yq = x @ w.t(), x @ wq.t()
    print("fp32 output     ", y.tolist())
    print("int8-weight out ", yq.tolist(), " max abs error", float((y - yq).abs().max()))
    m = PruningMask.from_magnitude(w, 0.5)
    print("pruned weight   ", m.apply(w).tolist(), " sparsity", m.sparsity())
    return y, yq, m


if __name__ == "__main__":
    main()
