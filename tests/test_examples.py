"""The example programs run and do what they say (CPU)."""
import os
import runpy
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(name):
    return runpy.run_path(os.path.join(ROOT, "examples", name))["main"]


def test_convnet_example_learns():
    before, after, final = _run("convnet_train.py")()
    assert after.loss < before[0] and final[1] == 1.0


def test_quantize_example():
    y, yq, m = _run("quantize_linear.py")()
    assert float((y - yq).abs().max()) < 0.02 and m.sparsity() == 0.5


def test_onnx_example(tmp_path):
    y0, y1 = _run("onnx_export.py")(str(tmp_path / "m.onnx"))
    assert y0.tolist() == y1.tolist()


def test_hello_script():
    import importlib
    cli = importlib.import_module("brain_b200.cli.main")
    assert cli.main(["script", os.path.join(ROOT, "examples", "hello.brain")]) == 0


def test_tiny_llama_example_cpu(monkeypatch):
    monkeypatch.setenv("CUDA_VISIBLE_DEVICES", "")
    losses = _run("train_llama_tiny.py")(steps=4)
    assert losses[-1] < losses[0]
