"""``brain`` command line (``python -m brain_b200 <command>``).

Commands mirror the reference dispatcher (crates/brain-cli/src/impl.rs:8-62):
  make     train a small classifier from a CSV (``features..., label``) and write a ``.brain`` /
           ``.bn`` checkpoint with an ``arch`` descriptor (make_cmd.rs:21-250: mlp = linear,relu,linear;
           convnet = conv2d,relu,maxpool2d,flatten,linear; sgd|adam; cross_entropy|mse).
  run      rebuild the layers from ``arch`` and predict on a CSV (run_cmd.rs:9-140).
  check    scan a checkpoint for NaN / Inf and print a summary (check_cmd.rs:7-60).
  train    data-parallel LLM training on synthetic tokens (LlamaLite / GptLite presets), launched
           one process per GPU with torchrun.
  bench    the headline training benchmark (delegates to bench.py) or the collective sweep.
  convert  between BRAIN_STATE_V1 text, the BRAINCK2 binary container, .bn and safetensors.
  tensor   list the tensors of a checkpoint.
  model    parameter counts and shapes of the model presets.
  dataset  write a synthetic classification CSV.
  doctor   report the CUDA device, native libraries and versions.
  space / chat / new   create, teach and talk to a BrainMind ``.bn`` (space_cmd.rs:16-200).
  script   run a file of REPL statements; repl: interactive tensor REPL; init: scaffold a project.
Exit codes: 0 ok, 1 error, 2 invalid usage, 3 I/O error (the reference's ExitCode values).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import sys

OK, ERROR, USAGE, IO_ERROR = 0, 1, 2, 3


def _load_csv(path: str, labeled: bool = True):
    import torch
    feats, labels = [], []
    try:
        with open(path) as f:
            for ln, line in enumerate(f, 1):
                line = line.strip()
                if not line or line.startswith("#"):
                    continue
                vals = [v.strip() for v in line.replace(";", ",").split(",")]
                try:
                    nums = [float(v) for v in vals]
                except ValueError:
                    if ln == 1:
                        continue  # header
                    raise ValueError(f"{path}:{ln}: not numeric")
                if labeled:
                    feats.append(nums[:-1])
                    labels.append(nums[-1])
                else:
                    feats.append(nums)
    except OSError as e:
        raise OSError(str(e))
    x = torch.tensor(feats, dtype=torch.float32)
    y = torch.tensor(labels) if labeled else None
    return x, y


def _build_arch(arch: str, n_features: int, hidden: int, n_out: int):
    from .. import nn
    if arch == "convnet":
        side = round(math.sqrt(n_features))
        s = side if side * side == n_features and side >= 3 else 6
        flat = 4 * (s // 2) * (s // 2)
        model = nn.Sequential(ReshapeImage(s), nn.Conv2d(1, 4, 3, padding=1), nn.ReLU(), nn.MaxPool2d(2, 2),
                              nn.Flatten(), nn.Linear(flat, n_out))
        return model, "conv2d,relu,maxpool2d,flatten,linear"
    model = nn.Sequential(nn.Linear(n_features, hidden), nn.ReLU(), nn.Linear(hidden, n_out))
    return model, "linear,relu,linear"


class ReshapeImage:
    """Callable module: [B, s*s] -> [B, 1, s, s] (zero padded / truncated)."""

    def __new__(cls, side):
        import torch

        class _R(torch.nn.Module):
            def __init__(self):
                super().__init__()
                self.side = side

            def forward(self, x):
                n = self.side * self.side
                if x.shape[1] < n:
                    x = torch.nn.functional.pad(x, (0, n - x.shape[1]))
                return x[:, :n].reshape(-1, 1, self.side, self.side)
        return _R()


def cmd_make(a) -> int:
    import torch
    from ..optim import SGD, Adam
    from ..train import Batch, TrainerBuilder
    try:
        x, y = _load_csv(a.data, True)
    except (OSError, ValueError) as e:
        print(f"error: {e}")
        return IO_ERROR if isinstance(e, OSError) else ERROR
    task = "regression" if a.loss == "mse" else "classification"
    n_classes = a.classes or (int(y.max().item()) + 1 if task == "classification" else 1)
    torch.manual_seed(a.seed)
    model, arch = _build_arch(a.arch, x.shape[1], a.hidden, n_classes)
    loss = None
    if task == "regression":
        def loss(out, t):
            return torch.nn.functional.mse_loss(out.squeeze(-1), t.float())
    else:
        y = y.long()
    opt = (Adam if a.optim == "adam" else SGD)(model.parameters(), lr=a.lr)
    tr = TrainerBuilder().model(model).optimizer(opt).loss(loss).build() if loss else \
        TrainerBuilder().model(model).optimizer(opt).build()
    batches = [Batch(x[i:i + a.batch], y[i:i + a.batch]) for i in range(0, len(x), a.batch)]
    print(f"make: arch={a.arch} dataset={a.data} samples={len(x)} features={x.shape[1]} classes={n_classes} "
          f"hidden={a.hidden} optim={a.optim} loss={a.loss} lr={a.lr} epochs={a.epochs} batch={a.batch}")
    s = tr.fit(batches, a.epochs)
    print(f"trained {s.steps} steps: loss {s.history[0].loss:.4f} -> {s.history[-1].loss:.4f}")
    st = tr.state({"arch": arch, "task": task, "features": str(x.shape[1]), "classes": str(n_classes)})
    if a.output.endswith(".bn"):
        from ..checkpoint import BrainModelFile
        bn = BrainModelFile(os.path.basename(a.output))
        for k, v in st.metadata.items():
            bn.with_meta(k, str(v))
        for nt in st.tensors:
            bn.add_tensor(nt.name, nt.tensor.double())
        bn.save_file(a.output)
    else:
        st.save_file(a.output)
    print(f"wrote {a.output}")
    return OK


def _load_state(path):
    from ..checkpoint import BrainModelFile, ModelState, load_brain_v2
    from ..checkpoint.formats import NamedTensor
    with open(path, "rb") as f:
        head = f.read(16)
    if head.startswith(b"BRAIN_BN"):
        bn = BrainModelFile.load_file(path)
        return ModelState([NamedTensor(k, v) for k, v in sorted(bn.archive.items())], dict(bn.metadata))
    if head.startswith(b"BRAINCK2"):
        ts, meta = load_brain_v2(path)
        return ModelState([NamedTensor(k, v) for k, v in ts.items()], {k: str(v) for k, v in meta.items()})
    return ModelState.load_file(path)


def cmd_run(a) -> int:
    import torch
    try:
        st = _load_state(a.model)
    except OSError as e:
        print(f"error: could not read '{a.model}': {e}")
        return IO_ERROR
    except ValueError as e:
        print(f"error: invalid model '{a.model}': {e}")
        return ERROR
    arch = st.metadata.get("arch", "linear")

    def order(nt):  # module index, then weight before bias (archives store names sorted)
        head, _, leaf = nt.name.rpartition(".")
        idx = int(head.split(".")[-1]) if head.split(".")[-1].isdigit() else 0
        return idx, 0 if leaf == "weight" else 1
    params = [nt.tensor for nt in sorted(st.tensors, key=order)]
    layers, pi = [], 0
    for name in arch.split(","):
        name = name.strip()
        if name == "linear":
            w, b = params[pi].float(), params[pi + 1].float()
            pi += 2
            layers.append(lambda x, w=w, b=b: x @ w.t() + b)
        elif name == "relu":
            layers.append(torch.relu)
        elif name == "conv2d":
            w, b = params[pi].float(), params[pi + 1].float()
            pi += 2
            side = round(math.sqrt(int(st.metadata.get("features", "36"))))
            side = side if side >= 3 else 6

            def conv(x, w=w, b=b, s=side):
                n = s * s
                if x.dim() == 2:
                    x = torch.nn.functional.pad(x, (0, max(0, n - x.shape[1])))[:, :n].reshape(-1, 1, s, s)
                return torch.nn.functional.conv2d(x, w, b, padding=1)
            layers.append(conv)
        elif name == "maxpool2d":
            layers.append(lambda x: torch.nn.functional.max_pool2d(x, 2, 2))
        elif name == "flatten":
            layers.append(lambda x: x.flatten(1))
        else:
            print(f"error: unknown layer '{name}' in arch")
            return ERROR
    try:
        x, _ = _load_csv(a.data, labeled=a.labeled)
    except (OSError, ValueError) as e:
        print(f"error: {e}")
        return IO_ERROR
    out = x
    for f in layers:
        out = f(out)
    if st.metadata.get("task", "classification") == "classification":
        for row in out.argmax(-1).tolist():
            print(row)
    else:
        for v in out.squeeze(-1).tolist():
            print(f"{v:.6f}")
    return OK


def cmd_check(a) -> int:
    import torch
    try:
        st = _load_state(a.model)
    except OSError as e:
        print(f"error: {e}")
        return IO_ERROR
    except ValueError as e:
        print(f"error: invalid model: {e}")
        return ERROR
    bad = 0
    total = 0
    for nt in st.tensors:
        t = nt.tensor.float()
        n_bad = int((~torch.isfinite(t)).sum())
        total += t.numel()
        bad += n_bad
        if n_bad:
            print(f"  {nt.name}: {n_bad} non-finite values")
    print(f"check: {len(st.tensors)} tensors, {total} values, {bad} non-finite; metadata {dict(st.metadata)}")
    return OK if bad == 0 else ERROR


def cmd_tensor(a) -> int:
    st = _load_state(a.model)
    for nt in st.tensors:
        t = nt.tensor
        print(f"{nt.name}\t{tuple(t.shape)}\t{t.dtype}\tmean={t.float().mean():.6g}\tstd={t.float().std() if t.numel() > 1 else 0:.6g}")
    return OK


def cmd_convert(a) -> int:
    from ..checkpoint import save_brain_v2
    st = _load_state(a.input)
    out = a.output
    if out.endswith(".safetensors"):
        from ..utils.safetensors import save_safetensors
        save_safetensors(out, {nt.name: nt.tensor for nt in st.tensors}, st.metadata)
    elif out.endswith(".bn"):
        from ..checkpoint import BrainModelFile
        bn = BrainModelFile(os.path.basename(out))
        for k, v in st.metadata.items():
            bn.with_meta(k, str(v))
        for nt in st.tensors:
            bn.add_tensor(nt.name, nt.tensor.double())
        bn.save_file(out)
    elif a.binary:
        save_brain_v2(out, {nt.name: nt.tensor for nt in st.tensors}, dict(st.metadata))
    else:
        st.save_file(out)
    print(f"converted {a.input} -> {out} ({len(st.tensors)} tensors)")
    return OK


def cmd_model(a) -> int:
    from ..models import GptLiteConfig, LlamaLiteConfig
    presets = {"llama3-8b": LlamaLiteConfig.llama3_8b(), "llama3-70b": LlamaLiteConfig.llama3_70b(),
               "llama-tiny": LlamaLiteConfig.tiny(), "gpt-lite": GptLiteConfig.lite_2x128()}
    names = [a.name] if a.name else list(presets)
    for n in names:
        c = presets[n]
        np_ = c.num_params() if hasattr(c, "num_params") else None
        print(json.dumps({"preset": n, "params": np_, **{k: v for k, v in vars(c).items()}}))
    return OK


def cmd_dataset(a) -> int:
    from ..train import SyntheticClassification
    d = SyntheticClassification.two_class_points(a.samples, a.seed)
    with open(a.output, "w") as f:
        for x, y in zip(d.inputs.tolist(), d.targets.tolist()):
            f.write(",".join(f"{v:.6f}" for v in x) + f",{int(y)}\n")
    print(f"wrote {a.samples} samples to {a.output}")
    return OK


def cmd_doctor(a) -> int:
    import torch
    from .. import _native
    print(f"torch {torch.__version__}, cuda available: {torch.cuda.is_available()}")
    if torch.cuda.is_available():
        p = torch.cuda.get_device_properties(0)
        print(f"device 0: {p.name}, sm_{p.major}{p.minor}, {p.multi_processor_count} SMs, {p.total_memory / 2**30:.1f} GiB")
    for lib in ("brain_kernels", "brain_comm", "brain_runtime"):
        print(f"{lib}: {'ok' if _native.available(lib) else 'missing (python -m brain_b200._build)'}")
    return OK


def cmd_train(a) -> int:
    import time

    import torch
    from ..models import GptLite, GptLiteConfig, LlamaLite, LlamaLiteConfig
    from ..parallel import DataParallel, dist as bdist
    ctx = bdist.init()
    if a.model == "gpt-lite":
        cfg = GptLiteConfig.lite_2x128()
        model = GptLite(cfg, device=ctx.device, dtype=torch.float32 if ctx.device.type == "cpu" else torch.bfloat16)
    else:
        cfg = {"llama3-8b": LlamaLiteConfig.llama3_8b(a.seq), "llama-tiny": LlamaLiteConfig.tiny()}[a.model]
        model = LlamaLite(cfg, device=ctx.device, dtype=torch.float32 if ctx.device.type == "cpu" else torch.bfloat16)
    dp = DataParallel(model, lr=a.lr, grad_dtype=torch.float32)
    g = torch.Generator(device=ctx.device).manual_seed(1 + ctx.rank)
    seq = min(a.seq, cfg.max_seq_len)
    for step in range(a.steps):
        t0 = time.time()
        tok = torch.randint(0, cfg.vocab_size, (a.batch, seq + 1), generator=g, device=ctx.device)
        loss = float(dp.train_step(tok[:, :-1], tok[:, 1:]))
        if ctx.is_master:
            print(f"{bdist.rank_prefix()} step {step} loss {loss:.4f} ({time.time() - t0:.3f}s)")
    if a.save and ctx.is_master:
        from ..checkpoint import save_brain_v2
        save_brain_v2(a.save, {n: p.detach() for n, p in model.named_parameters()}, {"steps": a.steps})
        print(f"saved {a.save}")
    bdist.shutdown()
    return OK


def cmd_bench(a) -> int:
    here = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    if a.collectives:
        from ..bench.collective_sweep import main as sweep
        return sweep([])
    import subprocess
    return subprocess.call([sys.executable, os.path.join(here, "bench.py")] + a.rest)


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(prog="brain", description="brain_b200 command line")
    sub = p.add_subparsers(dest="cmd")
    m = sub.add_parser("make")
    m.add_argument("output")
    m.add_argument("--data", required=True)
    m.add_argument("--arch", default="mlp", choices=["mlp", "convnet"])
    m.add_argument("--hidden", type=int, default=16)
    m.add_argument("--classes", type=int, default=0)
    m.add_argument("--optim", default="sgd", choices=["sgd", "adam"])
    m.add_argument("--loss", default="cross_entropy", choices=["cross_entropy", "mse"])
    m.add_argument("--lr", type=float, default=0.1)
    m.add_argument("--epochs", type=int, default=20)
    m.add_argument("--batch", type=int, default=8)
    m.add_argument("--seed", type=int, default=0)
    r = sub.add_parser("run")
    r.add_argument("model")
    r.add_argument("data")
    r.add_argument("--labeled", action="store_true", help="the CSV has a trailing label column to ignore")
    c = sub.add_parser("check")
    c.add_argument("model")
    t = sub.add_parser("tensor")
    t.add_argument("model")
    cv = sub.add_parser("convert")
    cv.add_argument("input")
    cv.add_argument("output")
    cv.add_argument("--binary", action="store_true", help="write the BRAINCK2 native-dtype container")
    mo = sub.add_parser("model")
    mo.add_argument("name", nargs="?")
    d = sub.add_parser("dataset")
    d.add_argument("output")
    d.add_argument("--samples", type=int, default=64)
    d.add_argument("--seed", type=int, default=0)
    sub.add_parser("doctor")
    tr = sub.add_parser("train")
    tr.add_argument("--model", default="llama-tiny", choices=["llama-tiny", "llama3-8b", "gpt-lite"])
    tr.add_argument("--steps", type=int, default=10)
    tr.add_argument("--batch", type=int, default=8)
    tr.add_argument("--seq", type=int, default=64)
    tr.add_argument("--lr", type=float, default=3e-4)
    tr.add_argument("--save", default="")
    sp = sub.add_parser("space")
    sp.add_argument("rest", nargs=argparse.REMAINDER)
    ch = sub.add_parser("chat", aliases=["chatbot"])
    ch.add_argument("rest", nargs=argparse.REMAINDER)
    nw = sub.add_parser("new")
    nw.add_argument("rest", nargs=argparse.REMAINDER)
    sc = sub.add_parser("script")
    sc.add_argument("file")
    sub.add_parser("repl")
    ini = sub.add_parser("init")
    ini.add_argument("name", nargs="?", default="brain_project")
    sub.add_parser("version")
    b = sub.add_parser("bench")
    b.add_argument("--collectives", action="store_true")
    b.add_argument("rest", nargs=argparse.REMAINDER)
    return p


def cmd_space(a) -> int:
    from .repl import space_command
    return space_command(a.rest)


def cmd_chat(a) -> int:
    from .repl import space_command
    return space_command(["chat"] + a.rest)


def cmd_new(a) -> int:
    from .repl import space_command
    return space_command(["new"] + a.rest)


def cmd_script(a) -> int:
    from .repl import run_script
    try:
        with open(a.file) as f:
            text = f.read()
    except OSError as e:
        print(f"error: could not read '{a.file}': {e}")
        return IO_ERROR
    return run_script(text)


def cmd_repl(a) -> int:
    from .repl import run_repl
    return run_repl()


def cmd_init(a) -> int:
    from .repl import scaffold_project
    return scaffold_project(a.name)


def cmd_version(a) -> int:
    import brain_b200
    print(f"brain_b200 v{getattr(brain_b200, '__version__', '0.1.0')}")
    return OK


COMMANDS = {"make": cmd_make, "run": cmd_run, "check": cmd_check, "tensor": cmd_tensor, "convert": cmd_convert,
            "model": cmd_model, "dataset": cmd_dataset, "doctor": cmd_doctor, "train": cmd_train, "bench": cmd_bench,
            "space": cmd_space, "chat": cmd_chat, "chatbot": cmd_chat, "new": cmd_new, "script": cmd_script,
            "repl": cmd_repl, "init": cmd_init, "version": cmd_version}


def main(argv=None) -> int:
    p = build_parser()
    try:
        a = p.parse_args(argv)
    except SystemExit as e:
        return USAGE if e.code else OK
    if not a.cmd:
        p.print_help()
        return USAGE
    return COMMANDS[a.cmd](a)


if __name__ == "__main__":
    sys.exit(main())
