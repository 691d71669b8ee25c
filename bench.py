#!/usr/bin/env python
"""Headline benchmark: Llama-3-8B-shaped bf16 pretraining throughput (train tok/s), data parallel
with sharded AdamW, one process per B200.

Model: 32 layers, d 4096, 32 q / 8 kv heads (GQA), SwiGLU FFN 14336, RMSNorm, RoPE theta 500000,
vocab 128256, random-init N(0, 0.02) (seed 0). Data: synthetic tokens uniform in [0, vocab)
(seeded), seq 4096, micro-batch 2 per GPU (weak scaling: global batch = 2 * N).

Usage: ``python bench.py --gpus N --steps K --warmup W``; for N > 1 launch with
``torch.distributed.run --nproc-per-node N``. Rank 0 prints one JSON line.

Timing: W untimed warm-up steps; K steps bracketed by barrier + synchronize, CUDA events on the
compute stream, max over ranks. The working set (weights, optimizer state, activations) is
hundreds of GB, far above the 126 MB L2, so no explicit L2 flush is needed. SM clocks and throttle
reasons are sampled with nvidia-smi during the timed region. A second loop measures the same
metric end to end through the public API (``DataParallel.train_step``): every step copies its
tokens from pinned host memory and reads the loss back to the host.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

REF_UNAVAILABLE = ("the reference (uxle/brain) is a pure-Rust Cargo workspace: its root has no setup.py/pyproject "
                   "and its pyo3 crate needs maturin + cargo, neither of which exists in this image, so "
                   "`pip install --target baseline/_ref` fails; it also has no GPU code path or Llama training")


def log(*a):
    print(*a, file=sys.stderr, flush=True)


class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception as e:  # nvidia-smi missing: report no clocks
            log("clock sampler unavailable:", e)
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=8)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="brain", choices=["brain", "reference", "torch"],
                    help="brain: this framework; reference: the reference's own code; torch: a plain PyTorch "
                         "eager + cuBLAS + SDPA + NCCL DDP implementation of the same model and config")
    ap.add_argument("--seq", type=int, default=4096)
    ap.add_argument("--micro-batch", type=int, default=2)
    ap.add_argument("--layers", type=int, default=32, help="development only: fewer layers is not the benchmark")
    ap.add_argument("--comm", default="nvlink", choices=["nccl", "nvlink"],
                    help="gradient reduction: fused NVLink kernels (default) or NCCL")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-overlap", action="store_true",
                    help="reduce gradients after backward instead of per bucket during backward")
    ap.add_argument("--overlap", action="store_true",
                    help="reduce per bucket during backward also below 4 GPUs (where little is exposed)")
    ap.add_argument("--overlap-mode", default="ce", choices=["ce", "sm"],
                    help="overlapped reduction: copy engines move the data (ce) or SM kernels do (sm)")
    ap.add_argument("--workload", default="train", choices=["train", "decode", "vit", "gptlite-cpu"],
                    help="train: Llama-3-8B DDP (headline); decode: Llama-3-70B-shape TP=N greedy decode; "
                         "vit: ViT-B/16 DDP images/s; gptlite-cpu: the GPT-lite data-parallel config on CPU ranks")
    ap.add_argument("--decode", default="auto", choices=["auto", "on", "off"],
                    help="also measure the 70B TP decode inside the train run (auto: when N == 8)")
    ap.add_argument("--decode-batch", type=int, default=32)
    ap.add_argument("--prompt-len", type=int, default=2048)
    ap.add_argument("--new-tokens", type=int, default=256)
    ap.add_argument("--decode-layers", type=int, default=80, help="development only")
    ap.add_argument("--l2-prefetch", action="store_true",
                    help="decode step: prefetch the small GEMMs' weights into L2 ahead of them")
    ap.add_argument("--decode-pdl", type=int, default=2,
                    help="programmatic dependent launch in the decode step: 0 off, 1 successors launch at a "
                         "kernel's start, 2 after its main loop")
    ap.add_argument("--torch-master", default="bf16", choices=["bf16", "fp32"],
                    help="--impl torch optimizer: fused AdamW on the bf16 parameters, or float32 master weights "
                         "and moments sharded ZeRO-1 style (the framework's precision)")
    ap.add_argument("--torch-graph", default="on", choices=["on", "off"],
                    help="--impl torch --workload decode: replay the decode step from a CUDA graph, or run it eagerly")
    ap.add_argument("--decode-shard-of", type=int, default=0,
                    help="development only: run one rank's shard of an N-way TP group on a single GPU")
    args = ap.parse_args()

    if args.impl == "reference":
        print(json.dumps({"impl": "reference", "unavailable": REF_UNAVAILABLE}), flush=True)
        return 0

    if args.impl == "torch":
        if args.workload == "decode":
            return run_torch_decode(args)
        return run_torch_vit(args) if args.workload == "vit" else run_torch_baseline(args)

    import torch
    import torch.distributed as dist

    from brain_b200 import _native
    from brain_b200.models import LlamaLite, LlamaLiteConfig
    from brain_b200.parallel import DataParallel, dist as bdist

    if args.workload == "gptlite-cpu":
        return run_gptlite_cpu(args)
    ctx = bdist.init(timeout_s=300)
    rank, world = ctx.rank, ctx.world_size
    if world != args.gpus:
        log(f"warning: --gpus {args.gpus} but WORLD_SIZE {world}")
    dev = ctx.device
    if args.workload == "vit":
        return run_vit(args, ctx)
    decode = None
    if args.workload == "decode" or args.decode == "on" or (args.decode == "auto" and world == 8):
        try:
            decode = run_decode(args, rank, world, dev)
        except Exception as e:  # the train measurement below still runs
            log(f"{bdist.rank_prefix()} decode measurement failed: {type(e).__name__}: {e}")
            decode = {"error": f"{type(e).__name__}: {e}"}
        torch.cuda.empty_cache()
        if args.workload == "decode":
            if rank == 0:
                print(json.dumps(decode), flush=True)
            bdist.shutdown()
            return 0
    cfg = LlamaLiteConfig.llama3_8b(max_seq_len=args.seq)
    if args.layers != cfg.num_layers:
        cfg = cfg.replace(num_layers=args.layers)
    torch.manual_seed(0)
    t0 = time.time()
    model = LlamaLite(cfg, device=dev, dtype=torch.bfloat16, seed=0)
    dp = DataParallel(model, lr=3e-4, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1, grad_dtype=torch.bfloat16,
                      comm=args.comm, overlap=(world >= 4 or args.overlap) and not args.no_overlap,
                      overlap_mode=args.overlap_mode)
    log(f"{bdist.rank_prefix()} model {cfg.num_params() / 1e9:.2f}B params ready in {time.time() - t0:.1f}s; "
        f"mem {torch.cuda.memory_allocated() / 2**30:.1f} GiB")

    B, S, V = args.micro_batch, args.seq, cfg.vocab_size
    gen = torch.Generator(device=dev).manual_seed(1 + rank)
    n_pool = 4
    pool = [torch.randint(0, V, (B, S + 1), generator=gen, device=dev) for _ in range(n_pool)]

    def step_dev(i):
        t = pool[i % n_pool]
        return dp.train_step(t[:, :-1], t[:, 1:])

    # ---------------------------------------------------------------- warm-up
    for i in range(args.warmup):
        loss = step_dev(i)
        if rank == 0 and i == 0:
            log(f"first loss {loss.item():.4f}")
    torch.cuda.synchronize()
    log(f"{bdist.rank_prefix()} warm-up done, peak mem {torch.cuda.max_memory_allocated() / 2**30:.1f} GiB")

    # ---------------------------------------------------------------- device-timed loop
    clocks = ClockSampler(torch.cuda.current_device()) if rank == 0 else None
    if clocks:
        clocks.start()
    time.sleep(0.3)  # every rank: let the sampler start, then align all ranks before timing
    bdist.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    trace = []  # device scalars: reading them after the loop adds no synchronisation to it
    with _native.launch_counter() as lc:
        start.record()
        for i in range(args.steps):
            loss = step_dev(args.warmup + i)
            trace.append(loss)
        end.record()
    torch.cuda.synchronize()
    if rank == 0:
        log("losses (timed loop): " + " ".join(f"{float(x):.4f}" for x in trace))
    bdist.barrier()
    clk = clocks.stop() if clocks else None
    ms = start.elapsed_time(end) / args.steps
    t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    final_loss = float(loss.item())

    # ---------------------------------------------------------------- end-to-end loop (public API)
    e2e = None
    if not args.no_e2e:
        host = [torch.randint(0, V, (B, S + 1), generator=torch.Generator().manual_seed(100 + rank * 1000 + i))
                .pin_memory() for i in range(n_pool)]
        dev_buf = torch.empty(B, S + 1, dtype=torch.int64, device=dev)
        bdist.barrier()
        torch.cuda.synchronize()
        s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s2.record()
        for i in range(args.steps):
            dev_buf.copy_(host[i % n_pool], non_blocking=True)
            lv = dp.train_step(dev_buf[:, :-1], dev_buf[:, 1:]).item()
        e2.record()
        torch.cuda.synchronize()
        bdist.barrier()
        ms2 = s2.elapsed_time(e2) / args.steps
        t2 = torch.tensor([ms2], device=dev)
        if world > 1:
            dist.all_reduce(t2, op=dist.ReduceOp.MAX)
        ms2 = float(t2.item())
        e2e = {"value": B * S * world / (ms2 / 1e3), "unit": "tokens/s", "ms_per_step": ms2,
               "h2d_bytes_per_step": B * (S + 1) * 8, "d2h_bytes_per_step": 4,
               "api": "brain_b200.parallel.DataParallel.train_step", "last_loss": lv}

    tok_s = B * S * world / (ms / 1e3)
    flops_tok = 6 * (cfg.num_params() - cfg.vocab_size * cfg.hidden_dim) + \
        6 * cfg.num_layers * S * cfg.num_heads * cfg.head_dim  # dense + causal attention (fwd+bwd)
    if rank == 0:
        out = {
            "metric": "train tok/s Llama-3-8B-shape DDP @1/2/4/8 B200; 70B-shape TP=8 decode tok/s",
            "value": tok_s, "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic (uniform random tokens, seeded; random-init N(0,0.02) weights)",
            "config": {"model": "Llama-3-8B-shape" + ("" if cfg.num_layers == 32 else f" ({cfg.num_layers} layers: NOT the benchmark)"),
                       "params": cfg.num_params(), "global_batch": B * world, "micro_batch_per_gpu": B,
                       "seq_len": S, "parallelism": f"dp{world}", "optimizer": "sharded AdamW (ZeRO-1), fused kernel",
                       "grad_dtype": "bf16", "comm": args.comm,
                       "grad_reduction": (f"per bucket during backward ({args.overlap_mode})" if dp.overlapped is not None
                                          else "after backward"),
                       "l2": "no flush: working set (weights+optimizer+activations) >> 126 MB L2"},
            "mfu_model_tflops_per_gpu": flops_tok * tok_s / world / 1e12,
            "nvlink": _ddp_link_roofline(cfg.num_params(), world, ms),
            "final_loss": final_loss,
            "clocks": clk,
            "e2e": e2e,
            "gpu_launches": lc.count,
            "impl": "brain",
        }
        if decode is not None:
            out["decode_70b"] = decode
        print(json.dumps(out), flush=True)
    del dp, model
    bdist.shutdown()
    return 0


def run_torch_baseline(args) -> int:
    """The headline training config on plain PyTorch (``brain_b200.bench.torch_baseline``): eager
    modules, cuBLAS, SDPA, fused torch AdamW, DistributedDataParallel over NCCL; same timing rules."""
    import datetime

    import torch
    import torch.distributed as dist

    from brain_b200.bench.torch_baseline import build
    from brain_b200.models.config import LlamaLiteConfig

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    cfg = LlamaLiteConfig.llama3_8b(max_seq_len=args.seq)
    if args.layers != cfg.num_layers:
        cfg = cfg.replace(num_layers=args.layers)
    model = build(cfg, dev, seed=0)
    ddp = (torch.nn.parallel.DistributedDataParallel(model, device_ids=[local], gradient_as_bucket_view=True)
           if world > 1 else model)
    if args.torch_master == "fp32":
        from brain_b200.bench.torch_baseline import MasterAdamW
        opt = MasterAdamW(model.parameters(), lr=3e-4, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1, world=world,
                          rank=rank)
    else:
        opt = torch.optim.AdamW(model.parameters(), lr=3e-4, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1,
                                fused=True)
    B, S, V = args.micro_batch, args.seq, cfg.vocab_size
    cos, sin = model.rope_tables(S, dev)
    gen = torch.Generator(device=dev).manual_seed(1 + rank)
    pool = [torch.randint(0, V, (B, S + 1), generator=gen, device=dev) for _ in range(4)]

    def step(t):
        loss = ddp(t[:, :-1], t[:, 1:], cos, sin)
        loss.backward()
        opt.step()
        opt.zero_grad(set_to_none=False)
        return loss

    def barrier():
        if world > 1:
            dist.barrier()

    def max_ms(v):
        t = torch.tensor([v], device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    warm = max(3, args.warmup)
    for i in range(warm):
        loss = step(pool[i % 4])
    torch.cuda.synchronize()
    log(f"[torch rank {rank}] warm-up done, loss {loss.item():.4f}, peak mem "
        f"{torch.cuda.max_memory_allocated() / 2**30:.1f} GiB")
    clocks = ClockSampler(torch.cuda.current_device()) if rank == 0 else None
    if clocks:
        clocks.start()
    time.sleep(0.3)
    barrier()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    trace = []
    s.record()
    for i in range(args.steps):
        loss = step(pool[(warm + i) % 4])
        trace.append(loss.detach())
    e.record()
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop() if clocks else None
    if rank == 0:
        log("losses (timed loop): " + " ".join(f"{float(x):.4f}" for x in trace))
    ms = max_ms(s.elapsed_time(e) / args.steps)
    host = [torch.randint(0, V, (B, S + 1), generator=torch.Generator().manual_seed(100 + rank * 1000 + i)).pin_memory()
            for i in range(4)]
    buf = torch.empty(B, S + 1, dtype=torch.int64, device=dev)
    barrier()
    torch.cuda.synchronize()
    s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s2.record()
    for i in range(args.steps):
        buf.copy_(host[i % 4], non_blocking=True)
        lv = step(buf).item()
    e2.record()
    torch.cuda.synchronize()
    barrier()
    ms2 = max_ms(s2.elapsed_time(e2) / args.steps)
    if rank == 0:
        print(json.dumps({
            "metric": "train tok/s Llama-3-8B-shape DDP @1/2/4/8 B200; 70B-shape TP=8 decode tok/s",
            "value": B * S * world / (ms / 1e3), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": max(3, args.warmup), "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (uniform random tokens, seeded; random-init N(0,0.02) weights)",
            "config": {"model": "Llama-3-8B-shape" + ("" if cfg.num_layers == 32 else f" ({cfg.num_layers} layers)"),
                       "global_batch": B * world, "micro_batch_per_gpu": B, "seq_len": S,
                       "parallelism": f"dp{world}",
                       "implementation": "plain PyTorch: eager nn modules, cuBLAS, F.scaled_dot_product_attention, "
                                         + ("float32 master weights and moments (ZeRO-1 sharded), fused torch AdamW"
                                            if args.torch_master == "fp32" else
                                            "torch.optim.AdamW(fused=True) on bf16 parameters")
                                         + ", DDP over NCCL; same initial weights as the framework's model",
                       "l2": "no flush: working set >> 126 MB L2"},
            "final_loss": float(loss.item()), "clocks": clk,
            "e2e": {"value": B * S * world / (ms2 / 1e3), "unit": "tokens/s", "ms_per_step": ms2,
                    "h2d_bytes_per_step": B * (S + 1) * 8, "d2h_bytes_per_step": 4,
                    "api": "torch module forward/backward + optimizer.step", "last_loss": lv},
            "impl": "torch"}), flush=True)
    del ddp, model, opt
    if world > 1:
        dist.destroy_process_group()
    return 0


def run_torch_vit(args) -> int:
    """The ViT-B/16 config on plain PyTorch (``brain_b200.bench.torch_baseline.TorchViT``): eager modules,
    cuBLAS, SDPA, fused torch AdamW, DistributedDataParallel over NCCL; same data, batch and timing."""
    import datetime

    import torch
    import torch.distributed as dist

    from brain_b200.bench.torch_baseline import TorchViT
    from brain_b200.models.config import ViTConfig

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    cfg = ViTConfig.vit_b16()
    B = 256
    model = TorchViT(cfg, dev)
    ddp = (torch.nn.parallel.DistributedDataParallel(model, device_ids=[local], gradient_as_bucket_view=True)
           if world > 1 else model)
    opt = torch.optim.AdamW(model.parameters(), lr=1e-4, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.05, fused=True)
    gen = torch.Generator(device=dev).manual_seed(10 + rank)
    pool = [(torch.randn(B, 3, cfg.image_size, cfg.image_size, device=dev, generator=gen).bfloat16(),
             torch.randint(0, cfg.num_classes, (B,), device=dev, generator=gen)) for _ in range(2)]

    def step(x, y):
        loss = ddp(x, y)
        loss.backward()
        opt.step()
        opt.zero_grad(set_to_none=False)
        return loss

    def barrier():
        if world > 1:
            dist.barrier()

    warm = max(3, args.warmup)
    for i in range(warm):
        loss = step(*pool[i % 2])
    torch.cuda.synchronize()
    clocks = ClockSampler(torch.cuda.current_device()) if rank == 0 else None
    if clocks:
        clocks.start()
    time.sleep(0.3)
    barrier()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for i in range(args.steps):
        loss = step(*pool[i % 2])
    e.record()
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop() if clocks else None
    ms = _max_over_ranks(s.elapsed_time(e) / args.steps, dev)
    host = [(x.cpu().pin_memory(), y.cpu().pin_memory()) for x, y in pool]
    xb, yb = torch.empty_like(pool[0][0]), torch.empty_like(pool[0][1])
    barrier()
    torch.cuda.synchronize()
    s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s2.record()
    for i in range(args.steps):
        xb.copy_(host[i % 2][0], non_blocking=True)
        yb.copy_(host[i % 2][1], non_blocking=True)
        lv = step(xb, yb).item()
    e2.record()
    torch.cuda.synchronize()
    ms2 = _max_over_ranks(s2.elapsed_time(e2) / args.steps, dev)
    if rank == 0:
        print(json.dumps({
            "metric": "train images/s ViT-B/16 DDP", "value": B * world / (ms / 1e3), "unit": "images/s",
            "n_gpus": world, "steps": args.steps, "warmup": warm, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (images ~N(0,1), uniform labels, seeded; random-init weights)",
            "config": {"model": "ViT-B/16", "global_batch": B * world, "image_size": cfg.image_size,
                       "parallelism": f"dp{world}",
                       "implementation": "plain PyTorch: eager nn modules, cuBLAS, F.scaled_dot_product_attention, "
                                         "torch.optim.AdamW(fused=True), DDP over NCCL",
                       "l2": "no flush: activations of 256 images >> 126 MB L2"},
            "final_loss": float(loss.item()), "clocks": clk,
            "e2e": {"value": B * world / (ms2 / 1e3), "unit": "images/s", "ms_per_step": ms2,
                    "h2d_bytes_per_step": B * 3 * cfg.image_size ** 2 * 2 + B * 8, "d2h_bytes_per_step": 4,
                    "api": "torch module forward/backward + optimizer.step", "last_loss": lv},
            "impl": "torch"}), flush=True)
    del ddp, model, opt
    if world > 1:
        dist.destroy_process_group()
    return 0


def _max_over_ranks(v, dev):
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], device=dev)
    if dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def run_vit(args, ctx) -> int:
    """ViT-B/16 DDP training throughput (images/s): 224x224x3 images ~N(0,1), 1000 classes with
    uniform labels, batch 256 per GPU (weak scaling), AdamW, bf16; gradients through the same
    data-parallel engine (fused NVLink reduce-scatter + AdamW by default)."""
    import torch

    from brain_b200 import _native
    from brain_b200.models.config import ViTConfig
    from brain_b200.models.families import ViT
    from brain_b200.parallel import DataParallel, dist as bdist

    rank, world, dev = ctx.rank, ctx.world_size, ctx.device
    cfg = ViTConfig.vit_b16()
    B = 256
    model = ViT(cfg, device=dev, dtype=torch.bfloat16, seed=0)
    dp = DataParallel(model, lr=1e-4, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.05, grad_dtype=torch.bfloat16,
                      comm=args.comm)
    gen = torch.Generator(device=dev).manual_seed(10 + rank)
    pool = [(torch.randn(B, 3, cfg.image_size, cfg.image_size, device=dev, generator=gen).bfloat16(),
             torch.randint(0, cfg.num_classes, (B,), device=dev, generator=gen)) for _ in range(2)]
    for i in range(max(3, args.warmup)):
        loss = dp.train_step(*pool[i % 2])
    torch.cuda.synchronize()
    clocks = ClockSampler(torch.cuda.current_device()) if rank == 0 else None
    if clocks:
        clocks.start()
    time.sleep(0.3)
    bdist.barrier()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with _native.launch_counter() as lc:
        s.record()
        for i in range(args.steps):
            loss = dp.train_step(*pool[i % 2])
        e.record()
    torch.cuda.synchronize()
    bdist.barrier()
    clk = clocks.stop() if clocks else None
    ms = _max_over_ranks(s.elapsed_time(e) / args.steps, dev)
    # end to end: pinned host images uploaded every step, loss read back
    host = [(x.cpu().pin_memory(), y.cpu().pin_memory()) for x, y in pool]
    xb = torch.empty_like(pool[0][0])
    yb = torch.empty_like(pool[0][1])
    bdist.barrier()
    torch.cuda.synchronize()
    s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s2.record()
    for i in range(args.steps):
        xb.copy_(host[i % 2][0], non_blocking=True)
        yb.copy_(host[i % 2][1], non_blocking=True)
        lv = dp.train_step(xb, yb).item()
    e2.record()
    torch.cuda.synchronize()
    ms2 = _max_over_ranks(s2.elapsed_time(e2) / args.steps, dev)
    if rank == 0:
        print(json.dumps({
            "metric": "train images/s ViT-B/16 DDP", "value": B * world / (ms / 1e3), "unit": "images/s",
            "n_gpus": world, "steps": args.steps, "warmup": max(3, args.warmup), "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (images ~N(0,1), uniform labels, seeded; random-init weights)",
            "config": {"model": "ViT-B/16", "global_batch": B * world, "image_size": cfg.image_size,
                       "parallelism": f"dp{world}", "comm": args.comm,
                       "l2": "no flush: activations of 256 images >> 126 MB L2"},
            "final_loss": float(loss.item()), "clocks": clk,
            "e2e": {"value": B * world / (ms2 / 1e3), "unit": "images/s", "ms_per_step": ms2,
                    "h2d_bytes_per_step": B * 3 * cfg.image_size ** 2 * 2 + B * 8, "d2h_bytes_per_step": 4,
                    "api": "brain_b200.parallel.DataParallel.train_step", "last_loss": lv},
            "gpu_launches": lc.count, "impl": "brain"}), flush=True)
    del dp, model
    bdist.shutdown()
    return 0


def run_gptlite_cpu(args) -> int:
    """The GPT-lite data-parallel configuration on CPU ranks (Gloo): 2 decoder layers, d 128, 4 heads,
    FFN 512 GELU, LayerNorm, learned positions, vocab 1024, seq 64, batch 8 per rank, f32, weights
    N(0, 0.02) seed 0, tokens uniform seed 1, next-token CE, AdamW lr 3e-4, 20 steps, gradients
    all-reduced as the mean. Wall-clock timed (CPU), max over ranks."""
    import torch
    import torch.distributed as dist

    from brain_b200.models.config import GptLiteConfig
    from brain_b200.models.families import GptLite
    from brain_b200.optim.optimizers import AdamW
    from brain_b200.parallel import dist as bdist

    ctx = bdist.init(backend="gloo", device="cpu", timeout_s=300)
    rank, world = ctx.rank, ctx.world_size
    cfg = GptLiteConfig.lite_2x128()
    model = GptLite(cfg, device="cpu", dtype=torch.float32, seed=0)
    opt = AdamW(list(model.parameters()), lr=3e-4)
    g = torch.Generator().manual_seed(1 + rank)
    B, S = 8, cfg.max_seq_len
    steps = 20
    data = [torch.randint(0, cfg.vocab_size, (B, S + 1), generator=g) for _ in range(steps)]

    def step(t):
        opt.zero_grad()
        loss = model.loss(t[:, :-1], t[:, 1:])
        loss.backward()
        for p in model.parameters():
            if p.grad is not None and world > 1:
                dist.all_reduce(p.grad)
                p.grad.div_(world)
        opt.step()
        return float(loss)

    warm = max(3, args.warmup)
    for w in range(warm):  # warm-up on separate batches (first-call allocations), then the 20 timed steps
        step(torch.randint(0, cfg.vocab_size, (B, S + 1), generator=torch.Generator().manual_seed(10_000 + w)))
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    losses = [step(t) for t in data]
    if world > 1:
        dist.barrier()
    ms = (time.perf_counter() - t0) * 1e3 / steps
    t = torch.tensor([ms])
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    if rank == 0:
        print(json.dumps({
            "metric": "train tok/s GPT-lite DP on CPU (gloo)", "value": B * S * world / (ms / 1e3),
            "unit": "tokens/s", "n_ranks": world, "steps": steps, "warmup": warm, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "dtype": "f32", "device": "cpu",
            "data": "synthetic (uniform tokens seed 1; N(0,0.02) weights seed 0)",
            "config": {"model": "GPT-lite 2x128", "batch_per_rank": B, "seq_len": S, "parallelism": f"dp{world}"},
            "first_loss": losses[0], "last_loss": losses[-1], "impl": "brain"}), flush=True)
    bdist.shutdown()
    return 0


def _ddp_link_roofline(params: int, world: int, step_ms: float) -> dict | None:
    """Bytes each rank must receive over NVLink per data-parallel step and the time they take at the
    measured peer-copy rate: the reduce-scatter pulls (N-1)/N of the bf16 gradients, the all-gather
    returns (N-1)/N of the bf16 weights. ``share_of_step`` is that transfer time over the step time:
    the link-bound floor that the per-bucket overlap hides behind backward."""
    if world <= 1:
        return None
    link_gbs = 770.0  # measured peer copy per direction per GPU on this B200 NVSwitch system
    nbytes = 2 * (world - 1) / world * params * 2
    t_ms = nbytes / (link_gbs * 1e9) * 1e3
    return {"bytes_in_per_rank_per_step": nbytes, "link_gbs": link_gbs, "transfer_ms_at_link_rate": t_ms,
            "share_of_step": t_ms / step_ms}


def run_torch_decode(args) -> int:
    """The 70B-shape TP=N greedy decode on plain PyTorch (``brain_b200.bench.torch_decode``): cuBLAS GEMMs,
    SDPA over a contiguous KV cache, NCCL all-reduce, the step replayed from one CUDA graph (or eager with
    ``--torch-graph off``); same batch, prompt, token counts and timing rules as the framework's arm."""
    import datetime

    import torch
    import torch.distributed as dist

    from brain_b200.bench.torch_decode import TorchTPDecoder
    from brain_b200.models.config import LlamaLiteConfig

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    B, S, NEW = args.decode_batch, args.prompt_len, args.new_tokens
    cfg = LlamaLiteConfig.llama3_70b(max_seq_len=S + NEW)
    if args.decode_layers != cfg.num_layers:
        cfg = cfg.replace(num_layers=args.decode_layers)
    shard_of = args.decode_shard_of or None
    graph = args.torch_graph == "on"
    srv = TorchTPDecoder(cfg, B, S + NEW, dev, world=world, rank=rank, shard_of=shard_of, seed=0)
    prompts = torch.randint(0, cfg.vocab_size, (B, S), generator=torch.Generator().manual_seed(1))
    warm = max(3, args.warmup)
    timed = NEW - 1 - warm
    if timed < 1:
        raise ValueError("--new-tokens must exceed warm-up + 1")

    def barrier():
        if world > 1:
            dist.barrier()

    dev_prompts = prompts.to(dev)
    barrier()
    torch.cuda.synchronize()
    p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    p0.record()
    srv.prefill(dev_prompts)
    p1.record()
    srv.step(graph=False)
    if graph:
        srv.capture()
    for _ in range(warm - 1):
        srv.step(graph)
    torch.cuda.synchronize()
    clocks = ClockSampler(torch.cuda.current_device()) if rank == 0 else None
    if clocks:
        clocks.start()
    time.sleep(0.3)
    barrier()
    torch.cuda.synchronize()
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s0.record()
    for _ in range(timed):
        srv.step(graph)
    s1.record()
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop() if clocks else None
    ms = _max_over_ranks(s0.elapsed_time(s1) / timed, dev)
    prefill_ms = _max_over_ranks(p0.elapsed_time(p1), dev)
    e2e = None
    if not args.no_e2e:
        pinned = prompts.pin_memory()
        barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        out = srv.generate(pinned.to(dev, non_blocking=True), NEW, graph=graph)
        host = out.cpu()
        e1.record()
        torch.cuda.synchronize()
        e2e_ms = _max_over_ranks(e0.elapsed_time(e1), dev)
        e2e = {"value": B * NEW / (e2e_ms / 1e3), "unit": "generated tokens/s (prefill included)",
               "ms_total": e2e_ms, "h2d_bytes_per_step": B * S * 8 / NEW, "d2h_bytes_per_step": host.numel() * 8 / NEW,
               "api": "brain_b200.bench.torch_decode.TorchTPDecoder.generate"}
    if rank == 0:
        print(json.dumps({
            "metric": "decode tok/s Llama-3-70B-shape TP=N", "value": B / (ms / 1e3), "unit": "tokens/s",
            "ms_per_step": ms, "n_gpus": world, "steps": timed, "warmup": warm, "higher_is_better": True,
            "dtype": "bf16", "data": "synthetic prompts (uniform tokens, seeded); random-init N(0,0.02) weights",
            "config": {"model": "Llama-3-70B-shape" + ("" if cfg.num_layers == 80 else f" ({cfg.num_layers} layers: NOT the benchmark)"),
                       "batch": B, "prompt_len": S, "new_tokens": NEW,
                       "parallelism": f"tp{world}" if not shard_of else f"one rank's shard of tp{shard_of} (NOT the benchmark)",
                       "kv_cache": "contiguous, read to capacity under a mask",
                       "decode_step": "one CUDA graph of torch ops" if graph else "eager torch ops",
                       "implementation": "plain PyTorch: F.linear (cuBLAS), F.scaled_dot_product_attention, "
                                         "F.rms_norm, NCCL all_reduce / all_gather",
                       "l2": "no flush: each step streams the rank's weights (>> 126 MB L2)"},
            "prefill_ms": prefill_ms, "prefill_tok_s": B * S / (prefill_ms / 1e3),
            "clocks": clk, "e2e": e2e, "impl": "torch"}), flush=True)
    srv.close()
    del srv
    if world > 1:
        dist.destroy_process_group()
    return 0


def run_decode(args, rank, world, dev) -> dict:
    """Llama-3-70B-shaped greedy decode, tensor parallel over all ranks (TP = N): prefill B prompts of
    S uniform tokens, then decode; the decode steps are CUDA-graph replays of the fused decode kernels.
    Returns the decode measurement (decode tokens/s over all sequences, max over ranks)."""
    import torch
    import torch.distributed as dist

    from brain_b200.models import LlamaLiteConfig
    from brain_b200.models.llama_tp import LlamaTPServe, decode_bytes_per_step
    from brain_b200.ops.decode import set_pdl
    from brain_b200.parallel import dist as bdist

    B, S, NEW = args.decode_batch, args.prompt_len, args.new_tokens
    cfg = LlamaLiteConfig.llama3_70b(max_seq_len=S + NEW)
    if args.decode_layers != cfg.num_layers:
        cfg = cfg.replace(num_layers=args.decode_layers)
    t0 = time.time()
    shard_of = args.decode_shard_of or None
    set_pdl(args.decode_pdl)
    srv = LlamaTPServe(cfg, max_batch=B, max_len=S + NEW, block_size=64, seed=0, shard_of=shard_of,
                       l2_prefetch=args.l2_prefetch)
    torch.cuda.synchronize()
    log(f"{bdist.rank_prefix()} 70B-shape TP={world} shard ready in {time.time() - t0:.1f}s, "
        f"mem {torch.cuda.memory_allocated() / 2**30:.1f} GiB")
    prompts = torch.randint(0, cfg.vocab_size, (B, S), generator=torch.Generator().manual_seed(1))
    warm = max(3, args.warmup)
    timed = NEW - 1 - warm
    if timed < 1:
        raise ValueError("--new-tokens must exceed warm-up + 1")

    def max_over_ranks(v):
        t = torch.tensor([v], device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---- device-timed: prefill, then `warm` steps (1 eager + replays), then `timed` replays
    dev_prompts = prompts.to(dev)
    bdist.barrier()
    torch.cuda.synchronize()
    p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    p0.record()
    srv.prefill(dev_prompts)
    p1.record()
    srv.step()
    srv.capture()
    for _ in range(warm - 1):
        srv.replay()
    torch.cuda.synchronize()
    clocks = ClockSampler(torch.cuda.current_device()) if rank == 0 else None
    if clocks:
        clocks.start()
    time.sleep(0.3)
    bdist.barrier()
    torch.cuda.synchronize()
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s0.record()
    for _ in range(timed):
        srv.replay()
    s1.record()
    torch.cuda.synchronize()
    bdist.barrier()
    clk = clocks.stop() if clocks else None
    srv.check()
    ms = max_over_ranks(s0.elapsed_time(s1) / timed)
    prefill_ms = max_over_ranks(p0.elapsed_time(p1))
    tokens = srv.hist[:, :S + NEW].cpu()

    # ---- end to end through the public API: pinned prompt upload, generate, tokens back to the host
    e2e = None
    if not args.no_e2e:
        pinned = prompts.pin_memory()
        bdist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        out = srv.generate(pinned.to(dev, non_blocking=True), NEW, use_graph=True)
        e1.record()
        torch.cuda.synchronize()
        e2e_ms = max_over_ranks(e0.elapsed_time(e1))
        e2e = {"value": B * NEW / (e2e_ms / 1e3), "unit": "generated tokens/s (prefill included)",
               "ms_total": e2e_ms, "h2d_bytes_per_step": B * S * 8 / NEW, "d2h_bytes_per_step": B * (S + NEW) * 8 / NEW,
               "api": "brain_b200.models.llama_tp.LlamaTPServe.generate",
               "same_tokens_as_timed_run": bool(torch.equal(out, tokens.long()))}
    avg_len = S + 1 + warm + timed / 2
    hbm = decode_bytes_per_step(cfg, shard_of or world, B, avg_len)
    res = {
        "metric": "decode tok/s Llama-3-70B-shape TP=N", "value": B / (ms / 1e3), "unit": "tokens/s",
        "ms_per_step": ms, "n_gpus": world, "steps": timed, "warmup": warm, "higher_is_better": True,
        "dtype": "bf16", "data": "synthetic prompts (uniform tokens, seeded); random-init N(0,0.02) weights",
        "config": {"model": "Llama-3-70B-shape" + ("" if cfg.num_layers == 80 else f" ({cfg.num_layers} layers: NOT the benchmark)"),
                   "batch": B, "prompt_len": S, "new_tokens": NEW,
                   "parallelism": f"tp{world}" if not shard_of else f"one rank's shard of tp{shard_of} (NOT the benchmark)",
                   "kv_cache": "paged, block 64", "pdl_mode": args.decode_pdl,
                   "l2_prefetch": args.l2_prefetch, "decode_step": "one CUDA graph of hand-written kernels",
                   "l2": "no flush: each step streams the rank's weights (>> 126 MB L2)"},
        "prefill_ms": prefill_ms, "prefill_tok_s": B * S / (prefill_ms / 1e3),
        "hbm_bytes_per_step_per_gpu": hbm, "hbm_gbs_achieved": hbm / (ms / 1e3) / 1e9,
        "clocks": clk, "e2e": e2e, "gpu_launches": srv.launches_per_step() * timed, "impl": "brain",
    }
    srv.close()
    del srv
    return res


if __name__ == "__main__":
    sys.exit(main())
