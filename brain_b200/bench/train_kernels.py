"""Training-kernel microbenchmark on one GPU at Llama-3-8B shapes (micro-batch 2 x seq 4096 = 8192
tokens): the tcgen05 GEMMs of a layer (forward, data and weight gradients), flash attention forward and
backward (32 q / 8 kv heads, head_dim 128, causal), RMSNorm, SwiGLU, RoPE, the fused LM-head
cross-entropy and AdamW. Each is timed with CUDA events over a few calls after warm-up and reported as
TFLOP/s or GB/s against the measured peaks (``MEASURED_PEAKS.json`` at the repository root).

Run: ``python -m brain_b200.bench.train_kernels [--only name,...] [--iters N]``; one JSON line per case.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import torch


def _peaks():
    here = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    try:
        with open(os.path.join(here, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["bf16_tflops"]), float(d["hbm_gbs"])
    except (OSError, KeyError, ValueError):
        return 1590.0, 6650.0


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", default="")
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--graph", action="store_true",
                    help="replay each case from a CUDA graph, so short kernels are timed without the per-call "
                         "host overhead (cases that cannot be captured fall back to eager calls)")
    ap.add_argument("--gemm-pair", default="auto", choices=["auto", "off"],
                    help="off: the single-CTA tcgen05 GEMM even where the CTA-pair kernel would run")
    a = ap.parse_args(argv)
    only = set(x for x in a.only.split(",") if x)

    from .. import ops
    from ..ops import attention as attn
    from ..ops.optim_kernels import adamw_

    dev = torch.device("cuda")
    tflops_peak, hbm_peak = _peaks()
    if a.gemm_pair == "off":
        from ..ops.gemm import set_pair_mode
        set_pair_mode(0)
    g = torch.Generator(device=dev).manual_seed(0)
    T, d, F, V = 8192, 4096, 14336, 128256
    B, S, Hq, Hkv, D = 2, 4096, 32, 8, 128

    def rnd(*shape, std=1.0):
        return (torch.randn(*shape, device=dev, generator=g) * std).bfloat16()

    def timeit(fn):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        run = fn
        if a.graph:
            try:
                graph = torch.cuda.CUDAGraph()
                side = torch.cuda.Stream()
                side.wait_stream(torch.cuda.current_stream())
                with torch.cuda.stream(side):
                    with torch.cuda.graph(graph):
                        fn()
                torch.cuda.current_stream().wait_stream(side)
                run = graph.replay
                run()
                torch.cuda.synchronize()
            except Exception as exc:  # not capturable: time eager calls
                print(json.dumps({"graph_capture_failed": str(exc)[:200]}), flush=True)
                torch.cuda.synchronize()
                run = fn
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(a.iters):
            run()
        e.record()
        torch.cuda.synchronize()
        return s.elapsed_time(e) / a.iters

    def report(name, ms, flops=None, nbytes=None, **extra):
        out = {"kernel": name, "ms": round(ms, 4)}
        if flops:
            tf = flops / (ms / 1e3) / 1e12
            out.update(tflops=round(tf, 1), frac_of_measured_bf16=round(tf / tflops_peak, 3))
        if nbytes:
            gbs = nbytes / (ms / 1e3) / 1e9
            out.update(gbs=round(gbs, 1), frac_of_measured_hbm=round(gbs / hbm_peak, 3))
        out.update(extra)
        print(json.dumps(out), flush=True)

    def want(n):
        return not only or n in only

    # ---- GEMMs of one layer: x W^T forward, dy W (dgrad), dy^T x (wgrad, f32 accumulate)
    x = rnd(T, d)
    for name, N, K in (("qkv", (Hq + 2 * Hkv) * D, d), ("o", d, Hq * D), ("gate_up", 2 * F, d), ("down", d, F)):
        if not any(want(f"gemm_{kind}_{name}") for kind in ("fwd", "dgrad", "wgrad")):
            continue  # allocate only what the selected cases use
        w = rnd(N, K, std=0.02)
        xi = x if K == d else rnd(T, K)
        dy = rnd(T, N)
        fl = 2.0 * T * N * K
        if want(f"gemm_fwd_{name}"):
            report(f"gemm_fwd_{name}", timeit(lambda: ops.gemm(xi, w, trans_b=True)), fl, M=T, N=N, K=K)
        if want(f"gemm_dgrad_{name}"):
            report(f"gemm_dgrad_{name}", timeit(lambda: ops.gemm(dy, w)), fl, M=T, N=K, K=N)
        if want(f"gemm_wgrad_{name}"):
            acc = torch.zeros(N, K, device=dev, dtype=torch.float32)
            report(f"gemm_wgrad_{name}", timeit(lambda: ops.gemm(dy, xi, trans_a=True, out=acc, beta=1.0)), fl,
                   M=N, N=K, K=T)
    # ---- fused QKV projection with RoPE on the q / k heads in the GEMM epilogue
    if want("gemm_fwd_qkv_rope"):
        from ..ops.gemm import gemm_rope
        N = (Hq + 2 * Hkv) * D
        wq = rnd(N, d, std=0.02)
        table = ops.rope_table(D, S, 500000.0, device=dev)
        report("gemm_fwd_qkv_rope", timeit(lambda: gemm_rope(x, wq, table, (Hq + Hkv) * D, D, S, 0)),
               2.0 * T * N * d, M=T, N=N, K=d)
    # ---- block-scaled fp8 GEMM (1 x 128 activation, 128 x 128 weight scales) against bf16, 16384 x 8192 x 4096
    if want("gemm_fp8") or want("gemm_bf16_square") or want("gemm_fp8_rowwise"):
        from ..quantization.fp8 import (fp8_gemm_blockscaled, fp8_gemm_rowwise, quantize_fp8_blockwise,
                                        quantize_fp8_rowwise, quantize_fp8_weight_blocks)
        Mq, Nq, Kq = 16384, 8192, 4096
        xa, wb = rnd(Mq, Kq), rnd(Nq, Kq, std=0.02)
        fl = 2.0 * Mq * Nq * Kq
        if want("gemm_bf16_square"):
            report("gemm_bf16_square", timeit(lambda: ops.gemm(xa, wb, trans_b=True)), fl, M=Mq, N=Nq, K=Kq)
        if want("gemm_fp8"):
            aq, sa = quantize_fp8_blockwise(xa)
            bq, sb = quantize_fp8_weight_blocks(wb)
            report("gemm_fp8", timeit(lambda: fp8_gemm_blockscaled(aq, sa, bq, sb)), fl, M=Mq, N=Nq, K=Kq,
                   note="tensor FLOPs at fp8; the bf16 figure is the denominator for both")
            report("fp8_quantize_activations", timeit(lambda: quantize_fp8_blockwise(xa)), None,
                   nbytes=Mq * Kq * 3 + Mq * Kq // 128 * 4)
        if want("gemm_fp8_rowwise"):
            aq, sa = quantize_fp8_rowwise(xa)
            bq, sb = quantize_fp8_rowwise(wb)
            report("gemm_fp8_rowwise", timeit(lambda: fp8_gemm_rowwise(aq, sa, bq, sb)), fl, M=Mq, N=Nq, K=Kq,
                   note="tensor FLOPs at fp8 (CTA pair, scales in the epilogue); bf16 peak as the denominator")
            report("fp8_quantize_rowwise", timeit(lambda: quantize_fp8_rowwise(xa)), None,
                   nbytes=Mq * Kq * 3 + Mq * 4)
    # ---- flash attention (causal): forward 2 GEMMs of S x S x D per head over half the square
    q, k, v = rnd(B, S, Hq, D), rnd(B, S, Hkv, D), rnd(B, S, Hkv, D)
    fwd_flops = 4.0 * B * Hq * S * S * D / 2
    if want("attention_fwd"):
        report("attention_fwd", timeit(lambda: attn._fwd(q, k, v, True, D ** -0.5)), fwd_flops)
    if want("attention_bwd"):
        o, lse = attn._fwd(q, k, v, True, D ** -0.5)
        do = rnd(B, S, Hq, D)
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        report("attention_bwd", timeit(lambda: attn._bwd(q, k, v, o, lse, do, dq, dk, dv, True, D ** -0.5)),
               2.5 * fwd_flops)
    # ---- memory-bound ops
    if want("rms_norm_fwd"):
        wn = torch.ones(d, device=dev, dtype=torch.bfloat16)
        report("rms_norm_fwd", timeit(lambda: ops.rms_norm(x, wn)), nbytes=2 * T * d * 2)
    if want("swiglu_fwd"):
        gu = rnd(T, 2 * F)
        report("swiglu_fwd", timeit(lambda: ops.activations.swiglu_fwd_only(gu)), nbytes=T * 3 * F * 2)
    if want("rms_norm_bwd"):
        from ..ops import norms as _norms
        wn = torch.ones(d, device=dev, dtype=torch.bfloat16)
        dy = rnd(T, d)
        _, _, _, rstd = _norms._fwd(_norms._RMS, x, wn, None, 1e-5)
        report("rms_norm_bwd", timeit(lambda: _norms._bwd(_norms._RMS, dy, x, wn, None, None, rstd)),
               nbytes=3 * T * d * 2)
    if want("swiglu_bwd"):
        gu = rnd(T, 2 * F)
        dy = rnd(T, F)
        report("swiglu_bwd", timeit(lambda: ops.activations.swiglu_bwd_only(dy, gu)), nbytes=T * 5 * F * 2)
    if want("rope_inplace"):
        qkv = rnd(B, S, (Hq + 2 * Hkv) * D)
        table = ops.rope_table(D, S, 500000.0, device=dev)
        qv = qkv.view(B, S, Hq + 2 * Hkv, D)[:, :, :Hq + Hkv]
        report("rope_inplace", timeit(lambda: ops.apply_rope_(qv, table)), nbytes=2 * B * S * (Hq + Hkv) * D * 2)
    if want("lm_head_cross_entropy"):
        hw = rnd(V, d, std=0.02)
        labels = torch.randint(0, V, (T,), device=dev, generator=g)
        h = rnd(T, d).requires_grad_(True)

        def ce():
            loss = ops.linear_cross_entropy(h, hw, labels)
            loss.backward()
        report("lm_head_cross_entropy_fwd_bwd", timeit(ce), 3 * 2.0 * T * V * d)
    if want("adamw"):
        n = 1 << 28
        p = torch.zeros(n, device=dev)
        m, vv = torch.zeros_like(p), torch.zeros_like(p)
        gr = torch.zeros(n, device=dev, dtype=torch.bfloat16)
        p16 = torch.zeros(n, device=dev, dtype=torch.bfloat16)
        report("adamw_flat", timeit(lambda: adamw_(p, m, vv, gr, lr=1e-3, beta1=0.9, beta2=0.95, eps=1e-8,
                                                    weight_decay=0.1, step=1, p16=p16)),
               nbytes=n * (12 + 12 + 2 + 2), elems=n)
    return 0


if __name__ == "__main__":
    sys.exit(main())
