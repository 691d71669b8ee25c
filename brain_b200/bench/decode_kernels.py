"""Decode-kernel microbenchmark on one GPU: the per-rank shapes of Llama-3-70B at TP=8 (or any TP
degree), batch 32, each kernel device-timed with CUDA events and reported against the HBM bytes it
must move (weights are rotated over enough copies that they never sit in the 126 MB L2).

Run: ``python -m brain_b200.bench.decode_kernels [--tp 8] [--batch 32] [--kv-len 2176]``; one JSON
line per kernel: {"kernel", "us", "bytes", "gbs", "frac_of_measured_hbm"}.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import sys

import torch


def _peak_hbm() -> float:
    here = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    try:
        with open(os.path.join(here, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"])
    except (OSError, KeyError, ValueError):
        return 6650.0


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--tp", type=int, default=8)
    ap.add_argument("--batch", type=int, default=32)
    ap.add_argument("--kv-len", type=int, default=2176)
    ap.add_argument("--iters", type=int, default=50)
    ap.add_argument("--splits", type=int, default=0, help="force a split-K count (0 = automatic)")
    ap.add_argument("--only", default="", help="comma-separated kernel names to run (default: all)")
    ap.add_argument("--attn-splits", default="", help="comma-separated decode-attention split counts to add")
    ap.add_argument("--pdl", type=int, default=2, help="programmatic dependent launch mode (see set_pdl)")
    ap.add_argument("--no-pdl", action="store_true", help="launch without programmatic dependent launch")
    ap.add_argument("--trace", action="store_true",
                    help="also run each GEMM once with per-CTA phase timestamps and print their spread")
    a = ap.parse_args(argv)
    only = set(x for x in a.only.split(",") if x)

    from ..models import LlamaLiteConfig
    from ..ops import check_status
    from ..ops.decode import (EPI_ARGMAX, EPI_PUSH, EPI_QKV, EPI_STORE, EPI_SWIGLU, ar_norm, decode_ext,
                              decode_splits, init_ar_slots, paged_decode_attention, set_pdl, skinny_gemm,
                              skinny_splits)
    from ..ops.rope import rope_table

    cfg = LlamaLiteConfig.llama3_70b()
    W, B, dev = a.tp, a.batch, torch.device("cuda")
    d, D = cfg.hidden_dim, cfg.head_dim
    hq, hkv, F = cfg.num_heads // W, cfg.num_kv_heads // W, cfg.intermediate_dim // W
    Vs = -(-cfg.vocab_size // W)
    peak = _peak_hbm()
    set_pdl(0 if a.no_pdl else a.pdl)
    g = torch.Generator(device=dev).manual_seed(0)

    def rnd(*shape, std=0.02):
        return (torch.randn(*shape, device=dev, generator=g) * std).bfloat16()

    def copies(shape):
        nbytes = 2 * math.prod(shape)
        k = max(2, math.ceil(512e6 / nbytes))  # > 4x L2 per rotation
        return [rnd(*shape) for _ in range(k)]

    x = rnd(B, d, std=1.0)
    xa = rnd(B, hq * D, std=1.0)
    xf = rnd(B, F, std=1.0)
    out = torch.empty(B, max(d, 2 * F, Vs), device=dev, dtype=torch.bfloat16)

    def timeit(fn, n):
        """Device time per call: n calls captured in one CUDA graph (no host launch cost), replayed."""
        for i in range(3):
            fn(i)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for i in range(n):
                fn(i)
        graph.replay()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        graph.replay()
        e.record()
        torch.cuda.synchronize()
        return s.elapsed_time(e) * 1e3 / n

    def want(name):
        return not only or name in only

    def report(name, us, nbytes, **extra):
        gbs = nbytes / (us * 1e-6) / 1e9
        print(json.dumps({"kernel": name, "us": round(us, 2), "bytes": nbytes, "gbs": round(gbs, 1),
                          "frac_of_measured_hbm": round(gbs / peak, 3), **extra}), flush=True)

    def gemm_case(name, N, K, epi, inp, ext_fn=lambda trace: decode_ext(trace=trace)):
        if not want(name):
            return
        ws = copies((N, K))
        sp = a.splits or skinny_splits(B, N, K)
        o = out[:, :N // 2] if epi == EPI_SWIGLU else out[:, :N]
        ext = ext_fn(None)

        def fn(i, ext=ext):
            skinny_gemm(inp, ws[i % len(ws)], epi, out=None if epi in (EPI_PUSH, EPI_ARGMAX) else o,
                        splits=sp, ext=ext)
        us = timeit(fn, a.iters)
        report(name, us, 2 * N * K + 2 * B * K + 2 * B * N, splits=sp, N=N, K=K)
        if a.trace:
            ctas = sp * -(-N // 128)
            tr = torch.zeros(ctas * 16, device=dev, dtype=torch.int64)
            tr_prev = torch.zeros_like(tr)
            torch.cuda.synchronize()
            fn(0, ext=ext_fn(tr_prev))
            fn(1, ext=ext_fn(tr))
            torch.cuda.synchronize()
            t = tr.view(ctas, 16).cpu().double()
            tp = tr_prev.view(ctas, 16).cpu().double()
            gap = {"prev_last_end_to_first_start_us": round(float(t[:, 0].min() - tp[:, 6].max()) / 1e3, 2),
                   "prev_span_us": round(float(tp[:, 6].max() - tp[:, 0].min()) / 1e3, 2)}
            base = t[:, 0].min()
            phases = {}
            for k, nm in enumerate(["start", "setup", "pdl_wait", "mma_done", "cluster_sync1", "cluster_sync2",
                                    "end"]):
                col = t[:, k]
                col = col[col > 0]
                if len(col):
                    d = (col - base) / 1e3
                    phases[nm] = [round(float(d.median()), 2), round(float(d.max()), 2)]
            steps = [("pdl_wait", 8, 9), ("stage_and_send", 9, 10), ("receive_wait", 10, 11),
                     ("reduce_epilogue", 11, 15)]
            if epi == EPI_PUSH:
                steps += [("push_stores", 11, 12), ("push_syncthreads", 12, 13), ("push_release_arrive", 13, 14)]
            cyc = {nm: round(float((t[:, b] - t[:, a_]).median()), 0) for nm, a_, b in steps}
            print(json.dumps({"trace": name, "us_median_max_since_first_start": phases,
                              "sm_cycles_median_per_step": cyc, "launch_gap": gap}), flush=True)

    # ---- QKV + RoPE + paged KV append
    bs = 64
    max_blocks = -(-(a.kv_len + 8) // bs)
    kv = torch.zeros(2, B * max_blocks, bs, hkv, D, device=dev, dtype=torch.bfloat16)
    table = torch.arange(B * max_blocks, device=dev, dtype=torch.int32).view(B, max_blocks)
    pos = torch.full((B,), a.kv_len - 1, device=dev, dtype=torch.int32)
    lens = pos + 1
    cs = rope_table(D, a.kv_len + 8, cfg.rope_theta, device=dev)
    gemm_case("skinny_gemm_qkv_rope", (hq + 2 * hkv) * D, d, EPI_QKV, x,
              lambda tr: decode_ext(hq=hq, hkv=hkv, pos=pos, rope_cs=cs, k_pool=kv[0], v_pool=kv[1],
                                    block_table=table, trace=tr))
    # ---- decode attention over the paged cache
    kv.normal_()
    q = rnd(B, hq, D, std=1.0)
    ao = torch.empty(B, hq, D, device=dev, dtype=torch.bfloat16)
    if want("paged_decode_attention"):
        # one layer's cache per call, rotating over caches larger than L2 together (as the 80 layers of a
        # decode step are): the K/V come from HBM
        ncache = max(2, math.ceil(512e6 / kv.numel() / 2))
        caches = [kv] + [torch.randn_like(kv) for _ in range(ncache - 1)]
        nbytes = B * a.kv_len * hkv * D * 2 * 2
        for sp in [None] + [int(x) for x in a.attn_splits.split(",") if x]:
            us = timeit(lambda i, sp=sp: paged_decode_attention(q, caches[i % ncache][0], caches[i % ncache][1], table,
                                                                lens, out=ao, splits=sp), a.iters)
            spn = sp or decode_splits(B, hkv, D, max_blocks * bs)
            report("paged_decode_attention", us, nbytes, kv_len=a.kv_len, splits=spn)
            if a.trace:
                tr = torch.zeros(B * hkv * spn * 8, device=dev, dtype=torch.int64)
                names = ["start", "len_read", "pdl_wait", "q_loaded", "first_chunk", "loop_end", "cluster_sync",
                         "end"]
                tr_prev = torch.zeros_like(tr)
                for mode in ("isolated", "after_previous"):
                    torch.cuda.synchronize()
                    if mode == "after_previous":
                        paged_decode_attention(q, caches[1][0], caches[1][1], table, lens, out=ao, splits=spn,
                                               trace=tr_prev)
                    paged_decode_attention(q, caches[2][0], caches[2][1], table, lens, out=ao, splits=spn, trace=tr)
                    torch.cuda.synchronize()
                    t = tr.view(-1, 8).cpu().double()
                    gap = None
                    if mode == "after_previous":
                        tp = tr_prev.view(-1, 8).cpu().double()
                        gap = {"prev_last_end_to_first_start_us": round(float(t[:, 0].min() - tp[:, 7].max()) / 1e3, 2),
                               "prev_first_end_to_first_start_us": round(float(t[:, 0].min() - tp[:, 7].min()) / 1e3, 2),
                               "prev_span_us": round(float(tp[:, 7].max() - tp[:, 0].min()) / 1e3, 2)}
                    base = t[:, 0].min()
                    rel = (t - base) / 1e3
                    phases = {nm: [round(float(rel[:, k].median()), 2), round(float(rel[:, k].max()), 2)]
                              for k, nm in enumerate(names)}
                    steps = {f"{names[k]}->{names[k + 1]}": round(float((t[:, k + 1] - t[:, k]).median()) / 1e3, 2)
                             for k in range(7)}
                    print(json.dumps({"trace": "paged_decode_attention", "splits": spn, "mode": mode,
                                      "us_median_max_since_first_start": phases, "us_median_per_step": steps,
                                      "launch_gap": gap}), flush=True)
        del caches
    # ---- out projection with all-reduce push (single rank: pushes to itself)
    slot = B * d
    slots = init_ar_slots(torch.empty(2 * slot, device=dev, dtype=torch.bfloat16))
    ctrl = torch.zeros(4, device=dev, dtype=torch.int32)
    def push_ext(tr=None):
        return decode_ext(world=1, rank=0, slot_elems=slot, ctrl=ctrl, peer_slots=[slots.data_ptr()], trace=tr)
    ext_push = push_ext()
    resid = rnd(B, d, std=1.0)
    gamma = torch.ones(d, device=dev, dtype=torch.bfloat16)
    normed = torch.empty_like(resid)

    def o_and_norm(i, w=copies((d, hq * D)) if want("o_push+ar_norm") else None):
        skinny_gemm(xa, w[i % len(w)], EPI_PUSH, ext=ext_push, splits=a.splits or skinny_splits(B, d, hq * D))
        ar_norm(slots.data_ptr(), ctrl, 1, slot, resid, gamma, 1e-5, normed)
    gemm_case("skinny_gemm_o_push", d, hq * D, EPI_PUSH, xa, push_ext)
    if want("o_push+ar_norm"):
        us = timeit(o_and_norm, a.iters)
        report("o_push+ar_norm", us, 2 * d * hq * D)
    # ---- gate/up with fused SwiGLU, down projection with push
    gemm_case("skinny_gemm_gate_up_swiglu", 2 * F, d, EPI_SWIGLU, x)
    gemm_case("skinny_gemm_down_push", d, F, EPI_PUSH, xf, push_ext)
    gemm_case("skinny_gemm_store_down", d, F, EPI_STORE, xf)
    gemm_case("skinny_gemm_store_o", d, hq * D, EPI_STORE, xa)
    # ---- vocabulary-parallel head with fused argmax
    keys = torch.zeros(B, device=dev, dtype=torch.int64)
    kslots = torch.zeros(2 * B, device=dev, dtype=torch.int64)
    gemm_case("skinny_gemm_head_argmax", Vs, d, EPI_ARGMAX, x,
              lambda tr: decode_ext(world=1, rank=0, slot_elems=B, ctrl=ctrl, keys=keys,
                                    peer_slots=[kslots.data_ptr()], trace=tr))
    bad = check_status()
    if bad:
        print(json.dumps({"error": f"kernel status {bad}"}), flush=True)
        return 1
    return 0


if __name__ == "__main__":
    sys.exit(main())
