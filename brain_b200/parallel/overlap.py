"""Gradient reduction overlapped with backward for ``DataParallel`` on the NVLink backend.

The flat gradient buffer is cut into buckets of whole transformer blocks, in the order backward
finishes them (the LM head and the last blocks first, the embedding last). Each bucket is sharded
over the ranks on its own: rank r owns piece r of every bucket and keeps the f32 master weights and
AdamW moments of its pieces. When backward has finished the blocks of a bucket (a backward hook on
the bucket's earliest block records an event on the compute stream), a side stream waits for that
event, runs a peer barrier (every rank's gradients of the bucket are complete) and then the fused
kernel for the bucket: it pulls the peers' gradients of this rank's piece over NVLink, reduces and
scales them, applies AdamW in the reference's order (decay, moments, bias-corrected update) and
pushes the updated bf16 weights into every rank's parameter buffer. The push is safe while backward
continues on the peers: a peer passed the bucket's barrier only after it finished those blocks, and
blocks of other buckets are not touched. The step ends with the remaining buckets, the compute stream
waiting for the side stream and a closing barrier, so the next forward sees every rank's update.

Reference: DataParallel::sync_gradients reduces by the mean after backward
(crates/brain-distributed/src/data_parallel.rs:32-70) and Adam::step applies the update
(crates/brain-optim/src/adam/mod.rs:95-214); here the two are fused and run during backward.
"""
from __future__ import annotations

import torch

from .. import _native

_native.register({
    "brain_comm_ddp_step_ctas": ("brain_comm", "ppiiillpppffffffffiis"),
    "brain_comm_copy_async": ("brain_comm", "llls"),
})


def _i64(vals):
    import ctypes
    return (ctypes.c_int64 * len(vals))(*[int(v) for v in vals])


def _blocks(model):
    for name in ("layers", "blocks"):
        mods = getattr(model, name, None)
        if isinstance(mods, torch.nn.ModuleList) and len(mods) > 0:
            return list(mods)
    enc = getattr(model, "encoder", None)
    if enc is not None:
        return _blocks(enc)
    return []


class OverlappedStep:
    def __init__(self, dp, bucket_bytes: int = 512 << 20, max_ctas: int = 64, mode: str = "ce"):
        """mode "ce": the copy engines pull the peers' gradient pieces into local staging and publish the
        updated weights, so only a short local reduce + AdamW kernel shares the SMs with backward;
        mode "sm": one kernel pulls, updates and pushes over NVLink with SM loads and stores."""
        self.dp = dp
        flat, opt = dp.flat, dp.optimizer
        self.flat, self.opt, self.comm = flat, opt, dp.comm
        self.world, self.rank = flat.world_size, flat.rank
        self.max_ctas = max_ctas
        self.mode = mode
        esz = flat.param_buf.element_size()
        index = {id(p): (o, p.numel()) for p, o in zip(flat.params, flat.offsets)}
        blocks = _blocks(dp.model)
        ranges = []  # (lo, hi, block) in flat order
        for blk in blocks:
            spans = [index[id(p)] for p in blk.parameters() if id(p) in index]
            if not spans:
                continue
            lo = min(o for o, _ in spans)
            hi = max(o + -(-n // 64) * 64 for o, n in spans)
            ranges.append((lo, hi, blk))
        ranges.sort(key=lambda r: r[0])
        contiguous = all(ranges[i][1] == ranges[i + 1][0] for i in range(len(ranges) - 1))
        if not ranges or not contiguous:
            raise ValueError("overlapped reduction needs the blocks' parameters contiguous in the flat buffer")
        # buckets in backward order: [tail params + last blocks], ..., [first blocks], [head params]
        self.buckets = []  # (lo, hi, trigger block or None)
        hi = flat.padded
        cur_hi, acc = hi, 0
        for lo, bhi, blk in reversed(ranges):
            acc += (bhi - lo) * esz
            if acc >= bucket_bytes:
                self.buckets.append((lo, cur_hi, blk))
                cur_hi, acc = lo, 0
        first_lo = ranges[0][0]
        if cur_hi > first_lo:
            self.buckets.append((first_lo, cur_hi, ranges[0][2]))
            cur_hi = first_lo
        if cur_hi > 0:
            self.buckets.append((0, cur_hi, None))  # embedding & co: reduced after backward returns
        # this rank's piece of every bucket, and its place in the concatenated optimizer state
        self.pieces = []  # (global offset, length, state offset)
        st = 0
        for lo, bhi, _ in self.buckets:
            piece = -(-(bhi - lo) // (self.world * 8)) * 8
            a = min(bhi, lo + self.rank * piece)
            b = min(bhi, a + piece)
            self.pieces.append((a, b - a, st))
            st += b - a
        # the flat optimizer's own shard state is not used: release it before allocating this layout's
        opt.master = opt.m = opt.v = None
        if flat.grad_buf.is_cuda:
            torch.cuda.empty_cache()
        with torch.no_grad():
            self.master = torch.empty(st, device=flat.param_buf.device, dtype=torch.float32)
            for a, n, s in self.pieces:
                self.master[s:s + n].copy_(flat.param_buf[a:a + n])
        self.m = torch.zeros_like(self.master)
        self.v = torch.zeros_like(self.master)
        if self.world == 1:
            # a single GPU: the per-bucket step is AdamW alone, on this GPU's own buffers
            self.gpeers = _i64([flat.grad_buf.data_ptr()])
            self.ppeers = _i64([flat.param_buf.data_ptr()])
        else:
            self.gbuf, goff = self.comm._buf_of(flat.grad_buf)
            self.pbuf, poff = self.comm._buf_of(flat.param_buf)
            if self.gbuf is None or self.pbuf is None:
                raise ValueError("overlapped reduction needs symmetric gradient and parameter buffers")
            self.gpeers = self.gbuf.peer_array(goff)
            self.ppeers = self.pbuf.peer_array(poff)
        self.gesz = flat.grad_buf.element_size()
        if mode == "ce":
            most = max(n for _, n, _ in self.pieces)
            self.staging = torch.empty(self.world, max(most, 8), device=flat.grad_buf.device, dtype=flat.grad_buf.dtype)
        self.bucket_params = [flat.params_in(lo, hi) for lo, hi, _ in self.buckets]
        self.side = torch.cuda.Stream()
        self.fired = [False] * len(self.buckets)
        self.hooks = []
        for i, (_, _, blk) in enumerate(self.buckets):
            if blk is not None:
                self.hooks.append(blk.register_full_backward_hook(lambda mod, gin, gout, i=i: self._launch(i)))
        self.args = None
        self.guarded, self.max_norm, self.stats_started = False, 0.0, False

    def arm(self, grad_scale: float, guarded: bool = False, max_norm: float = 0.0) -> None:
        """Before backward: this step's AdamW constants. ``guarded``: during backward each bucket is
        only reduced (into this rank's piece of the gradient buffer) and its statistics accumulated;
        AdamW runs in ``finish`` once the statistics of every bucket on every rank are known, so a
        non-finite element anywhere skips the step on all ranks and clipping uses the global norm."""
        opt = self.opt
        opt.step_count += 1
        t = opt.step_count
        b1, b2 = opt.betas
        self.args = (float(opt.lr), float(b1), float(b2), float(opt.eps), float(opt.weight_decay),
                     float(1 - b1 ** t), float(1 - b2 ** t), float(grad_scale))
        self.guarded, self.max_norm = guarded, float(max_norm)
        self.stats_started = False
        self.fired = [False] * len(self.buckets)

    def _launch(self, i: int) -> None:
        if self.args is None or self.fired[i]:
            return
        self.fired[i] = True
        self.flat.finalize_grads(self.bucket_params[i])  # parameters of the bucket no producer wrote
        ev = torch.cuda.Event()
        ev.record()
        a, n, s = self.pieces[i]
        lr, b1, b2, eps, wd, bc1, bc2, gs = self.args
        W, r, ge = self.world, self.rank, self.gesz
        bf16 = int(self.flat.grad_buf.dtype == torch.bfloat16)
        state = (self.master.data_ptr() + 4 * s, self.m.data_ptr() + 4 * s, self.v.data_ptr() + 4 * s)
        with torch.cuda.stream(self.side):
            self.side.wait_event(ev)
            if W > 1:
                self.comm.barrier(50)
            if n == 0:
                return
            if self.guarded:
                self._reduce_piece(a, n, gs)
                return
            if self.mode == "sm":
                _native.call("brain_comm_ddp_step_ctas", self.gpeers, self.ppeers, bf16, r, W, a, n, *state,
                             lr, b1, b2, eps, wd, bc1, bc2, gs, self.max_ctas, W, self.side.cuda_stream)
                return
            st = self.side.cuda_stream
            srcs = []
            for jj in range(W):
                j = (r + jj) % W
                if j == r:
                    srcs.append(self.flat.grad_buf.data_ptr())
                    continue
                dst = self.staging[j].data_ptr()
                _native.call("brain_comm_copy_async", self.gpeers[j] + a * ge, dst, n * ge, st)
                srcs.append(dst - a * ge)  # the kernel adds the piece offset back
            order = [(r + jj) % W for jj in range(W)]
            grads = [0] * W
            for j, p in zip(order, srcs):
                grads[j] = p
            _native.call("brain_comm_ddp_step_ctas", _i64(grads), _i64([self.flat.param_buf.data_ptr()]), bf16, r, W,
                         a, n, *state, lr, b1, b2, eps, wd, bc1, bc2, gs, self.max_ctas, 1, st)
            pe = self.flat.param_buf.element_size()
            for jj in range(1, W):
                j = (r + jj) % W
                _native.call("brain_comm_copy_async", self.flat.param_buf.data_ptr() + a * pe,
                             self.ppeers[j] + a * pe, n * pe, st)

    def _reduce_piece(self, a: int, n: int, gs: float) -> None:
        """Guarded mode, on the side stream: this rank's piece of a bucket becomes the scaled sum over the
        ranks (in place in the local gradient buffer, which no peer reads there) and its squares and
        non-finite flag are added to the step's statistics."""
        from ..ops import optim_kernels as K
        W, r, ge = self.world, self.rank, self.gesz
        piece = self.flat.grad_buf[a:a + n]
        if W > 1:
            dcode = 0 if self.flat.grad_buf.dtype == torch.float32 else 1
            st = self.side.cuda_stream
            if self.mode == "sm":
                peers = self.gpeers
            else:
                grads = [0] * W
                for jj in range(W):
                    j = (r + jj) % W
                    if j == r:
                        grads[j] = self.flat.grad_buf.data_ptr()
                        continue
                    dst = self.staging[j].data_ptr()
                    _native.call("brain_comm_copy_async", self.gpeers[j] + a * ge, dst, n * ge, st)
                    grads[j] = dst - a * ge  # the kernel adds the piece offset back
                peers = _i64(grads)
            _native.call("brain_comm_reduce_pull", peers, a, r, W, piece.data_ptr(), n, dcode, float(gs), st)
            gs = 1.0
        K.grad_stats(piece, gs, self.opt.stats, accumulate=self.stats_started)
        self.stats_started = True

    def _guarded_update(self) -> None:
        """Guarded mode, after backward: global statistics, then AdamW on every piece (skipped alike on
        every rank when anything was non-finite) and the new weights pushed to the peers."""
        from ..ops import optim_kernels as K
        opt, W = self.opt, self.world
        if not self.stats_started:
            opt.stats.zero_()
        if W > 1:
            self.comm.all_reduce(opt.stats)
        fi, coef = K.step_guard(opt.stats, self.max_norm, opt.found_inf, opt.coef)
        lr, b1, b2, eps, wd, bc1, bc2, gs = self.args
        t = opt.step_count
        pe = self.flat.param_buf.element_size()
        st = torch.cuda.current_stream().cuda_stream
        for a, n, s in self.pieces:
            if n == 0:
                continue
            K.adamw_(self.master[s:s + n], self.m[s:s + n], self.v[s:s + n], self.flat.grad_buf[a:a + n], lr=lr,
                     beta1=b1, beta2=b2, eps=eps, weight_decay=wd, step=t, grad_scale=1.0 if W > 1 else gs,
                     p16=self.flat.param_buf[a:a + n], found_inf=fi, coef=coef)
            for jj in range(1, W):
                j = (self.rank + jj) % W
                _native.call("brain_comm_copy_async", self.flat.param_buf.data_ptr() + a * pe,
                             self.ppeers[j] + a * pe, n * pe, st)

    def finish(self) -> None:
        """After backward: the buckets not yet reduced, then every rank's update visible everywhere."""
        stray = [p for p in self.flat.params if p.grad is not None]
        if stray:
            # an op without a main_grad path left a .grad after its bucket may already have been reduced
            raise RuntimeError(f"{len(stray)} parameter(s) received .grad instead of main_grad; the overlapped "
                               "reduction needs every gradient written into the flat buffer (use overlap=False)")
        for i in range(len(self.buckets)):
            self._launch(i)
        torch.cuda.current_stream().wait_stream(self.side)
        if self.guarded:
            self._guarded_update()
        if self.world > 1:
            self.comm.barrier(51)
        self.args = None

    def close(self) -> None:
        for h in self.hooks:
            h.remove()
        self.hooks = []
