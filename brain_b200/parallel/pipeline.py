"""Pipeline parallelism with a real 1F1B schedule (the reference's ``PipelineStage::step_1f1b`` returns
its input, crates/brain-distributed/src/pipeline.rs:8-26; ``ModelParallelStage`` is identity,
model_parallel.rs:8-26).

``PipelineStage`` owns a contiguous slice of layers. Activations and their gradients move between
neighbouring stages with NCCL point-to-point ``isend``/``irecv`` issued on a side stream, so
transfers overlap the next micro-batch's compute. The schedule is the standard one-forward-one-backward
order: ``world - rank - 1`` warm-up forwards, then alternating forward/backward, then cool-down
backwards, which bounds in-flight activations to ``world`` micro-batches.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def one_f_one_b_schedule(num_stages: int, stage: int, num_microbatches: int) -> list[tuple[str, int]]:
    """Ordered ("F", mb) / ("B", mb) actions of one stage."""
    warm = min(num_stages - stage - 1, num_microbatches)
    steady = num_microbatches - warm
    acts = [("F", i) for i in range(warm)]
    f, b = warm, 0
    for _ in range(steady):
        acts.append(("F", f))
        f += 1
        acts.append(("B", b))
        b += 1
    while b < num_microbatches:
        acts.append(("B", b))
        b += 1
    return acts


class PipelineStage:
    def __init__(self, module: torch.nn.Module, stage_id: int, num_stages: int, num_microbatches: int,
                 act_shape: tuple, dtype=torch.bfloat16, group=None, loss_fn=None):
        self.module, self.stage_id, self.num_stages = module, stage_id, num_stages
        self.num_microbatches = num_microbatches
        self.act_shape, self.dtype, self.group, self.loss_fn = act_shape, dtype, group, loss_fn
        self.device = next(module.parameters()).device
        self.comm_stream = torch.cuda.Stream(self.device) if self.device.type == "cuda" else None
        ranks = dist.get_process_group_ranks(group) if group is not None else list(range(dist.get_world_size()))
        self.prev = ranks[stage_id - 1] if stage_id > 0 else None
        self.next = ranks[stage_id + 1] if stage_id < num_stages - 1 else None

    @property
    def is_first(self):
        return self.stage_id == 0

    @property
    def is_last(self):
        return self.stage_id == self.num_stages - 1

    def _recv(self, src):
        t = torch.empty(self.act_shape, device=self.device, dtype=self.dtype)
        if self.comm_stream is not None:
            self.comm_stream.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(self.comm_stream):
                dist.irecv(t, src, group=self.group).wait()
            torch.cuda.current_stream().wait_stream(self.comm_stream)
        else:
            dist.recv(t, src, group=self.group)
        return t

    def _send(self, t, dst):
        """Non-blocking on every backend: two neighbouring stages may both be sending (an activation
        forward, a gradient backward) in the same 1F1B phase, and blocking sends would wait on each
        other. Returns (work, tensor); the tensor is kept alive until the work is waited on."""
        t = t.contiguous()
        if self.comm_stream is not None:
            self.comm_stream.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(self.comm_stream):
                work = dist.isend(t, dst, group=self.group)
            return work, t
        return dist.isend(t, dst, group=self.group), t

    def step_1f1b(self, microbatches=None, targets=None) -> float:
        """Run one optimizer-step's worth of micro-batches. Returns the mean loss on the last stage."""
        inputs, outputs, pending, losses = {}, {}, [], []
        for act, mb in one_f_one_b_schedule(self.num_stages, self.stage_id, self.num_microbatches):
            if act == "F":
                x = microbatches[mb] if self.is_first else self._recv(self.prev).requires_grad_(True)
                y = self.module(x)
                inputs[mb] = x
                if self.is_last:
                    loss = self.loss_fn(y, targets[mb]) / self.num_microbatches
                    outputs[mb] = loss
                    losses.append(float(loss.detach()) * self.num_microbatches)
                else:
                    outputs[mb] = y
                    w = self._send(y.detach(), self.next)
                    if w is not None:
                        pending.append(w)
            else:
                y = outputs.pop(mb)
                if self.is_last:
                    y.backward()
                else:
                    g = self._recv(self.next)
                    y.backward(g)
                x = inputs.pop(mb)
                if not self.is_first:
                    w = self._send(x.grad, self.prev)
                    if w is not None:
                        pending.append(w)
        for w, _ in pending:
            w.wait()
        if self.comm_stream is not None:
            torch.cuda.current_stream().wait_stream(self.comm_stream)
        return sum(losses) / len(losses) if losses else float("nan")


class ModelParallelStage(torch.nn.Module):
    """Place a slice of layers on a device (layer placement helper on top of pipeline stages)."""

    def __init__(self, layers, device):
        super().__init__()
        self.layers = torch.nn.ModuleList(layers).to(device)
        self.device = device

    def forward(self, x):
        x = x.to(self.device)
        for l in self.layers:
            x = l(x)
        return x


def split_layers(num_layers: int, num_stages: int) -> list[range]:
    """Contiguous, balanced layer ranges per stage."""
    base, extra = divmod(num_layers, num_stages)
    out, s = [], 0
    for i in range(num_stages):
        n = base + (1 if i < extra else 0)
        out.append(range(s, s + n))
        s += n
    return out
