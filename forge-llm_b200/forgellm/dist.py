"""Data parallelism for TrainableTransformer: one process per GPU, the batch
split by sequence, gradients averaged with NCCL over NVLink.

Sequences are independent under the block-diagonal causal mask
(src/L2/tensor.js:292-298), so the only exchange is the gradient all-reduce.
Each layer's gradients occupy one contiguous block of the model's flat
gradient buffer; that block's all-reduce (NCCL AVG) is launched as soon as the
tape replay has run the layer's last gradient-writing closure, so it overlaps
the backward of the layers below.  Every rank then takes the identical Adam
step on identical averaged gradients, keeping the replicas equal.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


class DataParallel:
    """Overlapped gradient averaging for one TrainableTransformer replica.

    `model` needs `flat_grads` (flat gradient buffer), `layer_offsets`
    ([(start, end)] per layer) and honours `grad_ready_hook`.  NCCL reduces
    with AVG; backends without AVG (gloo, used by the CPU tests) reduce with
    SUM and divide after the wait."""

    def __init__(self, model, group=None):
        self.model = model
        self.group = group
        self.world = dist.get_world_size(group)
        self.native_avg = dist.get_backend(group) == "nccl"
        self.handles = []
        head_end = model.layer_offsets[0][0] if model.layer_offsets else model.flat_grads.numel()
        self.blocks = {"head": (0, head_end)}
        for l, (a, b) in enumerate(model.layer_offsets):
            self.blocks[l] = (a, b)
        self.launched = set()
        model.grad_ready_hook = self._ready

    def _ready(self, key) -> None:
        if self.world == 1 or key in self.launched:
            return
        a, b = self.blocks[key]
        buf = self.model.flat_grads[a:b]
        op = dist.ReduceOp.AVG if self.native_avg else dist.ReduceOp.SUM
        self.handles.append((buf, dist.all_reduce(buf, op=op, group=self.group, async_op=True)))
        self.launched.add(key)

    def finish(self) -> None:
        """Launch any block not yet reduced, then make the current stream
        wait for every all-reduce of this step."""
        if self.world > 1:
            for key in self.blocks:
                if key not in self.launched:
                    self._ready(key)
            for buf, h in self.handles:
                h.wait()
                if not self.native_avg:
                    buf.div_(self.world)
        self.handles.clear()
        self.launched.clear()

    def detach(self) -> None:
        self.model.grad_ready_hook = None


def shard_rows(batch: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """Rows [rank*B/world, (rank+1)*B/world) of a [B, T+1] batch."""
    B = batch.shape[0]
    if B % world:
        raise ValueError(f"batch of {B} sequences does not split over {world} ranks")
    per = B // world
    return batch[rank * per:(rank + 1) * per]
