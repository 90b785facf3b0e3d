"""A whole TrainableTransformer training step captured as one CUDA graph.

`CapturedStep(model, opt, B, T)` records, once, exactly what one iteration of
the reference loop does (`train.js:265-269`: resetTape, zeroGrad, lossBatch,
backward, Adam.step) on the fused bf16 path, including the data-parallel
all-reduces when a `DataParallel` is attached, and then replays it.  Every
kernel still runs every step; replay removes the host work between them
(several hundred launches and their Python bookkeeping), which at small
per-GPU batches costs more than the GPU work itself.

The captured step reads its batch from a static device buffer, so a call
copies the new batch in (from host or device memory) and replays.  Adam's
step counter and lr schedule live on the device (`Adam.step_device`), so the
replayed step follows the schedule.  Building the graph runs `warmup` real
steps (they size every buffer and workspace); the parameters, Adam moments
and step counters are restored afterwards, so the first call is step 1.
"""
from __future__ import annotations

import torch

from . import autograd as AD
from . import tensor as TS


class CapturedStep:
    def __init__(self, model, opt, B: int, T: int, dp=None, warmup: int = 2):
        if not model._use_fused():
            raise ValueError("CapturedStep needs the fused bf16 path (precision bf16, supported shapes)")
        if opt._flat is None:
            raise ValueError("CapturedStep needs an Adam over the model's flat parameters")
        self.model, self.opt, self.dp = model, opt, dp
        self.B, self.T = B, T
        dev = model.flat_params.device
        # warm up on ids spread like real batches (a constant batch would make
        # every token share one embedding row and time a degenerate backward)
        gen = torch.Generator(device=dev).manual_seed(0)
        self.batch = torch.randint(0, model.cfg.vocabSize, (B, T + 1), dtype=torch.int32,
                                   device=dev, generator=gen)
        saved = [t.clone() for t in (model.flat_params, opt.m_flat, opt.v_flat)]
        t0 = opt.t
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):      # size every buffer and workspace first
            for _ in range(warmup):
                self._body()
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        from ._lib import lib
        n0 = lib().fcu_launch_count()
        saved_timer, TS.GEMM_TIMER = TS.GEMM_TIMER, None   # no host events inside the graph
        try:
            with torch.cuda.graph(self.graph):
                self.loss, self.info = self._body()
        finally:
            TS.GEMM_TIMER = saved_timer
        self.launches_per_step = int(lib().fcu_launch_count() - n0)   # this library's kernels
        for dst, src in zip((model.flat_params, opt.m_flat, opt.v_flat), saved):
            dst.copy_(src)
        opt.t = t0
        opt._t_dev.fill_(t0)
        model._shadow_stale = True
        model.bf16_weights()               # the weight copy follows the restored params
        torch.cuda.synchronize()

    def _body(self):
        AD.resetTape()
        self.model.zeroGrad()
        loss = self.model.lossBatch(self.batch)
        AD.backward(loss)
        if self.dp is not None:
            self.dp.finish()
        info = self.opt.step_device()
        return loss.data, info

    def __call__(self, batch) -> torch.Tensor:
        """One training step on `batch` ([B, T+1] token ids, host or device);
        returns the device loss tensor (reading it synchronises)."""
        if batch is not None:
            self.batch.copy_(torch.as_tensor(batch), non_blocking=True)
        self.graph.replay()
        self.opt.t += 1
        return self.loss
