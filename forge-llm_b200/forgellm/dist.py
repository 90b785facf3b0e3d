"""Data parallelism for TrainableTransformer: one process per GPU, the batch
split by sequence, gradients averaged with NCCL over NVLink.

Sequences are independent under the block-diagonal causal mask
(src/L2/tensor.js:292-298), so the only exchange is the gradient all-reduce.
Each layer's gradients occupy one contiguous block of the model's flat
gradient buffer; that block's all-reduce (NCCL AVG) is launched as soon as the
tape replay has run the layer's last gradient-writing closure, so it overlaps
the backward of the layers below.  Every rank then takes the identical Adam
step on identical averaged gradients, keeping the replicas equal.

On GPUs the collectives go through libforgecu's C-ABI (`NcclComm`, the
fcu_comm_* / fcu_allreduce_grads entry points: a non-blocking NCCL
communicator with bounded waits and abort on deadline).  torch.distributed
only bootstraps it (the 128-byte NCCL id is broadcast from rank 0) and runs
the gloo collectives of the CPU tests.
"""
from __future__ import annotations

import ctypes as C

import torch
import torch.distributed as dist


class NcclComm:
    """This rank's NCCL communicator, created and driven through libforgecu's
    C-ABI (include/forgecu.h, "data-parallel exchange").  Every collective is
    enqueued after the work already queued on the context's stream and runs on
    the communicator's own stream; `join()` makes the context's stream wait
    for all of them.  `poll()` is the host-side check between steps: it
    raises ForgeCUError (status FCU_ERR_TIMEOUT or FCU_ERR_NCCL) and aborts
    the communicator if the collectives do not finish in time or a peer
    failed."""

    def __init__(self, group=None, timeout_s: float = 120.0, device: int | None = None):
        from . import autograd as AD
        from ._lib import FCU_COMM_ID_BYTES, call
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.timeout_s = float(timeout_s)
        uid = C.create_string_buffer(FCU_COMM_ID_BYTES)
        if self.rank == 0:
            call("fcu_comm_unique_id", uid)
        obj = [uid.raw if self.rank == 0 else None]
        src = dist.get_global_rank(group, 0) if group is not None else 0
        dist.broadcast_object_list(obj, src=src, group=group)
        uid = C.create_string_buffer(obj[0], FCU_COMM_ID_BYTES)
        dev = torch.cuda.current_device() if device is None else device
        h = C.c_void_p()
        call("fcu_comm_init", dev, uid, self.world, self.rank, self.timeout_s, C.byref(h))
        self.handle = h
        self._AD = AD

    def _ctx(self):
        return self._AD.ctx().handle

    def allreduce_avg(self, t: torch.Tensor) -> None:
        from ._lib import call
        call("fcu_allreduce_grads", self._ctx(), self.handle, t.data_ptr(), t.numel())

    def reduce_scatter_avg(self, t: torch.Tensor) -> None:
        from ._lib import call
        call("fcu_reduce_scatter_grads", self._ctx(), self.handle, t.data_ptr(), t.numel())

    def allgather(self, t: torch.Tensor) -> None:
        from ._lib import call
        call("fcu_allgather_params", self._ctx(), self.handle, t.data_ptr(), t.numel(), t.element_size())

    def allreduce_sum_f64(self, t: torch.Tensor) -> None:
        from ._lib import call
        call("fcu_allreduce_sum_f64", self._ctx(), self.handle, t.data_ptr(), t.numel())

    def join(self) -> None:
        from ._lib import call
        call("fcu_comm_join", self._ctx(), self.handle)

    def poll(self, timeout_s: float | None = None) -> None:
        from ._lib import call
        call("fcu_comm_poll", self.handle, self.timeout_s if timeout_s is None else float(timeout_s))

    PROFILE_KINDS = ("allreduce", "reduce_scatter", "allgather", "sum_f64", "join")

    def profile(self, max_records: int) -> None:
        """Time the next `max_records` collectives and joins (outside stream
        capture) with CUDA events; 0 stops."""
        from ._lib import call
        call("fcu_comm_profile", self.handle, int(max_records))

    def profile_read(self, max_records: int = 4096) -> list:
        """The recorded collectives: [{kind, bytes, ready, start, end}] with
        times in ms from the first record's ready time (ready: the context's
        stream reached the call; start / end on the communicator's stream; a
        join's end is when the context's stream could continue)."""
        from ._lib import call
        out = (C.c_double * (5 * max_records))()
        n = C.c_int(0)
        call("fcu_comm_profile_read", self.handle, out, max_records, C.byref(n))
        recs = []
        for i in range(n.value):
            k, b, r, s, e = out[5 * i:5 * i + 5]
            recs.append({"kind": self.PROFILE_KINDS[int(k)], "bytes": int(b), "ready": r, "start": s, "end": e})
        return recs

    def abort(self) -> None:
        from ._lib import call
        if self.handle is not None:
            call("fcu_comm_abort", self.handle)

    def close(self) -> None:
        from ._lib import lib
        if self.handle is not None:
            lib().fcu_comm_destroy(self.handle)
            self.handle = None


class DataParallel:
    """Overlapped gradient averaging for one TrainableTransformer replica.

    `model` needs `flat_grads` (flat gradient buffer), `layer_offsets`
    ([(start, end)] per layer) and honours `grad_ready_hook`.  NCCL reduces
    with AVG; backends without AVG (gloo, used by the CPU tests) reduce with
    SUM and divide after the wait."""

    def __init__(self, model, group=None, shard: bool = False, comm: NcclComm | None = None,
                 timeout_s: float = 120.0):
        self.model = model
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.native_avg = dist.get_backend(group) == "nccl"
        # GPU ranks exchange through the C-ABI communicator; gloo (the CPU
        # tests) through torch.distributed
        self.comm = comm
        if self.comm is None and self.native_avg and self.world > 1 and model.flat_grads.is_cuda:
            self.comm = NcclComm(group, timeout_s=timeout_s)
        # shard=True (ZeRO-1, with ShardedAdam): each bucket is reduce-
        # scattered, rank r receiving the average of slice r of the bucket
        self.shard = shard
        self.handles = []
        head_end = model.layer_offsets[0][0] if model.layer_offsets else model.flat_grads.numel()
        self.blocks = {"head": (0, head_end)}
        for l, (a, b) in enumerate(model.layer_offsets):
            self.blocks[l] = (a, b)
        self.launched = set()
        if shard:
            for key, (a, b) in self.blocks.items():
                if (b - a) % self.world:
                    raise ValueError(f"bucket {key} ({b - a} values) does not split over {self.world} ranks")
        model.grad_ready_hook = self._ready

    def slices(self):
        """[(start, end)] of the flat buffers that this rank owns: its slice
        of every bucket, in bucket order."""
        out = []
        for a, b in self.blocks.values():
            n = (b - a) // self.world
            out.append((a + self.rank * n, a + (self.rank + 1) * n))
        return out

    def _ready(self, key) -> None:
        if self.world == 1 or key in self.launched:
            return
        a, b = self.blocks[key]
        buf = self.model.flat_grads[a:b]
        if self.comm is not None:
            if self.shard:
                self.comm.reduce_scatter_avg(buf)   # rank r receives slice r, in place
            else:
                self.comm.allreduce_avg(buf)
            self.launched.add(key)
            return
        op = dist.ReduceOp.AVG if self.native_avg else dist.ReduceOp.SUM
        if self.shard and self.native_avg:
            n = (b - a) // self.world
            own = buf[self.rank * n:(self.rank + 1) * n]     # in place: slice r of the bucket
            self.handles.append((own, dist.reduce_scatter_tensor(own, buf, op=op, group=self.group,
                                                                 async_op=True)))
        else:
            self.handles.append((buf, dist.all_reduce(buf, op=op, group=self.group, async_op=True)))
        self.launched.add(key)

    def finish(self) -> None:
        """Launch any block not yet reduced, then make the current stream
        wait for every all-reduce of this step."""
        if self.world > 1:
            for key in self.blocks:
                if key not in self.launched:
                    self._ready(key)
            if self.comm is not None:
                self.comm.join()
            for buf, h in self.handles:
                h.wait()
                if not self.native_avg:
                    buf.div_(self.world)
        self.handles.clear()
        self.launched.clear()

    def check(self, timeout_s: float | None = None) -> None:
        """Between steps: wait (bounded) until this rank's collectives have
        finished; raises ForgeCUError and aborts the communicator on a
        deadline miss or a failed peer."""
        if self.comm is not None:
            self.comm.poll(timeout_s)

    def detach(self) -> None:
        self.model.grad_ready_hook = None

    def close(self) -> None:
        """Detach and destroy the communicator (release any CUDA graph that
        replays its collectives first)."""
        self.detach()
        if self.comm is not None:
            self.comm.close()
            self.comm = None


class ShardedAdam:
    """Adam (autograd.js:214-244) with its state and update sharded over the
    data-parallel ranks (ZeRO-1): rank r keeps m and v only for its slice of
    every gradient bucket (DataParallel(shard=True) reduce-scatters the
    gradients into exactly those slices), updates those parameters, and the
    buckets' parameters (and their bf16 copy) are all-gathered back.  The
    global gradient norm for clipping is the all-reduced (fp64) sum of every
    rank's sum of squares, so the update is the replicated Adam's up to the
    summation order of that norm.  Optimizer memory and Adam traffic per GPU
    are 1/world of the replicated step's; the collective volume is the same
    (a reduce-scatter plus an all-gather instead of an all-reduce).

    Same surface as Adam: step(), step_device() (graph-capturable), t, the
    hyper-parameters, m_flat / v_flat (this rank's state)."""

    def __init__(self, model, dp: DataParallel, lr=3e-4, b1=0.9, b2=0.999, eps=1e-8, wd=0.0, clip=1.0,
                 totalSteps=1000):
        from . import autograd as AD
        if not dp.shard:
            raise ValueError("ShardedAdam needs DataParallel(model, shard=True)")
        self.model, self.dp = model, dp
        self.lr, self.b1, self.b2, self.eps, self.wd, self.clip = lr, b1, b2, eps, wd, clip
        self.total = totalSteps
        self.t = 0
        pf, gf = model.flat_params, model.flat_grads
        self._flat = (pf, gf)
        self.p = model.paramList
        self.own = dp.slices()
        n_own = sum(b - a for a, b in self.own)
        self.m_flat = torch.zeros(n_own, dtype=pf.dtype, device=pf.device)
        self.v_flat = torch.zeros_like(self.m_flat)
        self._ss = torch.zeros(1, dtype=torch.float64, device=pf.device)
        self._info3 = torch.zeros(3, dtype=torch.float64, device=pf.device)
        self._t_dev = torch.zeros(1, dtype=torch.int32, device=pf.device)
        self._h_dev = torch.zeros(8, dtype=torch.float64, device=pf.device)   # fcu_adam_hyper
        self._AD = AD

    def _shadow(self):
        owner = self._AD._SHADOWS.get(self.model.flat_params.data_ptr())
        return getattr(owner, "flat_params_bf16", None) if owner is not None else None

    def _zero_fill_pending(self):
        for p in self.p:
            if p._gzero:
                p.grad  # noqa: B018  (property zero-fills)

    def _global_sumsq(self, h):
        from ._lib import call
        pf, gf = self._flat
        for i, (a, b) in enumerate(self.own):
            call("fcu_sumsq", h, gf.data_ptr() + 4 * a, b - a, self._ss.data_ptr(), 1 if i else 0)
        if self.dp.comm is not None:
            self.dp.comm.allreduce_sum_f64(self._ss)
            self.dp.comm.join()
        else:
            dist.all_reduce(self._ss, op=dist.ReduceOp.SUM, group=self.dp.group)

    def _gather(self, shadow):
        pf = self.model.flat_params
        comm = self.dp.comm
        if comm is not None:
            for a, b in self.dp.blocks.values():
                comm.allgather(pf[a:b])
                if shadow is not None:
                    comm.allgather(shadow[a:b])
            comm.join()
            return
        for a, b in self.dp.blocks.values():
            n = (b - a) // self.dp.world
            r = self.dp.rank
            dist.all_gather_into_tensor(pf[a:b], pf[a + r * n:a + (r + 1) * n], group=self.dp.group)
            if shadow is not None:
                dist.all_gather_into_tensor(shadow[a:b], shadow[a + r * n:a + (r + 1) * n],
                                            group=self.dp.group)

    def _update(self, h, hyper_host, shadow):
        from ._lib import call
        import ctypes as C
        pf, gf = self._flat
        off = 0
        for i, (a, b) in enumerate(self.own):
            n = b - a
            sp = shadow.data_ptr() + 2 * a if shadow is not None else None
            mp, vp = self.m_flat.data_ptr() + 4 * off, self.v_flat.data_ptr() + 4 * off
            info = self._info3.data_ptr() if i == 0 else None
            if hyper_host is None:
                call("fcu_adam_update_dev", h, pf.data_ptr() + 4 * a, gf.data_ptr() + 4 * a, mp, vp, n,
                     self._h_dev.data_ptr(), self._ss.data_ptr(), info, sp)
            elif sp is not None:
                call("fcu_adam_step_shadow", h, pf.data_ptr() + 4 * a, gf.data_ptr() + 4 * a, mp, vp, n,
                     C.byref(hyper_host), self._ss.data_ptr(), info, sp)
            else:
                call("fcu_adam_step_sumsq", h, pf.data_ptr() + 4 * a, gf.data_ptr() + 4 * a, mp, vp, n,
                     C.byref(hyper_host), self._ss.data_ptr(), info)
            off += n

    def hyper(self):
        import math
        from ._lib import AdamHyper
        lr = self.lr * 0.5 * (1 + math.cos(math.pi * min(self.t / self.total, 1)))
        return AdamHyper(lr, self.b1, self.b2, self.eps, self.wd, self.clip,
                         1 - math.pow(self.b1, self.t), 1 - math.pow(self.b2, self.t))

    def step(self):
        """One step with the schedule computed on the host; returns the device
        {gnorm, scale, .} of this step."""
        h = self._AD.ctx().handle
        self._zero_fill_pending()
        self.t += 1
        self._t_dev.fill_(self.t)
        self._global_sumsq(h)
        shadow = self._shadow()
        self._update(h, self.hyper(), shadow)
        self._gather(shadow)
        return self._info3

    def step_device(self) -> torch.Tensor:
        """The same with the step counter and schedule on the device
        (fcu_adam_sched_advance + fcu_adam_update_dev), capturable in a CUDA
        graph.  Returns the device {gnorm, scale, lr}."""
        from ._lib import AdamSched, call
        import ctypes as C
        h = self._AD.ctx().handle
        self._zero_fill_pending()
        sched = AdamSched(self.lr, self.b1, self.b2, self.eps, self.wd, self.clip, float(self.total))
        call("fcu_adam_sched_advance", h, C.byref(sched), self._t_dev.data_ptr(), self._h_dev.data_ptr())
        self._global_sumsq(h)
        shadow = self._shadow()
        self._update(h, None, shadow)
        self._gather(shadow)
        self.t += 1
        return self._info3


def shard_rows(batch: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """Rows [rank*B/world, (rank+1)*B/world) of a [B, T+1] batch."""
    B = batch.shape[0]
    if B % world:
        raise ValueError(f"batch of {B} sequences does not split over {world} ranks")
    per = B // world
    return batch[rank * per:(rank + 1) * per]
