"""Reverse-mode tape and Adam, mirroring forge-llm's src/L2/autograd.js.

Same names and semantics as the JS module: a global tape of ``Node`` objects
(``resetTape``/``noGrad``/``tape``), ``op(out, bwd)`` attaches a closure,
``backward(loss)`` seeds ``loss.grad = 1`` and replays the closures in reverse
creation order, every gradient ACCUMULATES (``grad += ...``), ``zeroGrad``
zeroes an existing gradient, and ``Adam.step()`` does global-norm clipping,
cosine lr and bias-corrected Adam (autograd.js:214-244).

Differences that follow from the data living on the GPU:
  * ``Node.data`` / ``Node.grad`` are flat float32 CUDA tensors (the JS
    Float32Array); host code may still read and write elements.
  * A gradient that the JS would allocate as zeros and then ``+=`` into is
    written directly (the kernels' ``accumulate = 0``); ``zeroGrad`` marks a
    gradient as zero and the zeros are only materialised if read.
  * After ``backward`` has run an op's closure, the op output's gradient is
    released (leaf and param gradients are kept).  Set
    ``autograd.RETAIN_OP_GRADS = True`` to keep all of them, as the JS does.
"""
from __future__ import annotations

import math

import numpy as np
import torch

from . import _lib
from ._lib import AdamHyper, Context, call

RETAIN_OP_GRADS = False

# bf16 copies of flat parameter buffers that Adam keeps current:
# flat fp32 data_ptr -> owner with `.flat_params_bf16` and `._shadow_stale`.
_SHADOWS: dict = {}


def register_shadow(flat_params: torch.Tensor, owner) -> None:
    _SHADOWS[flat_params.data_ptr()] = owner


# ----------------------------------------------------------------- device helpers
def ctx() -> Context:
    """The fcu_ctx of the current device, bound to torch's current stream."""
    c = Context.get()
    c.bind_stream(torch.cuda.current_stream().cuda_stream)
    return c


def device() -> torch.device:
    if not torch.cuda.is_available():
        raise _lib.ForgeCUError("forgecu needs a CUDA device; none is available")
    return torch.device("cuda", torch.cuda.current_device())


def as_device(data, dtype=torch.float32) -> torch.Tensor:
    """Flat, contiguous tensor of `dtype` on the current CUDA device."""
    if isinstance(data, torch.Tensor):
        t = data
    elif isinstance(data, np.ndarray):
        t = torch.from_numpy(np.ascontiguousarray(data))
    else:
        t = torch.as_tensor(data)
    t = t.to(device=device(), dtype=dtype, non_blocking=True)
    return t.reshape(-1).contiguous()


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


# ----------------------------------------------------------------- tape
class _Tape:
    __slots__ = ("nodes", "enabled", "after")

    def __init__(self):
        self.nodes = []
        self.enabled = True
        self.after = {}   # id(node) -> callback run right after that node's closure


_tape = _Tape()


def tape() -> _Tape:
    return _tape


def resetTape() -> None:
    global _tape
    _tape = _Tape()


def noGrad(fn):
    e = _tape.enabled
    _tape.enabled = False
    try:
        return fn()
    finally:
        _tape.enabled = e


class Node:
    """A tensor on the tape (autograd.js:25-34)."""

    __slots__ = ("data", "_grad", "_gzero", "_gslot", "_b", "isParam", "_seeded_one",
                 "__weakref__")

    def __init__(self, data, requiresGrad: bool = True):
        self.data = data if (isinstance(data, torch.Tensor) and data.is_cuda
                             and data.dtype == torch.float32) else as_device(data)
        self._grad = None
        self._gzero = False
        self._gslot = None   # preallocated storage for the gradient (flat buffers)
        self._b = None
        self.isParam = False
        self._seeded_one = False
        if requiresGrad and _tape.enabled:
            _tape.nodes.append(self)

    @property
    def n(self) -> int:
        return self.data.numel()

    @property
    def grad(self):
        if self._grad is not None and self._gzero:
            self._grad.zero_()
            self._gzero = False
        return self._grad

    @grad.setter
    def grad(self, v):
        self._grad = None if v is None else as_device(v)
        self._gzero = False

    def zeroGrad(self) -> None:
        if self._grad is not None:
            self._gzero = True

    def _gout(self):
        """(gradient buffer, accumulate flag) for a closure about to `+=`."""
        if self._grad is None:
            if self._gslot is not None:
                self._grad = self._gslot
            else:
                self._grad = torch.empty_like(self.data)
            self._gzero = False
            return self._grad, 0
        if self._gzero:
            self._gzero = False
            return self._grad, 0
        return self._grad, 1


def leaf(data) -> Node:
    return Node(data)


def param(data) -> Node:
    n = Node(data)
    n.isParam = True
    return n


def op(out, bwd) -> Node:
    n = Node(out)
    n._b = bwd
    return n


def backward(loss: Node) -> None:
    """autograd.js:126-133."""
    loss.grad = torch.ones(loss.n, dtype=torch.float32, device=loss.data.device)
    loss._seeded_one = True           # the loss gradient is the constant 1
    nodes = _tape.nodes
    after = _tape.after
    for i in range(len(nodes) - 1, -1, -1):
        nd = nodes[i]
        if nd._b is not None and nd._grad is not None:
            nd._b(nd.grad)
            if not RETAIN_OP_GRADS and nd is not loss:
                nd._grad = None
                nd._b = None
            if after:
                cb = after.pop(id(nd), None)
                if cb is not None:
                    cb()


def after_backward_of(node: Node, callback) -> None:
    """Run `callback()` right after `node`'s closure during `backward` (the
    point where the gradients that closure writes are complete)."""
    _tape.after[id(node)] = callback


# ----------------------------------------------------------------- I-30 vector ops
def linear(W: Node, x: Node, N: int, K: int) -> Node:
    """out[N] = W[N,K] . x[K] (autograd.js:47-58): matmulT with one row."""
    from .tensor import matmulT
    return matmulT(x, W, 1, K, N)


def softmaxCE(logits: Node, target: int) -> Node:
    """-log softmax(logits)[target], grad p - onehot (autograd.js:110-124):
    the one-row crossEntropyMean."""
    from .tensor import crossEntropyMean
    return crossEntropyMean(logits, [int(target)], 1, logits.n)


def gradCheck(lossFn, params: dict, eps: float = 1e-3) -> dict:
    """Central-difference check of every `max(1, n//24)`-th element
    (autograd.js:192-210).  Host loop over device data; test utility."""
    worst, worst_name = 0.0, ""
    base = lossFn()
    backward(base)
    for name, p in params.items():
        n = p.n
        grad = p.grad.detach().cpu().numpy() if p.grad is not None else None
        for i in range(0, n, max(1, n // 24)):
            orig = float(p.data[i].item())
            p.data[i] = float(np.float32(orig + eps))
            lp = float(lossFn().data[0].item())
            p.data[i] = float(np.float32(orig - eps))
            lm = float(lossFn().data[0].item())
            p.data[i] = float(np.float32(orig))
            num = (lp - lm) / (2 * eps)
            ana = float(grad[i]) if grad is not None else 0.0
            rel = abs(num - ana) / max(1.0, abs(num), abs(ana))
            if rel > worst:
                worst, worst_name = rel, f"{name}[{i}]"
    return {"maxRelErr": worst, "at": worst_name, "loss": float(base.data[0].item())}


# ----------------------------------------------------------------- Adam
class AdamInfo(dict):
    """{lr, gnorm, scale} of one step; gnorm/scale are read from the device on
    first access (so a training loop that ignores them never synchronises)."""

    def __init__(self, lr: float, info_dev: torch.Tensor):
        super().__init__(lr=lr)
        self._dev = info_dev

    def _fetch(self):
        if "gnorm" not in self:
            v = self._dev.cpu().tolist()
            dict.__setitem__(self, "gnorm", v[0])
            dict.__setitem__(self, "scale", v[1])

    def __getitem__(self, k):
        if k in ("gnorm", "scale"):
            self._fetch()
        return dict.__getitem__(self, k)

    def __getattr__(self, k):
        try:
            return self[k]
        except KeyError as e:
            raise AttributeError(k) from e


class Adam:
    """Adam + global-norm clipping + cosine lr (autograd.js:214-244)."""

    def __init__(self, params, lr=3e-4, b1=0.9, b2=0.999, eps=1e-8, wd=0.0, clip=1.0,
                 totalSteps=1000, **kw):
        opts = dict(lr=lr, b1=b1, b2=b2, eps=eps, wd=wd, clip=clip, totalSteps=totalSteps)
        opts.update(kw)
        self.p = list(params)
        self.lr, self.b1, self.b2 = opts["lr"], opts["b1"], opts["b2"]
        self.eps, self.wd, self.clip = opts["eps"], opts["wd"], opts["clip"]
        self.total = opts["totalSteps"]
        self.t = 0
        self._flat = _flat_group(self.p)
        if self._flat is not None:
            pf, _ = self._flat
            self.m_flat = torch.zeros_like(pf)
            self.v_flat = torch.zeros_like(pf)
            self.m, self.v = _views_like(self.p, self.m_flat), _views_like(self.p, self.v_flat)
        else:
            self.m = [torch.zeros_like(p.data) for p in self.p]
            self.v = [torch.zeros_like(p.data) for p in self.p]
        self._sumsq = torch.zeros(1, dtype=torch.float64, device=device())
        self._info = torch.zeros(2, dtype=torch.float64, device=device())

    def hyper(self) -> AdamHyper:
        """This step's scheduled lr and bias corrections, in double as the JS."""
        lr = self.lr * 0.5 * (1 + math.cos(math.pi * min(self.t / self.total, 1)))
        return AdamHyper(lr, self.b1, self.b2, self.eps, self.wd, self.clip,
                         1 - math.pow(self.b1, self.t), 1 - math.pow(self.b2, self.t))

    def step_device(self) -> torch.Tensor:
        """Adam.step with the step counter and the lr schedule on the device
        (fcu_adam_step_sched): nothing in it depends on host values that
        change between steps, so it can be captured in a CUDA graph and
        replayed.  Needs the flat parameter layout (TrainableTransformer).
        Returns the device tensor {gnorm, scale, lr} of this step."""
        if self._flat is None:
            raise ValueError("step_device needs parameters that share one flat buffer")
        from ._lib import AdamSched
        pf, gf = self._flat
        if getattr(self, "_t_dev", None) is None:
            self._t_dev = torch.full((1,), self.t, dtype=torch.int32, device=pf.device)
            self._info3 = torch.zeros(3, dtype=torch.float64, device=pf.device)
            self._sched = AdamSched(self.lr, self.b1, self.b2, self.eps, self.wd, self.clip,
                                    float(self.total))
        for p in self.p:
            if p._gzero:
                p.grad  # noqa: B018  (property zero-fills)
        owner = _SHADOWS.get(pf.data_ptr())
        shadow = (owner.flat_params_bf16 if owner is not None
                  and getattr(owner, "flat_params_bf16", None) is not None else None)
        call("fcu_adam_step_sched", ctx().handle, ptr(pf), ptr(gf), ptr(self.m_flat),
             ptr(self.v_flat), pf.numel(), self._sched, ptr(self._t_dev), ptr(self._info3),
             ptr(shadow))
        self.t += 1
        return self._info3

    def step(self, sumsq_dev: torch.Tensor | None = None) -> AdamInfo:
        """One step.  `sumsq_dev` (device double [1]) overrides the local sum
        of squared gradients, e.g. after a data-parallel all-reduce."""
        self.t += 1
        if getattr(self, "_t_dev", None) is not None:
            self._t_dev.fill_(self.t)          # keep the device counter in step
        h = self.hyper()
        c = ctx()
        info = self._info
        if self._flat is not None and all(p._grad is not None for p in self.p):
            pf, gf = self._flat
            for p in self.p:          # materialise zeroed-but-unwritten grads
                if p._gzero:
                    p.grad  # noqa: B018  (property zero-fills)
            owner = _SHADOWS.get(pf.data_ptr())
            if (owner is not None and getattr(owner, "flat_params_bf16", None) is not None
                    and owner.flat_params_bf16.numel() == pf.numel()):
                call("fcu_adam_step_shadow", c.handle, ptr(pf), ptr(gf), ptr(self.m_flat),
                     ptr(self.v_flat), pf.numel(), h, ptr(sumsq_dev), ptr(info),
                     ptr(owner.flat_params_bf16))
                return AdamInfo(h.lr, info.clone())
            if sumsq_dev is None:
                call("fcu_adam_step", c.handle, ptr(pf), ptr(gf), ptr(self.m_flat),
                     ptr(self.v_flat), pf.numel(), h, ptr(info))
            else:
                call("fcu_adam_step_sumsq", c.handle, ptr(pf), ptr(gf), ptr(self.m_flat),
                     ptr(self.v_flat), pf.numel(), h, ptr(sumsq_dev), ptr(info))
            return AdamInfo(h.lr, info.clone())
        ss = sumsq_dev
        if ss is None:
            ss = self._sumsq
            first = True
            for p in self.p:
                g = p.grad
                if g is None:
                    continue
                call("fcu_sumsq", c.handle, ptr(g), g.numel(), ptr(ss), 0 if first else 1)
                first = False
            if first:
                ss.zero_()
        for j, p in enumerate(self.p):
            g = p.grad
            if g is None:
                continue
            call("fcu_adam_step_sumsq", c.handle, ptr(p.data), ptr(g), ptr(self.m[j]),
                 ptr(self.v[j]), p.n, h, ptr(ss), ptr(info))
        for owner in _SHADOWS.values():   # a bf16 weight copy may now be out of date
            owner._shadow_stale = True
        return AdamInfo(h.lr, info.clone())


def _flat_group(params):
    """(flat params, flat grads) when every param is a consecutive view of one
    flat buffer with matching gradient slots; else None."""
    if not params or any(p._gslot is None for p in params):
        return None
    base = params[0].data
    off = 0
    for p in params:
        if p.data.untyped_storage().data_ptr() != base.untyped_storage().data_ptr():
            return None
        if p.data.storage_offset() != base.storage_offset() + off:
            return None
        if p._gslot.storage_offset() - params[0]._gslot.storage_offset() != off:
            return None
        off += p.n
    st = base.storage_offset()
    flat_p = base.new_empty(0).set_(base.untyped_storage(), st, (off,), (1,))
    g0 = params[0]._gslot
    flat_g = g0.new_empty(0).set_(g0.untyped_storage(), g0.storage_offset(), (off,), (1,))
    return flat_p, flat_g


def _views_like(params, flat):
    out, off = [], 0
    for p in params:
        out.append(flat[off:off + p.n])
        off += p.n
    return out
