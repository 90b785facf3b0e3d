"""Tensor-level fused operators with hand-written backward, mirroring
forge-llm's src/L2/tensor.js (same names, argument order and meaning).

Each function enqueues one libforgecu kernel for its forward and attaches a
closure that enqueues the backward kernels, accumulating into the inputs'
gradients exactly as the JS closures do (``X.grad ??= zeros; X.grad += ...``).
"""
from __future__ import annotations

import torch

from ._lib import call
from .autograd import Node, as_device, ctx, op, ptr


def _i32(ids) -> torch.Tensor:
    return as_device(ids, torch.int32)


# When set to a list, every matmulT contraction appends (flops, start, end)
# CUDA events recorded on the launching stream (bench.py's live roofline).
GEMM_TIMER = None


def _timed(flops: int, fn) -> None:
    if GEMM_TIMER is None:
        fn()
        return
    s = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    fn()
    e1.record(s)
    GEMM_TIMER.append((flops, e0, e1))


def matmulT(X: Node, W: Node, M: int, K: int, N: int) -> Node:
    """Y[M,N] = X[M,K] . W[N,K]^T; backward dX = dY.W, dW = dY^T.X
    (tensor.js:34-53)."""
    c = ctx()
    out = torch.empty(M * N, dtype=torch.float32, device=X.data.device)
    _timed(2 * M * N * K, lambda: call("fcu_matmulT_fwd", c.handle, ptr(X.data), ptr(W.data),
                                       ptr(out), M, K, N))

    def bwd(g):
        cc = ctx()
        gX, ax = X._gout()
        gW, aw = W._gout()
        _timed(4 * M * N * K, lambda: call("fcu_matmulT_bwd", cc.handle, ptr(g), ptr(X.data),
                                           ptr(W.data), ptr(gX), ax, ptr(gW), aw, M, K, N))

    return op(out, bwd)


def embedLookup(W: Node, ids, V: int, D: int) -> Node:
    """X[T,D] = W[ids[t]]; backward scatter-adds into W (tensor.js:85-99)."""
    c = ctx()
    idt = _i32(ids)
    T = idt.numel()
    out = torch.empty(T * D, dtype=torch.float32, device=W.data.device)
    call("fcu_embed_fwd", c.handle, ptr(W.data), ptr(idt), T, V, D, ptr(out))

    def bwd(g):
        cc = ctx()
        gW, aw = W._gout()
        if not aw:
            gW.zero_()
        call("fcu_embed_bwd", cc.handle, ptr(g), ptr(idt), T, V, D, ptr(gW))

    return op(out, bwd)


def rmsNorm(X: Node, w: Node, T: int, D: int, eps: float = 1e-6) -> Node:
    """Y = X / rms(X) * w, eps inside the mean square (tensor.js:103-128)."""
    c = ctx()
    out = torch.empty(T * D, dtype=torch.float32, device=X.data.device)
    inv = torch.empty(T, dtype=torch.float32, device=X.data.device)
    call("fcu_rmsnorm_fwd", c.handle, ptr(X.data), ptr(w.data), T, D, float(eps), ptr(out), ptr(inv))

    def bwd(g):
        cc = ctx()
        gX, ax = X._gout()
        gw, aw = w._gout()
        call("fcu_rmsnorm_bwd", cc.handle, ptr(g), ptr(X.data), ptr(w.data), ptr(inv), T, D,
             ptr(gX), ax, ptr(gw), aw)

    return op(out, bwd)


def ropeRows(X: Node, T: int, nHead: int, dHead: int, pos0: int, theta: float = 10000,
             posStride: int = 0) -> Node:
    """Interleaved-pair RoPE at position pos0 + (t % posStride or t); backward
    is the transposed rotation (tensor.js:133-166)."""
    c = ctx()
    out = torch.empty(T * nHead * dHead, dtype=torch.float32, device=X.data.device)
    call("fcu_rope_fwd", c.handle, ptr(X.data), T, nHead, dHead, pos0, float(theta), posStride,
         ptr(out))

    def bwd(g):
        cc = ctx()
        gX, ax = X._gout()
        call("fcu_rope_bwd", cc.handle, ptr(g), T, nHead, dHead, pos0, float(theta), posStride,
             ptr(gX), ax)

    return op(out, bwd)


def sliceCols(X: Node, M: int, K: int, off: int, ln: int) -> Node:
    """Columns [off, off+len) of X[M,K]; backward scatters back (tensor.js:170-183)."""
    c = ctx()
    out = torch.empty(M * ln, dtype=torch.float32, device=X.data.device)
    call("fcu_slicecols_fwd", c.handle, ptr(X.data), M, K, off, ln, ptr(out))

    def bwd(g):
        cc = ctx()
        gX, ax = X._gout()
        if not ax and ln != K:
            gX.zero_()   # the other columns of a fresh gradient are zero
            ax = 1
        call("fcu_slicecols_bwd", cc.handle, ptr(g), M, K, off, ln, ptr(gX), ax)

    return op(out, bwd)


def _attn(Q: Node, K: Node, V: Node, B: int, T: int, nH: int, nKV: int, dHead: int) -> Node:
    if nH % nKV != 0:
        raise ValueError(f"GQA requires nH ({nH}) divisible by nKV ({nKV})")
    c = ctx()
    dev = Q.data.device
    out = torch.empty(B * T * nH * dHead, dtype=torch.float32, device=dev)
    lse = torch.empty(B * nH * T, dtype=torch.float32, device=dev)
    call("fcu_attn_fwd", c.handle, ptr(Q.data), ptr(K.data), ptr(V.data), B, T, nH, nKV, dHead,
         ptr(out), ptr(lse))
    node = None

    def bwd(g):
        cc = ctx()
        outs = [Q._gout(), K._gout(), V._gout()]
        acc = 1 if any(a for _, a in outs) else 0
        if acc:
            for t, a in outs:
                if not a:
                    t.zero_()
        call("fcu_attn_bwd", cc.handle, ptr(g), ptr(Q.data), ptr(K.data), ptr(V.data),
             ptr(node.data), ptr(lse), B, T, nH, nKV, dHead, ptr(outs[0][0]), ptr(outs[1][0]),
             ptr(outs[2][0]), acc)

    node = op(out, bwd)
    return node


def causalAttn(Q: Node, K: Node, V: Node, T: int, nH: int, nKV: int, dHead: int) -> Node:
    """Causal self-attention with GQA over one sequence (tensor.js:191-268)."""
    return _attn(Q, K, V, 1, T, nH, nKV, dHead)


def causalAttnBatch(Q: Node, K: Node, V: Node, B: int, T: int, nH: int, nKV: int,
                    dHead: int) -> Node:
    """Block-diagonal causal attention over B sequences (tensor.js:299-376)."""
    return _attn(Q, K, V, B, T, nH, nKV, dHead)


def swigluRows(G: Node, U: Node, T: int, H: int) -> Node:
    """O = silu(G) * U (tensor.js:272-290)."""
    c = ctx()
    n = T * H
    out = torch.empty(n, dtype=torch.float32, device=G.data.device)
    call("fcu_swiglu_fwd", c.handle, ptr(G.data), ptr(U.data), n, ptr(out))

    def bwd(g):
        cc = ctx()
        gG, aG = G._gout()
        gU, aU = U._gout()
        if aG != aU:
            (gU if aG else gG).zero_()
        call("fcu_swiglu_bwd", cc.handle, ptr(g), ptr(G.data), ptr(U.data), n, ptr(gG), ptr(gU),
             1 if (aG or aU) else 0)

    return op(out, bwd)


def weightedSum(Y: Node, t) -> Node:
    """out[0] = sum_i Y[i] t[i] (tensor.js:380-389)."""
    c = ctx()
    tt = as_device(t)
    out = torch.empty(1, dtype=torch.float32, device=Y.data.device)
    call("fcu_wsum_fwd", c.handle, ptr(Y.data), ptr(tt), Y.n, ptr(out))

    def bwd(g):
        cc = ctx()
        gY, a = Y._gout()
        call("fcu_axpy_dev", cc.handle, ptr(g), ptr(tt), tt.numel(), ptr(gY), a)

    return op(out, bwd)


def crossEntropyMean(logits: Node, targets, T: int, V: int) -> Node:
    """L = -(1/T) sum_t log softmax(logits_t)[targets_t]; backward
    dLogits += g * (P - OneHot)/T (tensor.js:393-417).  The forward kernel
    writes (P - OneHot)/T in the same pass that computes the loss."""
    c = ctx()
    tg = _i32(targets)
    dev = logits.data.device
    loss = torch.empty(1, dtype=torch.float32, device=dev)
    dunit = torch.empty(T * V, dtype=torch.float32, device=dev)
    call("fcu_ce_fwd", c.handle, ptr(logits.data), ptr(tg), T, V, ptr(loss), ptr(dunit))

    def bwd(g):
        # The usual case: this loss is the one backward() seeded with the
        # constant 1 and the logits have no gradient storage yet, so the
        # stored (P - OneHot)/T already is dLogits: adopt it, no second pass.
        if out._seeded_one and logits._grad is None and logits._gslot is None:
            logits._grad = dunit
            logits._gzero = False
            return
        cc = ctx()
        gL, a = logits._gout()
        call("fcu_axpy_dev", cc.handle, ptr(g), ptr(dunit), T * V, ptr(gL), a)

    out = op(loss, bwd)
    return out


def addTensors(a: Node, b: Node, n: int) -> Node:
    """Residual add, src/L6/train.js:230-238."""
    c = ctx()
    out = torch.empty(n, dtype=torch.float32, device=a.data.device)
    call("fcu_add_fwd", c.handle, ptr(a.data), ptr(b.data), n, ptr(out))

    def bwd(g):
        cc = ctx()
        ga, aa = a._gout()
        gb, ab = b._gout()
        call("fcu_add_bwd", cc.handle, ptr(g), n, ptr(ga), aa, ptr(gb), ab)

    return op(out, bwd)
