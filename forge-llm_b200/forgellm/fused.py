"""The bf16 fused training step of TrainableTransformer.

Same math as the op-by-op tape of `TrainableTransformer._forward` +
`crossEntropyMean` (src/L6/train.js:120-185, src/L2/tensor.js), same
parameter-gradient accumulation (`grad += ...`, per the parameter Nodes'
flags), but every contraction is a tcgen05 GEMM on bf16 operands that the
previous kernel wrote directly, and the JS's separate glue ops are folded
into neighbours:

* RoPE on q and k happens in the qkv GEMM's epilogue, and its backward in
  the attention backward's dQ/dK stores; q, k, v are never sliced apart
  (attention reads them by column offset from one [N, qkvOut] buffer);
* the residual adds (train.js:145,153) happen in the output-projection GEMM
  epilogues; in the backward the residual gradient is updated in place by
  the fused RMSNorm backward, which also emits its bf16 copy;
* gate and up are one GEMM against the contiguous [ffn_gate; ffn_up] block of
  the flat parameters (paramList order puts them back to back); SwiGLU and
  its backward run as separate HBM-bound kernels (a GEMM-epilogue variant of
  both exists, bit-identical, behind `fuse_swiglu`, and is slower on B200);
* cross-entropy writes (P - onehot)/T directly in bf16 for the LM-head
  backward.

Activations for the backward are kept per layer in buffers allocated once per
(B, T) shape.  Parameters stay fp32 (master) in the model's flat buffer; a bf16
copy of them (the GEMMs' weight operand) is kept current by Adam.
"""
from __future__ import annotations

import ctypes as C
import os

import torch

from . import autograd as AD
from ._lib import (GEMM_DW, GEMM_DX, GEMM_FWD, OUT_BF16, OUT_BF16_ROPE, OUT_BF16_SWIGLU,
                   OUT_BF16_SWIGLU_BWD, OUT_F32, OUT_F32_RESIDUAL, GemmOut, call)
from .tensor import _timed

BF16 = torch.bfloat16
F32 = torch.float32


def fused_supported(cfg) -> bool:
    """Shapes the fused kernels take: 16-byte TMA rows everywhere and a
    tensor-core attention head size."""
    qD, kvD = cfg.nHeads * cfg.dHead, cfg.nKvHeads * cfg.dHead
    return (cfg.dim % 8 == 0 and cfg.hidden % 8 == 0 and cfg.vocabSize % 8 == 0
            and cfg.dHead in (16, 32, 64, 128) and (qD + kvD) % 32 == 0
            and cfg.qkvOut % 8 == 0 and qD % 8 == 0 and cfg.dim <= 2048
            and cfg.dim == qD)


class _Layer:
    __slots__ = ("x", "inv1", "xn", "qkv", "o", "lse", "x1", "inv2", "xn2", "gu", "act")


class FusedStep:
    def __init__(self, model, B: int, T: int):
        self.m = model
        c = model.cfg
        self.B, self.T, self.N = B, T, B * T
        dev = model.flat_params.device
        N, D, H, V = self.N, c.dim, c.hidden, c.vocabSize
        qD = c.nHeads * c.dHead
        e = lambda *s, dt=F32: torch.empty(*s, dtype=dt, device=dev)  # noqa: E731
        self.layers = []
        for _ in range(c.nLayers):
            L = _Layer()
            L.x = e(N * D)
            L.inv1 = e(N)
            L.xn = e(N * D, dt=BF16)
            L.qkv = e(N * c.qkvOut, dt=BF16)
            L.o = e(N * qD, dt=BF16)
            L.lse = e(B * c.nHeads * T)
            L.x1 = e(N * D)
            L.inv2 = e(N)
            L.xn2 = e(N * D, dt=BF16)
            L.gu = e(N * 2 * H, dt=BF16)
            L.act = e(N * H, dt=BF16)
            self.layers.append(L)
        self.br = e(N * D)          # branch output (wo / down GEMM) before its residual add
        self.xL = e(N * D)
        self.invf = e(N)
        self.xf = e(N * D, dt=BF16)
        self.logits = e(N * V)
        self.dlogits = e(N * V, dt=BF16)
        self.loss = e(1)
        # backward scratch, reused by every layer
        self.gx = e(N * D)
        self.gx_b = e(N * D, dt=BF16)
        self.dxn = e(N * D)
        self.dact = e(N * H, dt=BF16)
        self.dgu = e(N * 2 * H, dt=BF16)
        self.dO = e(N * qD, dt=BF16)
        self.dqkv = e(N * c.qkvOut, dt=BF16)
        self.ids = None
        # SwiGLU in the gate|up and down-gradient GEMM epilogues: the same
        # bits as the standalone kernels, but off by default -- on B200 the
        # GEMM epilogue's stores already limit those short-K products, and
        # the extra g/u/act traffic there (measured at the config-5 shapes:
        # 644 us vs 360 + 150 us forward, 842 us vs 207 + 210 us backward;
        # the whole batch-64 step 66.7 ms fused vs 61.9 ms with CTA-pair
        # tiles) costs more than the separate HBM passes it saves.
        # FORGECU_FUSE_SWIGLU=1 turns it on.
        self.fuse_swiglu = os.environ.get("FORGECU_FUSE_SWIGLU") == "1"
        self.can_fuse_swiglu = H % 128 == 0

    # ------------------------------------------------------------ helpers
    def _gemm(self, h, op, A, B, M, N, K, mode, out, accumulate=0, residual=None, rope=False,
              out2=None, aux=None):
        c = self.m.cfg
        o = GemmOut(mode, out.data_ptr(), accumulate,
                    residual.data_ptr() if residual is not None else None,
                    self.T if rope else 0, (c.nHeads + c.nKvHeads) * c.dHead if rope else 0,
                    c.dHead if rope else 0, float(c.ropeTheta) if rope else 0.0,
                    out2.data_ptr() if out2 is not None else None,
                    aux.data_ptr() if aux is not None else None)
        _timed(2 * M * N * K,
               lambda: call("fcu_gemm_bf16", h, op, A.data_ptr(), B.data_ptr(), M, N, K, C.byref(o)))

    # ------------------------------------------------------------ forward
    def forward(self, ids: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
        """Loss (device [1]) of one block-diagonal batch; ids/targets int32 [N]."""
        m, c = self.m, self.m.cfg
        h = AD.ctx().handle
        N, D, H, V, T, B = self.N, c.dim, c.hidden, c.vocabSize, self.T, self.B
        qD = c.nHeads * c.dHead
        W = m.bf16_weights()
        P = m.params
        self.ids = ids
        call("fcu_embed_fwd", h, P["tok_emb"].data.data_ptr(), ids.data_ptr(), N, V, D,
             self.layers[0].x.data_ptr() if c.nLayers else self.xL.data_ptr())
        eps = float(c.normEps)
        if c.nLayers:
            L0 = self.layers[0]
            call("fcu_rmsnorm_fwd_bf16", h, L0.x.data_ptr(), P["layers"][0]["ln1"].data.data_ptr(), N, D,
                 eps, L0.xn.data_ptr(), L0.inv1.data_ptr())
        else:
            call("fcu_rmsnorm_fwd_bf16", h, self.xL.data_ptr(), P["ln_f"].data.data_ptr(), N, D, eps,
                 self.xf.data_ptr(), self.invf.data_ptr())
        for l, L in enumerate(self.layers):
            Lp, Lw = P["layers"][l], W["layers"][l]
            self._gemm(h, GEMM_FWD, L.xn, Lw["wqkv"], N, c.qkvOut, D, OUT_BF16_ROPE, L.qkv, rope=True)
            call("fcu_attn_fwd_bf16", h, L.qkv.data_ptr(), c.qkvOut, B, T, c.nHeads, c.nKvHeads,
                 c.dHead, L.o.data_ptr(), L.lse.data_ptr())
            # x1 = x + o.wo^T, added inside the ln2 normalisation
            self._gemm(h, GEMM_FWD, L.o, Lw["wo"], N, D, qD, OUT_F32, self.br)
            call("fcu_rmsnorm_fwd_bf16_add", h, L.x.data_ptr(), self.br.data_ptr(),
                 Lp["ln2"].data.data_ptr(), N, D, eps, L.x1.data_ptr(), L.xn2.data_ptr(),
                 L.inv2.data_ptr())
            if self.fuse_swiglu and self.can_fuse_swiglu:
                self._gemm(h, GEMM_FWD, L.xn2, Lw["ffn_gu"], N, 2 * H, D, OUT_BF16_SWIGLU, L.gu,
                           out2=L.act)
            else:
                self._gemm(h, GEMM_FWD, L.xn2, Lw["ffn_gu"], N, 2 * H, D, OUT_BF16, L.gu)
                call("fcu_swiglu_fwd_bf16", h, L.gu.data_ptr(), N, H, L.act.data_ptr())
            # x_next = x1 + act.down^T, added inside the next ln1 (or ln_f)
            self._gemm(h, GEMM_FWD, L.act, Lw["ffn_down"], N, D, H, OUT_F32, self.br)
            if l + 1 < c.nLayers:
                Ln = self.layers[l + 1]
                call("fcu_rmsnorm_fwd_bf16_add", h, L.x1.data_ptr(), self.br.data_ptr(),
                     P["layers"][l + 1]["ln1"].data.data_ptr(), N, D, eps, Ln.x.data_ptr(),
                     Ln.xn.data_ptr(), Ln.inv1.data_ptr())
            else:
                call("fcu_rmsnorm_fwd_bf16_add", h, L.x1.data_ptr(), self.br.data_ptr(),
                     P["ln_f"].data.data_ptr(), N, D, eps, self.xL.data_ptr(), self.xf.data_ptr(),
                     self.invf.data_ptr())
        self._gemm(h, GEMM_FWD, self.xf, W["tok_emb"], N, V, D, OUT_F32, self.logits)
        call("fcu_ce_fwd_bf16grad", h, self.logits.data_ptr(), targets.data_ptr(), N, V,
             self.loss.data_ptr(), self.dlogits.data_ptr())
        return self.loss

    # ------------------------------------------------------------ backward
    def backward(self, g: torch.Tensor | None) -> None:
        """Accumulate d(g * loss)/d(params) into the parameters' gradients;
        `g` (device [1]) None means 1."""
        m, c = self.m, self.m.cfg
        h = AD.ctx().handle
        N, D, H, V, T, B = self.N, c.dim, c.hidden, c.vocabSize, self.T, self.B
        qD = c.nHeads * c.dHead
        W = m.bf16_weights()
        P = m.params
        hook = getattr(m, "grad_ready_hook", None)
        if g is not None:
            call("fcu_scale_bf16_dev", h, self.dlogits.data_ptr(), N * V, g.data_ptr())
        # LM head (tied): dxf = dlogits . E ; dE (+)= dlogits^T . xf
        self._gemm(h, GEMM_DX, self.dlogits, W["tok_emb"], N, D, V, OUT_F32, self.dxn)
        gE, aE = P["tok_emb"]._gout()
        self._gemm(h, GEMM_DW, self.dlogits, self.xf, V, D, N, OUT_F32, gE, accumulate=aE)
        gl, al = P["ln_f"]._gout()
        call("fcu_rmsnorm_bwd_fused", h, self.dxn.data_ptr(), self.xL.data_ptr(),
             P["ln_f"].data.data_ptr(), self.invf.data_ptr(), N, D, self.gx.data_ptr(), 0,
             self.gx_b.data_ptr(), gl.data_ptr(), al)
        for l in range(c.nLayers - 1, -1, -1):
            L, Lp, Lw = self.layers[l], P["layers"][l], W["layers"][l]
            # ff = act . Wdown^T  (dY = g_x2, in gx / gx_b); d act -> d[g | u]
            if self.fuse_swiglu and self.can_fuse_swiglu:
                self._gemm(h, GEMM_DX, self.gx_b, Lw["ffn_down"], N, H, D, OUT_BF16_SWIGLU_BWD,
                           self.dgu, aux=L.gu)
            else:
                self._gemm(h, GEMM_DX, self.gx_b, Lw["ffn_down"], N, H, D, OUT_BF16, self.dact)
                call("fcu_swiglu_bwd_bf16", h, self.dact.data_ptr(), L.gu.data_ptr(), N, H,
                     self.dgu.data_ptr())
            gd, ad = Lp["ffn_down"]._gout()
            self._gemm(h, GEMM_DW, self.gx_b, L.act, D, H, N, OUT_F32, gd, accumulate=ad)
            # [g | u] = xn2 . [Wgate; Wup]^T
            self._gemm(h, GEMM_DX, self.dgu, Lw["ffn_gu"], N, D, 2 * H, OUT_F32, self.dxn)
            gg, ag = Lp["ffn_gate"]._gout()
            Lp["ffn_up"]._gout()
            self._gemm(h, GEMM_DW, self.dgu, L.xn2, 2 * H, D, N, OUT_F32, m.grad_block(l, "ffn_gu"),
                       accumulate=ag)
            # x2 = x1 + ff and xn2 = rmsNorm(x1): g_x1 = g_x2 + rmsNorm'(dxn2), in place
            g2, a2 = Lp["ln2"]._gout()
            call("fcu_rmsnorm_bwd_fused", h, self.dxn.data_ptr(), L.x1.data_ptr(),
                 Lp["ln2"].data.data_ptr(), L.inv2.data_ptr(), N, D, self.gx.data_ptr(), 1,
                 self.gx_b.data_ptr(), g2.data_ptr(), a2)
            # ao = O . Wo^T
            self._gemm(h, GEMM_DX, self.gx_b, Lw["wo"], N, qD, D, OUT_BF16, self.dO)
            go, ao = Lp["wo"]._gout()
            self._gemm(h, GEMM_DW, self.gx_b, L.o, D, qD, N, OUT_F32, go, accumulate=ao)
            call("fcu_attn_bwd_bf16", h, self.dO.data_ptr(), L.qkv.data_ptr(), c.qkvOut,
                 L.o.data_ptr(), L.lse.data_ptr(), B, T, c.nHeads, c.nKvHeads, c.dHead,
                 float(c.ropeTheta), self.dqkv.data_ptr())
            # qkv = xn . Wqkv^T
            self._gemm(h, GEMM_DX, self.dqkv, Lw["wqkv"], N, D, c.qkvOut, OUT_F32, self.dxn)
            gq, aq = Lp["wqkv"]._gout()
            self._gemm(h, GEMM_DW, self.dqkv, L.xn, c.qkvOut, D, N, OUT_F32, gq, accumulate=aq)
            # x1 = x + ao and xn = rmsNorm(x): g_x = g_x1 + rmsNorm'(dxn), in place
            g1, a1 = Lp["ln1"]._gout()
            call("fcu_rmsnorm_bwd_fused", h, self.dxn.data_ptr(), L.x.data_ptr(),
                 Lp["ln1"].data.data_ptr(), L.inv1.data_ptr(), N, D, self.gx.data_ptr(), 1,
                 self.gx_b.data_ptr() if l > 0 else None, g1.data_ptr(), a1)
            if hook is not None:
                hook(l)
        gE, _ = P["tok_emb"]._gout()
        call("fcu_embed_bwd", h, self.gx.data_ptr(), self.ids.data_ptr(), N, V, D, gE.data_ptr())
        if hook is not None:
            hook("head")
