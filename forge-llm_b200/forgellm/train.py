"""TrainableTransformer, initWeights and train(), mirroring forge-llm's
src/L6/train.js (and the Config of src/L6/transformer.js:29-53).

The model wiring is the JS wiring op for op (train.js:120-159).  Parameters
live in ONE flat device buffer in paramList order and their gradients in one
flat gradient buffer, so Adam is a single pass and data-parallel all-reduce
works on contiguous buckets.
"""
from __future__ import annotations

import ctypes as C
import math

import numpy as np
import torch

from . import autograd as AD
from ._lib import ModelCfg, RngState, call, lib  # noqa: F401
from .autograd import Adam, Node, backward, resetTape
from .tensor import (addTensors, causalAttn, causalAttnBatch, crossEntropyMean, embedLookup,
                     matmulT, rmsNorm, ropeRows, sliceCols, swigluRows)


class Config:
    """Model hyper-parameters (src/L6/transformer.js:29-53)."""

    def __init__(self, o=None, **kw):
        o = dict(o or {}, **kw)
        self.dim = o.get("dim", 288)
        self.hidden = o.get("hidden", 768)
        self.nLayers = o.get("nLayers", 6)
        self.nHeads = o.get("nHeads", 6)
        self.nKvHeads = o.get("nKvHeads", 6)
        self.vocabSize = o.get("vocabSize", 32000)
        self.maxSeq = o.get("maxSeq", 1024)
        self.normEps = o.get("normEps", 1e-5)
        self.ropeTheta = o.get("ropeTheta", 10000)
        self.bosId = o.get("bosId", 1)
        self.eosId = o.get("eosId", 2)
        self._derive()

    def _derive(self):
        if self.nHeads % self.nKvHeads != 0:
            raise ValueError(f"GQA requires nHeads({self.nHeads}) divisible by "
                             f"nKvHeads({self.nKvHeads})")
        self.dHead = self.dim // self.nHeads
        self.kvDim = self.nKvHeads * self.dHead
        self.qkvOut = (self.nHeads + 2 * self.nKvHeads) * self.dHead
        self.groupSize = self.nHeads // self.nKvHeads

    def c(self) -> ModelCfg:
        return ModelCfg(self.vocabSize, self.dim, self.nLayers, self.nHeads, self.nKvHeads,
                        self.hidden, float(self.normEps), float(self.ropeTheta))


class RNG:
    """The seeded generator of src/L0/numeric.js:27-49 (host, in libforgecu)."""

    def __init__(self, seed: int = 0x9E3779B9):
        self._s = RngState()
        lib().fcu_rng_init(C.byref(self._s), C.c_uint32(seed & 0xFFFFFFFF))

    def next(self) -> float:
        return lib().fcu_rng_next(C.byref(self._s))

    def normal(self) -> float:
        return lib().fcu_rng_normal(C.byref(self._s))

    def int(self, n: int) -> int:
        return lib().fcu_rng_int(C.byref(self._s), int(n))

    def normals(self, n: int, scale: float = 1.0) -> np.ndarray:
        out = np.empty(int(n), np.float32)
        lib().fcu_rng_fill_normal(C.byref(self._s), out.ctypes.data, int(n), float(scale))
        return out

    def ints(self, n: int, hi: int) -> np.ndarray:
        out = np.empty(int(n), np.int32)
        lib().fcu_rng_fill_int(C.byref(self._s), out.ctypes.data, int(n), int(hi))
        return out


PARAM_NAMES = ("ln1", "ln2", "wqkv", "wo", "ffn_gate", "ffn_up", "ffn_down")


def param_shapes(cfg: Config):
    """(name, numel) in paramList order (train.js:60-78)."""
    D, H, V = cfg.dim, cfg.hidden, cfg.vocabSize
    qD = cfg.nHeads * cfg.dHead
    out = [("tok_emb", V * D), ("ln_f", D)]
    for l in range(cfg.nLayers):
        out += [(f"layer.{l}.ln1", D), (f"layer.{l}.ln2", D), (f"layer.{l}.wqkv", cfg.qkvOut * D),
                (f"layer.{l}.wo", D * qD), (f"layer.{l}.ffn_gate", H * D),
                (f"layer.{l}.ffn_up", H * D), (f"layer.{l}.ffn_down", D * H)]
    return out


def init_weights_flat(cfg: Config, seed: int = 1337) -> np.ndarray:
    """initWeights (train.js:33-57) as one flat float32 host array."""
    c = cfg.c()
    n = int(lib().fcu_model_num_params(C.byref(c)))
    flat = np.empty(n, np.float32)
    call("fcu_init_weights", C.byref(c), C.c_uint32(seed & 0xFFFFFFFF), flat.ctypes.data)
    return flat


def initWeights(cfg: Config, seed: int = 1337) -> dict:
    """The JS weight object: {tok_emb, ln_f, wcls: None, "layer.l": {...}}."""
    flat = init_weights_flat(cfg, seed)
    w, off = {"wcls": None}, 0
    for name, n in param_shapes(cfg):
        arr = flat[off:off + n]
        off += n
        if name.startswith("layer."):
            _, l, p = name.split(".")
            w.setdefault(f"layer.{l}", {})[p] = arr
        else:
            w[name] = arr
    return w


def _flatten_weights(w: dict, cfg: Config) -> np.ndarray:
    parts = [np.asarray(w["tok_emb"], np.float32).ravel(), np.asarray(w["ln_f"], np.float32).ravel()]
    for l in range(cfg.nLayers):
        L = w[f"layer.{l}"]
        parts += [np.asarray(L[p], np.float32).ravel() for p in PARAM_NAMES]
    return np.concatenate(parts)


class TrainableTransformer:
    """src/L6/train.js:83-227."""

    def __init__(self, config, weights=None, seed: int = 1337):
        self.cfg = config if isinstance(config, Config) else Config(config)
        c = self.cfg
        if weights is None:
            flat_host = init_weights_flat(c, seed)
        elif isinstance(weights, dict):
            if weights.get("wcls") is not None:
                raise NotImplementedError("untied LM head (wcls) is not supported")
            flat_host = _flatten_weights(weights, c)
        else:
            flat_host = np.asarray(weights, np.float32).ravel()
        dev = AD.device()
        self.flat_params = torch.from_numpy(flat_host).to(dev)
        self.flat_grads = torch.zeros_like(self.flat_params)
        self.paramList = []
        self.params = {"tok_emb": None, "ln_f": None, "wcls": None, "layers": []}
        off = 0
        for name, n in param_shapes(c):
            p = Node(self.flat_params[off:off + n], requiresGrad=False)
            p.isParam = True
            p._gslot = self.flat_grads[off:off + n]
            self.paramList.append(p)
            off += n
            if name.startswith("layer."):
                _, l, pn = name.split(".")
                l = int(l)
                if l == len(self.params["layers"]):
                    self.params["layers"].append({})
                self.params["layers"][l][pn] = p
            else:
                self.params[name] = p
        self.layer_offsets = self._layer_offsets()
        self.offsets = {}
        off = 0
        for name, n in param_shapes(c):
            self.offsets[name] = (off, off + n)
            off += n
        self.w = None
        # bf16 fused step: None = automatic (bf16 precision and supported
        # shapes), True / False to force.
        self.fused = None
        self._fused_steps = {}
        self.flat_params_bf16 = None
        self._shadow_stale = True
        self._shadow_version = -1
        self._bf16_views = None
        self._build()

    # ------------------------------------------------------------ bf16 fused path
    def _use_fused(self) -> bool:
        from ._lib import FCU_PREC_BF16
        from .fused import fused_supported
        if self.fused is False:
            return False
        ok = AD.ctx().precision == FCU_PREC_BF16 and fused_supported(self.cfg)
        if self.fused is True and not ok:
            raise ValueError("fused step needs bf16 precision and supported shapes")
        return ok

    def bf16_weights(self) -> dict:
        """bf16 views of the weights the fused GEMMs read (re-converted from
        the fp32 parameters when host code or a per-tensor optimizer changed
        them; Adam's flat step keeps them current itself)."""
        if self.flat_params_bf16 is None:
            self.flat_params_bf16 = torch.empty(self.flat_params.numel(), dtype=torch.bfloat16,
                                                device=self.flat_params.device)
            AD.register_shadow(self.flat_params, self)
        if self._shadow_stale or self._shadow_version != self.flat_params._version:
            call("fcu_to_bf16", AD.ctx().handle, self.flat_params.data_ptr(),
                 self.flat_params.numel(), self.flat_params_bf16.data_ptr())
            self._shadow_stale = False
            self._shadow_version = self.flat_params._version
        if self._bf16_views is None:
            s, o = self.flat_params_bf16, self.offsets
            v = lambda name: s[o[name][0]:o[name][1]]  # noqa: E731
            layers = []
            for l in range(self.cfg.nLayers):
                p = f"layer.{l}."
                layers.append({"wqkv": v(p + "wqkv"), "wo": v(p + "wo"),
                               "ffn_gu": s[o[p + "ffn_gate"][0]:o[p + "ffn_up"][1]],
                               "ffn_down": v(p + "ffn_down")})
            self._bf16_views = {"tok_emb": v("tok_emb"), "layers": layers}
        return self._bf16_views

    def grad_block(self, l: int, which: str) -> torch.Tensor:
        """Gradient view of ffn_gate followed by ffn_up of layer l."""
        assert which == "ffn_gu"
        o = self.offsets
        return self.flat_grads[o[f"layer.{l}.ffn_gate"][0]:o[f"layer.{l}.ffn_up"][1]]

    def _fused_loss(self, ids, tgt, B: int, T: int) -> Node:
        from .fused import FusedStep
        key = (B, T)
        fs = self._fused_steps.get(key)
        if fs is None:
            self._fused_steps.clear()           # one shape's buffers at a time
            fs = self._fused_steps[key] = FusedStep(self, B, T)
        idt = AD.as_device(ids, torch.int32)
        tgt = AD.as_device(tgt, torch.int32)
        loss = fs.forward(idt, tgt)
        node = None

        def bwd(g):
            fs.backward(None if getattr(node, "_seeded_one", False) else g)

        node = AD.op(loss, bwd)
        return node

    def _layer_offsets(self):
        """(start, end) of each layer's block in the flat buffers."""
        head = self.cfg.vocabSize * self.cfg.dim + self.cfg.dim
        per = (self.flat_params.numel() - head) // max(1, self.cfg.nLayers)
        return [(head + l * per, head + (l + 1) * per) for l in range(self.cfg.nLayers)]

    def _build(self):
        self.wclsNode = self.params["wcls"] or self.params["tok_emb"]  # tied head (train.js:97)

    def forward(self, ids, pos0: int = 0) -> Node:
        return self._forward(ids, 1, len(ids), pos0)

    def forwardBatch(self, batchIds) -> Node:
        B, T = len(batchIds), len(batchIds[0])
        flat = [i for row in batchIds for i in row]
        return self._forward(flat, B, T, 0)

    def _forward(self, flatIds, B: int, T: int, pos0: int) -> Node:
        """train.js:120-159, op for op."""
        c, ps = self.cfg, self.params
        qD, kvD = c.nHeads * c.dHead, c.nKvHeads * c.dHead
        N = B * T
        hook = getattr(self, "grad_ready_hook", None)
        x = embedLookup(ps["tok_emb"], flatIds, c.vocabSize, c.dim)
        if hook is not None:   # tok_emb's last gradient term is the embedding scatter-add
            AD.after_backward_of(x, lambda: hook("head"))
        for l in range(c.nLayers):
            L = ps["layers"][l]
            xn = rmsNorm(x, L["ln1"], N, c.dim, c.normEps)
            if hook is not None:  # ln1's closure is the last to write layer l's grads
                AD.after_backward_of(xn, (lambda ll: (lambda: hook(ll)))(l))
            qkv = matmulT(xn, L["wqkv"], N, c.dim, c.qkvOut)
            q = sliceCols(qkv, N, c.qkvOut, 0, qD)
            k = sliceCols(qkv, N, c.qkvOut, qD, kvD)
            v = sliceCols(qkv, N, c.qkvOut, qD + kvD, kvD)
            qr = ropeRows(q, N, c.nHeads, c.dHead, pos0, c.ropeTheta, T)
            kr = ropeRows(k, N, c.nKvHeads, c.dHead, pos0, c.ropeTheta, T)
            att = (causalAttn(qr, kr, v, T, c.nHeads, c.nKvHeads, c.dHead) if B == 1 else
                   causalAttnBatch(qr, kr, v, B, T, c.nHeads, c.nKvHeads, c.dHead))
            ao = matmulT(att, L["wo"], N, qD, c.dim)
            x = addTensors(x, ao, N * c.dim)
            xn2 = rmsNorm(x, L["ln2"], N, c.dim, c.normEps)
            g = matmulT(xn2, L["ffn_gate"], N, c.dim, c.hidden)
            u = matmulT(xn2, L["ffn_up"], N, c.dim, c.hidden)
            act = swigluRows(g, u, N, c.hidden)
            ff = matmulT(act, L["ffn_down"], N, c.hidden, c.dim)
            x = addTensors(x, ff, N * c.dim)
        xf = rmsNorm(x, ps["ln_f"], N, c.dim, c.normEps)
        return matmulT(xf, self.wclsNode, N, c.dim, c.vocabSize)

    def loss(self, ids, targets) -> Node:
        """Forward + mean cross-entropy, next-token targets (train.js:166-171)."""
        T = len(targets)
        ids_t = list(ids)[:T] if not isinstance(ids, torch.Tensor) else ids[:T]
        if self._use_fused():
            return self._fused_loss(ids_t, targets, 1, T)
        logits = self.forward(ids_t)
        return crossEntropyMean(logits, targets, T, self.cfg.vocabSize)

    def lossBatch(self, batchIds) -> Node:
        """Block-diagonal batch loss (train.js:177-185).  batchIds: B rows of
        T+1 ids (nested lists, a numpy array or an int tensor, host or device)."""
        if isinstance(batchIds, (np.ndarray, torch.Tensor)):
            arr = batchIds
            B, T = arr.shape[0], arr.shape[1] - 1
            ids, tgt = arr[:, :T].reshape(-1), arr[:, 1:].reshape(-1)
        else:
            B, T = len(batchIds), len(batchIds[0]) - 1
            ids = [r[i] for r in batchIds for i in range(T)]
            tgt = [r[i + 1] for r in batchIds for i in range(T)]
        if self._use_fused():
            return self._fused_loss(ids, tgt, B, T)
        logits = self._forward(ids, B, T, 0)
        return crossEntropyMean(logits, tgt, B * T, self.cfg.vocabSize)

    def backward(self, lossNode: Node) -> float:
        """train.js:188-191: returns the loss value (synchronises)."""
        backward(lossNode)
        return float(lossNode.data[0].item())

    def zeroGrad(self) -> None:
        for p in self.paramList:
            p.zeroGrad()

    def exportWeights(self) -> dict:
        """train.js:199-220: host float32 copies in the JS weight layout."""
        flat = self.flat_params.detach().cpu().numpy()
        w, off = {"wcls": None}, 0
        for name, n in param_shapes(self.cfg):
            arr = flat[off:off + n].copy()
            off += n
            if name.startswith("layer."):
                _, l, p = name.split(".")
                w.setdefault(f"layer.{l}", {})[p] = arr
            else:
                w[name] = arr
        return w

    def countParams(self) -> int:
        return int(self.flat_params.numel())


def train(model: TrainableTransformer, data, opts=None, **kw) -> list:
    """Training loop (train.js:246-276): B random windows per step, block-
    diagonal batch loss, Adam with clip 1 and wd 0.01.

    The token stream is uploaded once.  Every step's window starts are drawn
    before the loop, from the forge-llm RNG in the JS's order (B draws per
    step, step by step; the RNG serves nothing else), and uploaded in one
    copy; step k gathers its windows on the device (fcu_gather_windows) from
    starts[k*B:(k+1)*B].  So the batches are the reference's, and no host
    buffer is rewritten while the GPU may still read it: the loop only syncs
    to log.  On the fused bf16 path the step is replayed as one CUDA graph
    (`graph=False` in the options runs it op by op); the gather writes
    straight into the graph's batch buffer.  `onBatch(step, batch)`, if
    given, is called after each step's gather with the device batch tensor
    (stream-ordered: clone it to keep it)."""
    from . import autograd as AD
    from ._lib import call
    opts = dict(opts or {}, **kw)
    steps = opts.get("steps", 100)
    B = opts.get("batchSize", 8)
    seqLen = opts.get("seqLen", 32)
    lr = opts.get("lr", 1e-2)
    logEvery = opts.get("logEvery", 10)
    rng = RNG(opts.get("seed", 7))
    opt = Adam(model.paramList, lr=lr, totalSteps=steps, clip=1.0, wd=0.01)
    dev = model.flat_params.device
    tokens = torch.as_tensor(np.asarray(data, dtype=np.int32)).to(dev)
    n = tokens.numel()
    T1 = seqLen + 1
    use_graph = opts.get("graph", True) and model._use_fused()
    cs = None
    if use_graph:
        from .graph import CapturedStep
        cs = CapturedStep(model, opt, B, seqLen)
        batch = cs.batch
    else:
        batch = torch.empty((B, T1), dtype=torch.int32, device=dev)
    span = max(1, n - seqLen - 1)
    starts_host = np.array([rng.int(span) for _ in range(steps * B)], dtype=np.int32)
    starts = torch.as_tensor(starts_host).to(dev)   # one synchronous upload
    on_batch = opts.get("onBatch")
    history = []
    for step in range(steps):
        call("fcu_gather_windows", AD.ctx().handle, tokens.data_ptr(), n,
             starts.data_ptr() + 4 * step * B, B, T1, batch.data_ptr())
        if on_batch is not None:
            on_batch(step, batch)
        if cs is not None:
            loss_dev = cs(None)
            info_dev = cs.info
        else:
            resetTape()
            model.zeroGrad()
            lossNode = model.lossBatch(batch)
            loss_dev = lossNode.data
            model.backward(lossNode)
            info = opt.step()
        if step % logEvery == 0 or step == steps - 1:
            l = float(loss_dev.reshape(-1)[0].item())
            if cs is not None:
                g_, _, lr_ = (float(x) for x in info_dev.cpu().tolist())
                info = {"gnorm": g_, "lr": lr_}
            history.append({"step": step, "loss": l, "lr": info["lr"], "gnorm": info["gnorm"]})
            print(f"  step {step:4d}  loss {l:.4f}  lr {info['lr']:.2e}  |g| {info['gnorm']:.3f}")
    if cs is not None:
        cs.graph.reset()
    return history
