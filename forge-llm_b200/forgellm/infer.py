"""The inference side of forge-llm on the GPU: QuantLinear over GGUF block
formats (src/L4/nn.js:19-41), the KV caches and single-query attentions of
src/L5/attention.js, and Transformer.forward, one decode step
(src/L6/transformer.js:67-185), for one or several sequences at once.

Weights stay in their GGML byte layout on the device and are read by
fcu_quant_matvec (one pass over W for every sequence of the step); the KV
cache rows are written by fcu_decode_rope_kv and read by fcu_attn_decode.  As
everywhere in this package, no torch kernel computes: torch only allocates.
Quantizing from fp32 (quantizeRow, the export path) is not part of this
module: weights come as GGML bytes (a GGUF file, llama-quantize, the JS
writer), or as fp32 (type 0).
"""
from __future__ import annotations

import math

import numpy as np
import torch

from ._lib import call, lib
from .autograd import ctx, device

F32, F16, Q4_0, Q5_0, Q8_0, Q4_K, Q5_K, Q6_K = 0, 1, 2, 6, 8, 12, 13, 14


def row_bytes(type_: int, n: int) -> int:
    """rowBytes (src/L3/quant.js:62)."""
    rb = int(lib().fcu_ggml_row_bytes(int(type_), int(n)))
    if rb < 0:
        raise ValueError(f"unsupported GGML type {type_}")
    return rb


def _dev_f32(x) -> torch.Tensor:
    t = x if isinstance(x, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(x, np.float32))
    return t.to(device=device(), dtype=torch.float32).contiguous()


class QuantLinear:
    """W[N, K] as a GGML byte stream on the device (nn.js:19-41).
    `bytes_` is a uint8 array / tensor of N * rowBytes(type, K) bytes, or for
    type 0 a float32 array of N * K values."""

    def __init__(self, type_: int, bytes_, N: int, K: int):
        self.type, self.N, self.K = int(type_), int(N), int(K)
        if isinstance(bytes_, torch.Tensor):
            b = bytes_.detach().contiguous().view(torch.uint8).reshape(-1)
        else:
            b = torch.from_numpy(np.ascontiguousarray(bytes_).view(np.uint8).reshape(-1))
        if b.numel() != N * row_bytes(type_, K):
            raise ValueError(f"QuantLinear: {b.numel()} bytes for {N} rows of {K} (type {type_})")
        self.bytes = b.to(device())

    @staticmethod
    def fromF32(W, N: int, K: int, type_: int = 0) -> "QuantLinear":
        if type_ != F32:
            raise NotImplementedError("quantizing on the device is not provided; pass GGML bytes")
        return QuantLinear(F32, np.asarray(W, np.float32), N, K)

    def forward(self, x, out: torch.Tensor | None = None) -> torch.Tensor:
        """out[N] = W . x, or out[M, N] for x [M, K] (M vectors, one pass over W)."""
        X = _dev_f32(x)
        M = X.numel() // self.K
        if M * self.K != X.numel():
            raise ValueError(f"QuantLinear.forward: input of {X.numel()} values, K = {self.K}")
        if out is None:
            out = torch.empty((M, self.N) if x.ndim == 2 else (self.N,), dtype=torch.float32, device=X.device)
        call("fcu_quant_matvec", ctx().handle, self.type, self.bytes.data_ptr(), self.N, self.K, X.data_ptr(), M,
             out.data_ptr())
        return out

    def toF32(self) -> torch.Tensor:
        """dequantize of the whole tensor, [N * K] (nn.js:34-37)."""
        out = torch.empty(self.N * self.K, dtype=torch.float32, device=self.bytes.device)
        call("fcu_dequantize_rows", ctx().handle, self.type, self.bytes.data_ptr(), self.N, self.K, None, self.N,
             out.data_ptr())
        return out

    def rows(self, ids: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """Dequantized rows ids (device int32) -> [len(ids), K] (the quantized
        embedding lookup, transformer.js:122-132)."""
        n = ids.numel()
        if out is None:
            out = torch.empty((n, self.K), dtype=torch.float32, device=self.bytes.device)
        call("fcu_dequantize_rows", ctx().handle, self.type, self.bytes.data_ptr(), self.N, self.K, ids.data_ptr(),
             n, out.data_ptr())
        return out

    def bytesSize(self) -> int:
        return self.bytes.numel()


class KVCache:
    """Contiguous KV cache (attention.js:128-154): k, v [nLayers, maxSeq,
    kvDim] per sequence, `batch` sequences side by side (sequence b owns
    rows [b * maxSeq, (b + 1) * maxSeq) of every layer)."""

    def __init__(self, nLayers: int, maxSeq: int, kvDim: int, batch: int = 1):
        self.nLayers, self.maxSeq, self.kvDim, self.batch = nLayers, maxSeq, kvDim, batch
        self.k = torch.zeros(nLayers, batch * maxSeq, kvDim, dtype=torch.float32, device=device())
        self.v = torch.zeros_like(self.k)
        self.len = 0
        self.block_size, self.max_blocks, self.table = maxSeq, 1, None

    def rows_per_layer(self) -> int:
        return self.k.shape[1]

    def put(self, layer: int, pos: int, k, v, seq: int = 0) -> None:
        r = seq * self.maxSeq + pos
        self.k[layer, r].copy_(_dev_f32(k).reshape(-1))
        self.v[layer, r].copy_(_dev_f32(v).reshape(-1))
        self.len = max(self.len, pos + 1)

    def kView(self, layer: int, upto: int, seq: int = 0) -> torch.Tensor:
        return self.k[layer, seq * self.maxSeq:seq * self.maxSeq + upto]

    def vView(self, layer: int, upto: int, seq: int = 0) -> torch.Tensor:
        return self.v[layer, seq * self.maxSeq:seq * self.maxSeq + upto]

    def sliceK(self, layer: int, pos: int, seq: int = 0) -> torch.Tensor:
        return self.k[layer, seq * self.maxSeq + pos]

    def sliceV(self, layer: int, pos: int, seq: int = 0) -> torch.Tensor:
        return self.v[layer, seq * self.maxSeq + pos]

    def reset(self) -> None:
        self.len = 0

    def bytes(self) -> int:
        return 2 * self.k.numel() * 4


class PagedKVCache(KVCache):
    """Block-allocated KV cache (attention.js:157-187): blocks of blockSize
    rows; sequence b's logical block i lives in physical block
    table[b, i] (default: b * nBlocks + i, the reference's linear layout)."""

    def __init__(self, nLayers: int, maxSeq: int, kvDim: int, blockSize: int = 64, batch: int = 1,
                 table: np.ndarray | None = None, physBlocks: int | None = None):
        self.nLayers, self.maxSeq, self.kvDim, self.batch = nLayers, maxSeq, kvDim, batch
        self.blockSize = self.block_size = blockSize
        self.nBlocks = self.max_blocks = -(-maxSeq // blockSize)
        phys = physBlocks if physBlocks is not None else batch * self.nBlocks
        self.k = torch.zeros(nLayers, phys * blockSize, kvDim, dtype=torch.float32, device=device())
        self.v = torch.zeros_like(self.k)
        self.len = 0
        if table is None:
            self.table = None
            self._table_host = np.arange(batch * self.nBlocks, dtype=np.int32).reshape(batch, self.nBlocks)
        else:
            t = np.ascontiguousarray(table, np.int32).reshape(batch, self.nBlocks)
            if t.min() < 0 or t.max() >= phys:
                raise ValueError("PagedKVCache: block table entry outside the physical blocks")
            self._table_host = t
            self.table = torch.from_numpy(t).to(device())

    def _row(self, pos: int, seq: int = 0) -> int:
        return int(self._table_host[seq, pos // self.blockSize]) * self.blockSize + pos % self.blockSize

    def kOff(self, layer: int, pos: int, seq: int = 0) -> int:
        return (layer * self.k.shape[1] + self._row(pos, seq)) * self.kvDim

    def put(self, layer: int, pos: int, k, v, seq: int = 0) -> None:
        r = self._row(pos, seq)
        self.k[layer, r].copy_(_dev_f32(k).reshape(-1))
        self.v[layer, r].copy_(_dev_f32(v).reshape(-1))
        self.len = max(self.len, pos + 1)

    def sliceK(self, layer: int, pos: int, seq: int = 0) -> torch.Tensor:
        return self.k[layer, self._row(pos, seq)]

    def sliceV(self, layer: int, pos: int, seq: int = 0) -> torch.Tensor:
        return self.v[layer, self._row(pos, seq)]

    def contiguousKV(self, layer: int, upto: int, seq: int = 0):
        idx = torch.tensor([self._row(p, seq) for p in range(upto)], device=self.k.device)
        return self.k[layer].index_select(0, idx), self.v[layer].index_select(0, idx)


def _single_query(out, q, K, V, n, d, scale, causal, qOff, kOff):
    """One query row against K/V rows [kOff/d, kOff/d + n) of d values."""
    Kd, Vd, qd = _dev_f32(K), _dev_f32(V), _dev_f32(q)
    end = min(n, qOff + 1) if causal else n
    end = max(end, 0)
    lens = torch.tensor([end], dtype=torch.int32, device=Kd.device)
    if out is None:
        out = torch.empty(d, dtype=torch.float32, device=Kd.device)
    cap = max(n, 1)
    call("fcu_attn_decode", ctx().handle, qd.data_ptr(), d, Kd.data_ptr() + 4 * kOff, Vd.data_ptr() + 4 * kOff, d,
         None, 1, cap, lens.data_ptr(), 1, 1, 1, d, float(scale), out.data_ptr())
    return out


def attentionDecode(out, q, K, V, n, d, scale, causal=True, qOff=0, kOff=0, s=None):
    """attention.js:31-57 (the scores buffer `s` is not needed)."""
    return _single_query(out, q, K, V, n, d, scale, causal, qOff, kOff)


def flashAttention(out, q, K, V, n, d, scale, causal=True, qOff=0, kOff=0, block=64):
    """attention.js:89-125: the same online-softmax arithmetic as
    attentionDecode on the GPU (chunks of 256 positions, merged)."""
    return _single_query(out, q, K, V, n, d, scale, causal, qOff, kOff)


def attentionNaive(out, q, K, V, n, d, scale, causal=True, qOff=0, kOff=0):
    """attention.js:63-79."""
    return _single_query(out, q, K, V, n, d, scale, causal, qOff, kOff)


class Transformer:
    """Inference model (transformer.js:67-185) on the GPU.  loadWeights takes
    the export dict (tok_emb, ln_f, layer.{l}.{ln1, ln2, wqkv, wo, ffn_gate,
    ffn_up, ffn_down}, optional wcls) with fp32 arrays or QuantLinear values.
    forward(token, pos, cache) is one decode step of one sequence;
    forwardBatch(tokens, positions, cache) steps cache.batch sequences at once
    (each at its own position) and returns logits [B, vocab]."""

    def __init__(self, config):
        from .train import Config
        self.cfg = config if isinstance(config, Config) else Config(config)
        c = self.cfg
        self.layers = []
        self.tokEmb = self.wcls = self.lnF = None
        self.maxSeq = c.maxSeq

    @staticmethod
    def _ql(w, N, K):
        return w if isinstance(w, QuantLinear) else QuantLinear(F32, np.asarray(w, np.float32), N, K)

    def loadWeights(self, w: dict) -> "Transformer":
        c = self.cfg
        self.tokEmb = self._ql(w["tok_emb"], c.vocabSize, c.dim)
        self.wcls = self._ql(w["wcls"], c.vocabSize, c.dim) if w.get("wcls") is not None else self.tokEmb
        self.lnF = _dev_f32(w["ln_f"])
        self.layers = []
        for l in range(c.nLayers):
            L = w[f"layer.{l}"]
            self.layers.append(dict(
                ln1=_dev_f32(L["ln1"]), ln2=_dev_f32(L["ln2"]),
                wqkv=self._ql(L["wqkv"], c.qkvOut, c.dim), wo=self._ql(L["wo"], c.dim, c.dim),
                gate=self._ql(L["ffn_gate"], c.hidden, c.dim), up=self._ql(L["ffn_up"], c.hidden, c.dim),
                down=self._ql(L["ffn_down"], c.dim, c.hidden)))
        self._bufs = {}
        return self

    def _buffers(self, B):
        b = self._bufs.get(B)
        if b is None:
            c = self.cfg
            dev = device()
            z = lambda *s: torch.empty(*s, dtype=torch.float32, device=dev)  # noqa: E731
            b = self._bufs[B] = dict(x=z(B, c.dim), xb=z(B, c.dim), xb2=z(B, c.dim), inv=z(B), q=z(B, c.qkvOut),
                                     att=z(B, c.dim), g=z(B, c.hidden), u=z(B, c.hidden), h=z(B, c.hidden),
                                     logits=z(B, c.vocabSize),
                                     ids=torch.empty(B, dtype=torch.int32, device=dev),
                                     pos=torch.empty(B, dtype=torch.int32, device=dev),
                                     lens=torch.empty(B, dtype=torch.int32, device=dev))
        return b

    def forward(self, token: int, pos: int, cache: KVCache, graph: bool = False) -> torch.Tensor:
        """One token at position pos (transformer.js:134-185): logits [vocab]."""
        return self.forwardBatch([token], [pos], cache, graph=graph)[0]

    def forwardBatch(self, tokens, positions, cache: KVCache, graph: bool = False) -> torch.Tensor:
        """Logits [B, vocab] of one decode step.  graph=True replays the step
        as a CUDA graph: the first call for a (batch size, cache) pair runs
        op by op and captures the same launches; later calls copy the tokens
        and positions into the step's device buffers and replay, which removes
        the ~140 host launches per step.  The returned logits buffer is
        rewritten by the next step."""
        c = self.cfg
        B = len(tokens)
        if B > cache.batch:
            raise ValueError(f"{B} sequences for a cache of {cache.batch}")
        bf = self._buffers(B)
        host = np.array([list(tokens), list(positions), [p + 1 for p in positions]], np.int32)
        dev_host = torch.from_numpy(host)
        bf["ids"].copy_(dev_host[0])
        bf["pos"].copy_(dev_host[1])
        bf["lens"].copy_(dev_host[2])
        cache.len = max(cache.len, max(positions) + 1)
        if not graph:
            return self._step(B, cache)
        from ._lib import lib
        import ctypes
        graphs = self.__dict__.setdefault("_graphs", {})
        key = (B, id(cache))
        scr = ctypes.c_size_t(0)
        lib().fcu_ctx_scratch_bytes(ctx().handle, ctypes.byref(scr))
        g = graphs.get(key)
        # a graph holds the context scratch's address: if the scratch has
        # grown since the capture, capture again
        if g is not None and g[1] == scr.value and g[2] is cache.k:
            g[0].replay()
            return bf["logits"]
        out = self._step(B, cache)          # this step, op by op (sizes every workspace)
        lib().fcu_ctx_scratch_bytes(ctx().handle, ctypes.byref(scr))
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        graph_ = torch.cuda.CUDAGraph()
        with torch.cuda.stream(side):
            with torch.cuda.graph(graph_, stream=side):
                self._step(B, cache)
        torch.cuda.current_stream().wait_stream(side)
        ctx()                               # the context follows the caller's stream again
        graphs[key] = (graph_, scr.value, cache.k)
        return out

    def _step(self, B: int, cache: KVCache) -> torch.Tensor:
        """The launches of one decode step on the step's device buffers."""
        c = self.cfg
        bf = self._bufs[B]
        h = ctx().handle
        D, dH = c.dim, c.dHead
        x, xb, xb2, inv, q, att = bf["x"], bf["xb"], bf["xb2"], bf["inv"], bf["q"], bf["att"]
        self.tokEmb.rows(bf["ids"], out=x)
        table = cache.table.data_ptr() if cache.table is not None else None
        rows = cache.rows_per_layer()
        for l, L in enumerate(self.layers):
            call("fcu_rmsnorm_fwd", h, x.data_ptr(), L["ln1"].data_ptr(), B, D, float(c.normEps), xb.data_ptr(),
                 inv.data_ptr())
            L["wqkv"].forward(xb, out=q)
            kc = cache.k.data_ptr() + 4 * l * rows * c.kvDim
            vc = cache.v.data_ptr() + 4 * l * rows * c.kvDim
            call("fcu_decode_rope_kv", h, q.data_ptr(), c.qkvOut, B, c.nHeads, c.nKvHeads, dH, float(c.ropeTheta),
                 bf["pos"].data_ptr(), kc, vc, c.kvDim, table, cache.max_blocks, cache.block_size)
            call("fcu_attn_decode", h, q.data_ptr(), c.qkvOut, kc, vc, c.kvDim, table, cache.max_blocks,
                 cache.block_size, bf["lens"].data_ptr(), B, c.nHeads, c.nKvHeads, dH, 1 / math.sqrt(dH),
                 att.data_ptr())
            L["wo"].forward(att, out=xb2)
            call("fcu_add_fwd", h, x.data_ptr(), xb2.data_ptr(), B * D, x.data_ptr())
            call("fcu_rmsnorm_fwd", h, x.data_ptr(), L["ln2"].data_ptr(), B, D, float(c.normEps), xb.data_ptr(),
                 inv.data_ptr())
            L["gate"].forward(xb, out=bf["g"])
            L["up"].forward(xb, out=bf["u"])
            call("fcu_swiglu_fwd", h, bf["g"].data_ptr(), bf["u"].data_ptr(), B * c.hidden, bf["h"].data_ptr())
            L["down"].forward(bf["h"], out=xb2)
            call("fcu_add_fwd", h, x.data_ptr(), xb2.data_ptr(), B * D, x.data_ptr())
        call("fcu_rmsnorm_fwd", h, x.data_ptr(), self.lnF.data_ptr(), B, D, float(c.normEps), xb.data_ptr(),
             inv.data_ptr())
        self.wcls.forward(xb, out=bf["logits"])
        return bf["logits"]
