"""The inference-side kernels against the CPU oracle (oracle/forge_oracle_infer.c,
pinned to the reference's printed I-20..I-54 values).

- fcu_dequantize_rows: bit-identical to dequantize (src/L3/quant.js:109-209)
  for every supported GGML type, whole tensors and gathered rows (an id
  outside the tensor gives a NaN row).
- fcu_quant_matvec: QuantLinear.forward (src/L4/nn.js:27-32) for M = 1..11
  vectors, relL2 <= 1e-5 against the oracle's double-accumulated dotQ /
  matvec (the GPU accumulates in fp32), on ragged shapes: tensors whose byte
  size is not a multiple of 16, a 1-row tensor, the config-5 LM head.
- fcu_attn_decode: attentionDecode (src/L5/attention.js:31-57) per head with
  GQA, lengths 0 .. 1000 (one chunk and several merged), contiguous and paged
  caches with a shuffled block table: max |diff| <= 1e-5.
- fcu_decode_rope_kv: applyRopeHead with the fp32 ropeTable (q and k rotated
  to 1e-6) and the k / v rows land in the right cache row.
- infer.Transformer: decode steps token by token against the oracle's
  inference forward (src/L6/transformer.js:134-185) with f32, Q8_0, Q4_K,
  Q5_K and Q6_K weights, logits relL2 <= 1e-5; several sequences in one step
  and a paged cache give bit-identical logits to one sequence at a time.
"""
import math

import numpy as np
import pytest

import oracle as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

TOL = 1e-5
TYPES = [O.F32, O.F16, O.Q4_0, O.Q5_0, O.Q8_0, O.Q4_K, O.Q5_K, O.Q6_K]


def _ctx():
    from forgellm.autograd import ctx
    return ctx().handle


def _bytes_for(t, W, N, K, seed):
    """GGML bytes of W [N, K]: the oracle's quantizeRow where the reference
    has a writer; for Q4_0 / Q5_0 (read-only formats in the reference) random
    blocks with a finite f16 scale."""
    if t in (O.Q4_0, O.Q5_0):
        rng = np.random.default_rng(seed)
        bb = O.block_bytes(t)
        nb = N * K // 32
        raw = rng.integers(0, 256, size=(nb, bb), dtype=np.uint8)
        d = (rng.random(nb) * 0.1 + 0.01).astype(np.float16).view(np.uint16)
        raw[:, 0] = d & 0xFF
        raw[:, 1] = d >> 8
        return raw.reshape(-1)
    return O.quantize_row(t, W)


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("t", TYPES)
def test_dequantize_rows_bit_exact(t):
    from forgellm import _lib
    N, K = 9, 512
    W = (O.RNG(70 + t).normals(N * K) * np.float32(0.8)).astype(np.float32)
    b = _bytes_for(t, W, N, K, t)
    rb = O.row_bytes(t, K)
    assert b.size == N * rb
    want = O.dequantize(t, b, N * K).reshape(N, K)
    wb = _dev(b)
    out = torch.full((N, K), 7.0, device="cuda")
    _lib.call("fcu_dequantize_rows", _ctx(), t, wb.data_ptr(), N, K, None, N, out.data_ptr())
    ids = _dev(np.array([3, 0, 8, 3, -1, 9], np.int32))
    g = torch.empty((6, K), device="cuda")
    _lib.call("fcu_dequantize_rows", _ctx(), t, wb.data_ptr(), N, K, ids.data_ptr(), 6, g.data_ptr())
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    gg = g.cpu().numpy()
    for r, src in enumerate([3, 0, 8, 3]):
        assert np.array_equal(gg[r], want[src])
    assert np.isnan(gg[4]).all() and np.isnan(gg[5]).all()


@pytest.mark.parametrize("t", TYPES)
@pytest.mark.parametrize("N,K,M", [(37, 512, 1), (3, 256, 3), (1, 256, 1), (130, 2048, 8), (50, 768, 11)])
def test_quant_matvec_matches_oracle(t, N, K, M):
    from forgellm import _lib
    if K % O.block_size(t):
        pytest.skip("K not a multiple of the block")
    W = (O.RNG(80 + t + N).normals(N * K) * np.float32(0.5)).astype(np.float32)
    b = _bytes_for(t, W, N, K, t + N)
    X = O.RNG(90 + M).normals(M * K)
    want = np.stack([O.quantlinear_fwd(t, b, X[m * K:(m + 1) * K], N, K) for m in range(M)])
    wb, xd = _dev(b), _dev(X)
    Y = torch.full((M, N), float("nan"), device="cuda")
    for _ in range(2):
        _lib.call("fcu_quant_matvec", _ctx(), t, wb.data_ptr(), N, K, xd.data_ptr(), M, Y.data_ptr())
    torch.cuda.synchronize()
    assert _lib.lib().fcu_check_device_error(_ctx()) == 0
    got = Y.cpu().numpy()
    assert np.isfinite(got).all()
    assert O.rel_l2(want.ravel(), got.ravel()) <= TOL


@pytest.mark.parametrize("t", [O.Q4_K, O.Q8_0, O.Q6_K])
def test_quant_matvec_config5_lm_head(t):
    """The config-5 tied LM head (32000 x 768) as one decode-step matvec."""
    from forgellm import _lib
    N, K = 32000, 768
    W = (O.RNG(5).normals(N * K) * np.float32(0.02)).astype(np.float32)
    b = O.quantize_row(t, W)
    x = O.RNG(6).normals(K)
    want = O.quantlinear_fwd(t, b, x, N, K)
    Y = torch.empty(N, device="cuda")
    wb, xd = _dev(b), _dev(x)
    _lib.call("fcu_quant_matvec", _ctx(), t, wb.data_ptr(), N, K, xd.data_ptr(), 1, Y.data_ptr())
    torch.cuda.synchronize()
    assert O.rel_l2(want, Y.cpu().numpy()) <= TOL


def test_quant_matvec_rejects_bad_shapes():
    from forgellm import _lib
    L = _lib.lib()
    w = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    x = torch.zeros(512, device="cuda")
    y = torch.zeros(4, device="cuda")
    h = _ctx()
    assert L.fcu_quant_matvec(h, O.Q4_K, w.data_ptr(), 4, 300, x.data_ptr(), 1, y.data_ptr()) == _lib.FCU_ERR_ARG
    assert L.fcu_quant_matvec(h, 3, w.data_ptr(), 4, 256, x.data_ptr(), 1, y.data_ptr()) == _lib.FCU_ERR_ARG
    assert L.fcu_quant_matvec(h, O.Q8_0, w.data_ptr() + 2, 4, 64, x.data_ptr(), 1, y.data_ptr()) == _lib.FCU_ERR_ARG


def _cache_rows(table, b, n, block):
    return [int(table[b, p // block]) * block + p % block for p in range(n)]


@pytest.mark.parametrize("nH,nKV,dH", [(12, 4, 64), (4, 4, 16), (16, 2, 128), (4, 2, 256), (32, 8, 128),
                                       (8, 8, 32), (6, 2, 96)])
@pytest.mark.parametrize("paged", [False, True])
def test_attn_decode_matches_oracle(nH, nKV, dH, paged):
    from forgellm import _lib
    lens = [0, 1, 5, 256, 257, 1000]
    B = len(lens)
    block = 64 if paged else 1024
    max_blocks = 1024 // block
    kvDim = nKV * dH
    phys = B * max_blocks
    if paged:
        table = np.random.default_rng(3).permutation(phys).astype(np.int32).reshape(B, max_blocks)
    else:
        table = np.arange(phys, dtype=np.int32).reshape(B, max_blocks)
    rng = O.RNG(40 + dH)
    kc = rng.normals(phys * block * kvDim).reshape(phys * block, kvDim)
    vc = rng.normals(phys * block * kvDim).reshape(phys * block, kvDim)
    ld = (nH + 2 * nKV) * dH
    q = rng.normals(B * ld).reshape(B, ld)
    out = torch.full((B, nH * dH), float("nan"), device="cuda")
    kd, vd, qd = _dev(kc), _dev(vc), _dev(q)
    ld_lens = _dev(np.array(lens, np.int32))
    td = _dev(table) if paged else None
    scale = 1 / math.sqrt(dH)
    for _ in range(2):
        _lib.call("fcu_attn_decode", _ctx(), qd.data_ptr(), ld, kd.data_ptr(), vd.data_ptr(), kvDim,
                  td.data_ptr() if td is not None else None, max_blocks, block, ld_lens.data_ptr(), B, nH, nKV,
                  dH, scale, out.data_ptr())
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    g = nH // nKV
    for b, n in enumerate(lens):
        rows = _cache_rows(table, b, n, block)
        for h in range(nH):
            kvh = h // g
            K_ = kc[rows, kvh * dH:(kvh + 1) * dH].ravel() if n else np.zeros(dH, np.float32)
            V_ = vc[rows, kvh * dH:(kvh + 1) * dH].ravel() if n else np.zeros(dH, np.float32)
            want = O.attention_decode(q[b, h * dH:(h + 1) * dH], K_, V_, n, dH, scale, True, max(n - 1, 0), 0)
            assert np.max(np.abs(want - got[b, h * dH:(h + 1) * dH])) <= TOL, (b, n, h)


@pytest.mark.parametrize("paged", [False, True])
def test_decode_rope_kv_rotates_and_writes_the_cache(paged):
    from forgellm import _lib
    B, nH, nKV, dH, theta = 3, 4, 2, 32, 10000.0
    block = 16 if paged else 128
    max_blocks = 128 // block
    phys = B * max_blocks
    table = (np.random.default_rng(1).permutation(phys).astype(np.int32).reshape(B, max_blocks) if paged
             else np.arange(phys, dtype=np.int32).reshape(B, max_blocks))
    kvDim, ld = nKV * dH, (nH + 2 * nKV) * dH
    pos = np.array([0, 37, 127], np.int32)
    qkv = O.RNG(2).normals(B * ld).reshape(B, ld)
    kc = torch.zeros(phys * block, kvDim, device="cuda")
    vc = torch.zeros_like(kc)
    xd, posd, td = _dev(qkv), _dev(pos), _dev(table)   # held: the kernels read them later
    tptr = td.data_ptr() if paged else None
    _lib.call("fcu_decode_rope_kv", _ctx(), xd.data_ptr(), ld, B, nH, nKV, dH, theta, posd.data_ptr(),
              kc.data_ptr(), vc.data_ptr(), kvDim, tptr, max_blocks, block)
    # a position outside the cache changes nothing
    bad = _dev(np.array([128, -1, 500], np.int32))
    before = xd.clone()
    _lib.call("fcu_decode_rope_kv", _ctx(), xd.data_ptr(), ld, B, nH, nKV, dH, theta, bad.data_ptr(),
              kc.data_ptr(), vc.data_ptr(), kvDim, tptr, max_blocks, block)
    torch.cuda.synchronize()
    assert torch.equal(before, xd)
    cosT, sinT = O.rope_table(128, dH, theta)
    got = xd.cpu().numpy()
    kch, vch = kc.cpu().numpy(), vc.cpu().numpy()
    for b in range(B):
        want = qkv[b].astype(np.float64).copy()
        p = int(pos[b])
        for hd in range(nH + nKV):
            for i in range(0, dH, 2):
                c, s = float(cosT[p * dH // 2 + i // 2]), float(sinT[p * dH // 2 + i // 2])
                a, bb = want[hd * dH + i], want[hd * dH + i + 1]
                want[hd * dH + i], want[hd * dH + i + 1] = a * c - bb * s, a * s + bb * c
        want = want.astype(np.float32)
        assert np.max(np.abs(got[b] - want)) <= 1e-6 * max(1.0, float(np.abs(want).max()))
        row = _cache_rows(table, b, p + 1, block)[p]
        assert np.array_equal(kch[row], got[b, nH * dH:(nH + nKV) * dH])
        assert np.array_equal(vch[row], qkv[b, (nH + nKV) * dH:])
    written = {_cache_rows(table, b, int(pos[b]) + 1, block)[int(pos[b])] for b in range(B)}
    others = [r for r in range(phys * block) if r not in written]
    assert not np.any(kch[others]) and not np.any(vch[others])


CFG = dict(dim=256, hidden=512, nLayers=2, nHeads=4, nKvHeads=2, vocabSize=128, maxSeq=32)


def _models(w_type, tok_type):
    import forgellm as F
    from forgellm.train import Config, init_weights_flat
    cfg = Config(**CFG)
    ocfg = O.Config(**{k: v for k, v in CFG.items() if k != "maxSeq"})
    P = init_weights_flat(cfg, 11)
    w = O.unflatten_weights(ocfg, P)
    om = O.InferModel(ocfg, w, max_seq=CFG["maxSeq"], w_type=w_type, tok_type=tok_type)
    gw = {"tok_emb": F.QuantLinear(tok_type, om.tok, cfg.vocabSize, cfg.dim), "ln_f": w["ln_f"]}
    for l in range(cfg.nLayers):
        L = {"ln1": w[f"layer.{l}"]["ln1"], "ln2": w[f"layer.{l}"]["ln2"]}
        shapes = {"wqkv": (cfg.qkvOut, cfg.dim), "wo": (cfg.dim, cfg.dim), "ffn_gate": (cfg.hidden, cfg.dim),
                  "ffn_up": (cfg.hidden, cfg.dim), "ffn_down": (cfg.dim, cfg.hidden)}
        for k, (n_, k_) in shapes.items():
            L[k] = F.QuantLinear(w_type, om.mats[k][l], n_, k_)
        gw[f"layer.{l}"] = L
    return cfg, om, F.Transformer(cfg).loadWeights(gw)


@pytest.mark.parametrize("w_type,tok_type", [(O.F32, O.F32), (O.Q8_0, O.Q8_0), (O.Q4_K, O.Q8_0),
                                             (O.Q5_K, O.F32), (O.Q6_K, O.Q6_K)])
def test_transformer_decode_matches_oracle(w_type, tok_type):
    import forgellm as F
    cfg, om, tr = _models(w_type, tok_type)
    cache = F.KVCache(cfg.nLayers, cfg.maxSeq, cfg.kvDim)
    ids = O.RNG(12).ints(12, cfg.vocabSize)
    for t, tok in enumerate(ids):
        want = om.forward(int(tok), t)
        got = tr.forward(int(tok), t, cache).cpu().numpy()
        assert O.rel_l2(want, got) <= TOL, (t, O.rel_l2(want, got))


def test_transformer_batch_and_paged_cache_match_single_sequences():
    """Three sequences stepped together (each at its own position) and a
    paged cache with a shuffled block table give the logits of stepping each
    sequence alone, bit for bit."""
    import forgellm as F
    cfg, _, tr = _models(O.Q4_K, O.Q8_0)
    seqs = [O.RNG(20 + s).ints(9, cfg.vocabSize) for s in range(3)]
    alone = []
    for s in range(3):
        cache = F.KVCache(cfg.nLayers, cfg.maxSeq, cfg.kvDim)
        alone.append([tr.forward(int(t), p, cache).cpu().numpy().copy() for p, t in enumerate(seqs[s])])
    table = np.random.default_rng(5).permutation(3 * 4).astype(np.int32).reshape(3, 4)
    for cache in (F.KVCache(cfg.nLayers, cfg.maxSeq, cfg.kvDim, batch=3),
                  F.PagedKVCache(cfg.nLayers, cfg.maxSeq, cfg.kvDim, blockSize=8, batch=3, table=table)):
        # sequence s starts s steps late, so the three sit at different positions
        pos = [0, 0, 0]
        for step in range(11):
            active = [s for s in range(3) if step >= s and pos[s] < 9]
            if not active:
                continue
            # the batch covers all three rows of the cache; inactive rows re-run
            # their last step (rewriting the same cache row with the same values)
            toks = [int(seqs[s][min(pos[s], 8)]) if s in active else int(seqs[s][max(pos[s] - 1, 0)])
                    for s in range(3)]
            ps = [pos[s] if s in active else max(pos[s] - 1, 0) for s in range(3)]
            logits = tr.forwardBatch(toks, ps, cache).cpu().numpy()
            for s in active:
                assert np.array_equal(logits[s], alone[s][pos[s]]), (type(cache).__name__, s, pos[s])
                pos[s] += 1


def test_transformer_graph_replay_matches_eager():
    """forwardBatch(graph=True): the first step runs op by op and captures,
    later steps replay the captured launches with new tokens and positions;
    every step's logits equal the eager step's bit for bit (one sequence and
    a paged batch of three)."""
    import forgellm as F
    cfg, _, tr = _models(O.Q4_K, O.Q8_0)
    ids = O.RNG(31).ints(10, cfg.vocabSize)
    eager, graphed = F.KVCache(cfg.nLayers, cfg.maxSeq, cfg.kvDim), F.KVCache(cfg.nLayers, cfg.maxSeq, cfg.kvDim)
    for t, tok in enumerate(ids):
        want = tr.forward(int(tok), t, eager).cpu().numpy().copy()
        got = tr.forward(int(tok), t, graphed, graph=True).cpu().numpy()
        assert np.array_equal(want, got), t
    table = np.random.default_rng(7).permutation(12).astype(np.int32).reshape(3, 4)
    pe = F.PagedKVCache(cfg.nLayers, cfg.maxSeq, cfg.kvDim, blockSize=8, batch=3, table=table)
    pg = F.PagedKVCache(cfg.nLayers, cfg.maxSeq, cfg.kvDim, blockSize=8, batch=3, table=table)
    seqs = [O.RNG(40 + s).ints(6, cfg.vocabSize) for s in range(3)]
    for p in range(6):
        toks = [int(seqs[s][p]) for s in range(3)]
        ps = [p + s for s in range(3)]
        want = tr.forwardBatch(toks, ps, pe).cpu().numpy().copy()
        got = tr.forwardBatch(toks, ps, pg, graph=True).cpu().numpy()
        assert np.array_equal(want, got), p
