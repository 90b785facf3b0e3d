#!/usr/bin/env python
"""bench.py -- training tokens/s of forge-llm's ~125M Llama-style
TrainableTransformer step (fwd + bwd + Adam) on 1..8 B200s.

Workload: vocab 32000, d_model 768, 12 layers, 12 q / 4 kv
heads x 64, SwiGLU hidden 2048, RMSNorm eps 1e-5, RoPE 10000, context 1024,
global batch 64 sequences split over the ranks (strong scaling), weights
initWeights(cfg, 5) ~N(0, 0.02), tokens uniform in [0, 32000) from RNG(5),
Adam lr 3e-4.  A step is one lossBatch + backward + Adam.step through the
forgellm API (the JS TrainableTransformer API), every kernel from
libforgecu.so.

One JSON line on rank 0.  `value` = whole-job tokens/s with the batch already
in HBM; `e2e` = the same step through the public API with the batch copied
from pinned host memory and the loss read back every step.  `roofline` is the
matmulT contractions (the dominant kernels), timed live with CUDA events on
the launching stream inside the timed region.  `cpu_baseline` is the CPU
oracle (a restatement of the reference's JS loops) timed on a bounded sample
on this host.  `--impl reference` times that CPU path alone (the reference is
JavaScript and no JS runtime exists on this box).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "forge-llm_b200"))

C5 = dict(vocabSize=32000, dim=768, nLayers=12, nHeads=12, nKvHeads=4, hidden=2048,
          normEps=1e-5, ropeTheta=10000)
GLOBAL_BATCH, SEQ, LR, SEED = 64, 1024, 3e-4, 5
# DRAM bytes (read, written) of one launch of each distinct GEMM of the
# config-5 step (batch 64), from one single-pass ncu capture of the 147 GEMM
# launches of a step of `bench.py --steps 1 --warmup 1` (dram__bytes_read.sum /
# dram__bytes_write.sum, captured with `ncu --metrics ... -k regex:gemm_bf16 -s 147 -c 147`),
# each shape the mean over its launches.  The twelve per-layer shapes run 12
# times a step, the three LM-head shapes once.
GEMM_DRAM_BY_SHAPE = {
    "qkv_fwd": (102966784, 113806336),
    "wo_fwd": (101923178, 140066282),
    "gateup_fwd": (107071125, 475336021),
    "down_fwd": (271996309, 159808874),
    "down_dx": (103879466, 208736618),
    "down_dw": (369171861, 729685),
    "gateup_dx": (593923242, 174608661),
    "gateup_dw": (682318506, 19698837),
    "wo_dx": (101923114, 56008597),
    "wo_dw": (201403925, 361834),
    "qkv_dx": (169844970, 149911466),
    "qkv_dw": (275875925, 19459712),
    "logits_fwd": (903636736, 8327181312),
    "lm_dx": (6781332480, 194534400),
    "lm_dw": (5208344064, 97285632),
}
GEMM_LAUNCHES_B64 = 12 * 12 + 3


def gemm_dram_bytes_per_launch_b64() -> float:
    """Mean DRAM bytes per GEMM launch of the batch-64 step (the roofline's
    `traffic`), from the per-shape captures above."""
    total = 0
    for k, (r, w) in GEMM_DRAM_BY_SHAPE.items():
        total += (1 if k in ("logits_fwd", "lm_dx", "lm_dw") else 12) * (r + w)
    return total / GEMM_LAUNCHES_B64


def gemm_algorithmic_bytes(tokens: int):
    """(bytes, launches) of the fused bf16 step's GEMMs: every operand read
    once and every output written once (bf16 activations, fp32 branch
    outputs / input gradients / weight gradients, fp32 logits)."""
    D, H, V, L = C5["dim"], C5["hidden"], C5["vocabSize"], C5["nLayers"]
    qkv, qD, N = (C5["nHeads"] + 2 * C5["nKvHeads"]) * 64, C5["nHeads"] * 64, tokens
    b, f = 2, 4
    per_layer = [
        N * D * b + qkv * D * b + N * qkv * b,            # qkv (RoPE epilogue)
        N * qD * b + D * qD * b + N * D * f,              # wo -> fp32 branch
        N * D * b + 2 * H * D * b + N * 2 * H * b,        # gate | up
        N * H * b + D * H * b + N * D * f,                # down -> fp32 branch
        N * D * b + D * H * b + N * H * b,                # down dX
        N * D * b + N * H * b + D * H * f,                # down dW
        N * 2 * H * b + 2 * H * D * b + N * D * f,        # gate|up dX
        N * 2 * H * b + N * D * b + 2 * H * D * f,        # gate|up dW
        N * D * b + D * qD * b + N * qD * b,              # wo dX
        N * D * b + N * qD * b + D * qD * f,              # wo dW
        N * qkv * b + qkv * D * b + N * D * f,            # qkv dX
        N * qkv * b + N * D * b + qkv * D * f,            # qkv dW
    ]
    head = [N * D * b + V * D * b + N * V * f,            # logits (fp32)
            N * V * b + V * D * b + N * D * f,            # LM-head dX
            N * V * b + N * D * b + V * D * f]            # LM-head dW
    return L * sum(per_layer) + sum(head), 12 * L + 3
MATMUL_PARAMS = 100_073_472
FLOP_PER_TOKEN = 6 * MATMUL_PARAMS + 12 * 3 * 2 * 768 * 1024   # 657.06 MFLOP (fwd + bwd)
METRIC = "train tokens/s fwd+bwd+Adam (125M Llama-style, ctx 1024, global batch 64)"


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p, "measured"
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []
        self.t = None
        self.mid_thread = None
        self.mid_lines = []

    def start(self):
        """Start sampling every 100 ms; returns once the sampler produces
        output, with that pre-region sample discarded."""
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            t0 = time.time()
            while not self.lines and time.time() - t0 < 3.0:
                time.sleep(0.01)
            self.lines.clear()
        except Exception:
            self.proc = None

    def mid(self):
        """One extra query while the GPU works through the steps just
        enqueued, so a region shorter than the sampling period still has a
        sample taken under load."""
        self.mid_lines = []

        def run():
            self.mid_lines = self._one_shot()

        self.mid_thread = threading.Thread(target=run, daemon=True)
        self.mid_thread.start()

    def _one_shot(self):
        try:
            r = subprocess.run(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.Q}",
                                "--format=csv,noheader,nounits"], capture_output=True, text=True,
                               timeout=5)
            return [ln.strip() for ln in r.stdout.splitlines() if ln.strip()]
        except Exception:
            return []

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        end = []
        if self.mid_thread is not None:
            self.mid_thread.join(timeout=6)
            end = self.mid_lines
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        if self.t:
            self.t.join(timeout=2)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines + end:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def cpu_baseline(threads: int, tokens: int = 16):
    """The CPU oracle on a bounded sample of the same workload: one sequence
    of `tokens` tokens through the full config-5 model, forward + backward +
    Adam over all 100M parameters.  Returns tokens/s."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import numpy as np
    import oracle as O
    O.set_threads(threads)
    cfg = O.Config(**C5)
    P = O.init_weights(cfg, SEED)
    ids = O.RNG(SEED).ints(tokens + 1, C5["vocabSize"])
    G = np.zeros_like(P)
    m, v = np.zeros_like(P), np.zeros_like(P)
    t0 = time.perf_counter()
    O.model_step(cfg, P, ids[:-1], ids[1:], 1, tokens, G)
    O.adam_step(P, G, m, v, 1, lr=LR)
    dt = time.perf_counter() - t0
    return tokens / dt, dt


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    toks = 16
    for _ in range(args.warmup):
        cpu_baseline(threads, toks)
    vals = [cpu_baseline(threads, toks) for _ in range(args.steps)]
    tps = sum(v[0] for v in vals) / len(vals)
    sec = sum(v[1] for v in vals) / len(vals)
    line = {
        "impl": "reference", "metric": METRIC, "value": tps, "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": sec * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "c5-125m-train-step", "model": "llama-125m (forge-llm TrainableTransformer)",
                   "global_batch": GLOBAL_BATCH, "seq_len": SEQ, "parallelism": "none (host CPU)"},
        "cpu_baseline": {"value": tps, "unit": "tokens/s", "cores": threads, "kind": "port",
                         "sample": f"1 sequence x {toks} tokens of the config-5 model, fwd+bwd+Adam "
                                   "over all 100M params; the reference is JavaScript and this box "
                                   "has no JS runtime, so its C restatement (oracle/) runs"},
        "e2e": {"value": tps, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "same_config": False,
        "note": (f"tokens/s of a bounded sample (1 sequence x {toks} tokens, fwd+bwd+Adam over all 100M "
                 f"parameters, {threads} host threads) standing in for the 64 x 1024-token step, whose "
                 "CPU run would take hours; at 16 tokens the per-token attention work is far smaller "
                 "than at 1024, and the reference's own path is single-threaded JavaScript (the GPU "
                 "arm's cpu_baseline is the 1-thread figure)"),
    }
    print(json.dumps(line), flush=True)


def run_micro_gemm(args):
    """One tcgen05 contraction of the train step, timed alone (profiling aid):
    `--micro gemm --shape M,N,K --op fwd|dx|dw`.  Prints TFLOP/s."""
    import torch
    import ctypes
    import forgellm as F
    from forgellm import autograd as AD
    from forgellm._lib import GemmOut, OUT_BF16, OUT_F32, call
    F.set_precision("bf16")
    M, N, K = (int(x) for x in args.shape.split(","))
    op = {"fwd": 0, "dx": 1, "dw": 2}[args.op]
    g = torch.Generator(device="cuda").manual_seed(0)
    na = M * K if op != 2 else K * M
    nb = N * K if op == 0 else K * N
    A = torch.randn(na, device="cuda", generator=g).to(torch.bfloat16)
    Bm = torch.randn(nb, device="cuda", generator=g).to(torch.bfloat16)
    bf16_out = args.out == "bf16"
    C = torch.empty(M * N, device="cuda", dtype=torch.bfloat16 if bf16_out else torch.float32)
    o = GemmOut(OUT_BF16 if bf16_out else OUT_F32, C.data_ptr(), 0, None, 0, 0, 0, 0.0)
    h = AD.ctx().handle

    def run():
        call("fcu_gemm_bf16", h, op, A.data_ptr(), Bm.data_ptr(), M, N, K, ctypes.byref(o))

    for _ in range(args.warmup):
        run()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        run()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    tf = 2.0 * M * N * K / (ms / 1e3) / 1e12
    pk, kind = peaks()
    print(json.dumps({"micro": "gemm_bf16_tc", "op": args.op, "M": M, "N": N, "K": K, "out": args.out,
                      "ms": ms, "tflops": tf, "frac_of_burst_peak": tf / pk["bf16_tflops"],
                      "peak_kind": kind}), flush=True)


def _time_ms(fn, steps, warmup):
    """Mean CUDA-event milliseconds of fn() over `steps` calls after `warmup`."""
    import torch
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


def run_config(args):
    """The operator configs C1-C4 of the hot path, each on its seeded inputs
    through the public API, one JSON line each (`--config c1|c2|c3|c4`)."""
    import torch
    import forgellm as F
    from forgellm import autograd as AD
    from forgellm._lib import call
    F.set_precision(args.precision)
    pk, kind = peaks()
    dev = "cuda"
    out = {"config": args.config, "precision": args.precision, "data": "synthetic (forge-llm RNG)"}
    if args.config == "c2":                      # matmulT fwd + dX + dW, 4096 x 2048 -> 8192
        M, K, N = 4096, 2048, 8192
        rng = F.RNG(2)
        X = F.param(torch.from_numpy(rng.normals(M * K)).to(dev))
        W = F.param(torch.from_numpy(rng.normals(N * K)).to(dev))
        g = torch.from_numpy(rng.normals(M * N)).to(dev)

        def step():
            F.resetTape()
            X.grad, W.grad = None, None
            Y = F.matmulT(X, W, M, K, N)
            Y.grad = g
            Y._b(Y.grad)

        ms = _time_ms(step, args.steps, args.warmup)
        fl = 3 * 2.0 * M * N * K
        tf = fl / (ms / 1e3) / 1e12
        out.update(metric="matmulT fwd+bwd TFLOP/s", value=tf, unit="TFLOP/s", ms=ms,
                   roofline={"bound": "tensor", "achieved": tf, "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                             "frac": tf / pk["bf16_tflops"], "peak_kind": f"bf16 dense burst ({kind})",
                             "note": "op-level path: fp32 operands converted to bf16 inside the timed call"})
    elif args.config == "c3":                    # crossEntropyMean fwd + bwd, 8192 x 32000
        T, V = 8192, 32000
        rng = F.RNG(3)
        logits = F.param(torch.from_numpy(rng.normals(T * V, 2.0)).to(dev))
        targets = torch.from_numpy(rng.ints(T, V)).to(dev)

        def step():
            F.resetTape()
            logits.grad = None
            F.backward(F.crossEntropyMean(logits, targets, T, V))

        ms = _time_ms(step, args.steps, args.warmup)
        gb = (2.0 * T * V * 4 + T * 4) / 1e9
        bw = gb / (ms / 1e3)
        out.update(metric="crossEntropyMean fwd+bwd GB/s", value=bw, unit="GB/s", ms=ms,
                   roofline={"bound": "hbm", "achieved": bw, "peak": pk["hbm_gbs"], "unit": "GB/s",
                             "frac": bw / pk["hbm_gbs"], "traffic_algorithmic_gb": gb, "peak_kind": kind})
    elif args.config == "c4":                    # causal GQA attention with RoPE, fused-path kernels
        B, T, nH, nKV, dH = 8, 2048, 32, 8, 64
        W = (nH + 2 * nKV) * dH
        rng = F.RNG(4)
        qkv = torch.from_numpy(rng.normals(B * T * W)).to(dev).to(torch.bfloat16)
        dO = torch.from_numpy(rng.normals(B * T * nH * dH)).to(dev).to(torch.bfloat16)
        O = torch.empty(B * T * nH * dH, device=dev, dtype=torch.bfloat16)
        lse = torch.empty(B * nH * T, device=dev)
        dqkv = torch.empty_like(qkv)
        h = AD.ctx().handle

        def step():
            call("fcu_attn_fwd_bf16", h, qkv.data_ptr(), W, B, T, nH, nKV, dH, O.data_ptr(), lse.data_ptr())
            call("fcu_attn_bwd_bf16", h, dO.data_ptr(), qkv.data_ptr(), W, O.data_ptr(), lse.data_ptr(),
                 B, T, nH, nKV, dH, 10000.0, dqkv.data_ptr())

        ms = _time_ms(step, args.steps, args.warmup)
        fl = 3 * 2 * 2.0 * B * nH * (T * T / 2) * dH
        tf = fl / (ms / 1e3) / 1e12
        out.update(metric="causalAttn fwd+bwd TFLOP/s", value=tf, unit="TFLOP/s", ms=ms,
                   roofline={"bound": "tensor", "achieved": tf, "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                             "frac": tf / pk["bf16_tflops"], "peak_kind": f"bf16 dense burst ({kind})",
                             "note": "algorithmic FLOPs (fwd 4, bwd 8 x B*H*T^2/2*d), recompute not counted"})
    else:                                        # c1: the tiny char-LM train step
        cfg = F.Config(vocabSize=64, dim=64, nLayers=2, nHeads=4, nKvHeads=4, hidden=176)
        m = F.TrainableTransformer(cfg, seed=1)
        opt = F.Adam(m.paramList, lr=3e-3)
        ids = F.RNG(1).ints(65, 64)
        inp, tgt = ids[:64], ids[1:65]

        def step():
            F.resetTape()
            m.zeroGrad()
            m.backward(m.loss(inp, tgt))
            opt.step()

        ms = _time_ms(step, args.steps, args.warmup)
        out.update(metric="tiny train step (launch-latency bound)", value=ms * 1e3, unit="us/step",
                   higher_is_better=False, tokens_per_s=64 / (ms / 1e3), ms=ms, mode="eager")
        if m._use_fused():                       # the same step replayed as one CUDA graph
            from forgellm.graph import CapturedStep
            mg = F.TrainableTransformer(cfg, seed=1)
            cs = CapturedStep(mg, F.Adam(mg.paramList, lr=3e-3), 1, 64)
            batch = torch.from_numpy(ids.reshape(1, 65)).to(dev)
            gms = _time_ms(lambda: cs(batch), args.steps, args.warmup)
            out.update(value=gms * 1e3, tokens_per_s=64 / (gms / 1e3), ms=gms, mode="cuda graph",
                       eager_us_per_step=ms * 1e3, launches_per_step=cs.launches_per_step)
            cs.graph.reset()
    print(json.dumps(out), flush=True)


def run_decode(args):
    """The inference-side kernels (`--config decode`), one JSON line each:
    QuantLinear matvec (fcu_quant_matvec) per GGML format on a weight larger
    than L2, decode attention (fcu_attn_decode) over a batch of long KV
    caches, and one decode step of the config-5 model with Q4_K matrices for
    1 and 32 sequences.  Weight bytes are random GGML blocks with finite f16
    scales (their values do not change the work); the cache and vectors are
    N(0, 1)."""
    import math

    import torch
    import forgellm as F
    from forgellm import autograd as AD
    from forgellm import infer as I
    from forgellm._lib import call
    pk, kind = peaks()
    h = AD.ctx().handle
    dev = "cuda"
    gen = torch.Generator(device=dev).manual_seed(7)

    def ggml_bytes(t, N, K):
        rb = I.row_bytes(t, K)
        if t == I.F32:
            return torch.randn(N * K, device=dev, generator=gen).view(torch.uint8)
        if t == I.F16:
            return torch.randn(N * K, device=dev, generator=gen).half().view(torch.uint8)
        b = torch.randint(0, 256, (N * rb,), dtype=torch.uint8, device=dev, generator=gen)
        bb = {I.Q4_0: 18, I.Q5_0: 22, I.Q8_0: 34, I.Q4_K: 144, I.Q5_K: 176, I.Q6_K: 210}[t]
        blk = b.view(-1, bb)
        d = torch.full((blk.shape[0],), 0.01, device=dev).half().view(torch.uint8).view(-1, 2)
        if t == I.Q6_K:
            blk[:, 208:210] = d
        else:
            blk[:, 0:2] = d
            if t in (I.Q4_K, I.Q5_K):
                blk[:, 2:4] = d
        return b

    K = 4096
    for t, name in ((I.Q4_K, "Q4_K"), (I.Q5_K, "Q5_K"), (I.Q6_K, "Q6_K"), (I.Q8_0, "Q8_0"), (I.F16, "F16"),
                    (I.F32, "F32")):
        rb = I.row_bytes(t, K)
        N = max(4096, (512 << 20) // rb)       # ~512 MiB of weights: well beyond the 126 MB L2
        W = ggml_bytes(t, N, K)
        for M in (1, 8):
            X = torch.randn(M, K, device=dev, generator=gen)
            Y = torch.empty(M, N, device=dev)
            ms = _time_ms(lambda: call("fcu_quant_matvec", h, t, W.data_ptr(), N, K, X.data_ptr(), M, Y.data_ptr()),
                          args.steps, args.warmup)
            gb = (N * rb + M * K * 4 + M * N * 4) / 1e9
            bw = gb / (ms / 1e3)
            print(json.dumps({"config": "decode", "kernel": "fcu_quant_matvec", "type": name, "N": N, "K": K, "M": M,
                              "metric": "QuantLinear.forward GB/s", "value": bw, "unit": "GB/s", "ms": ms,
                              "roofline": {"bound": "hbm", "achieved": bw, "peak": pk["hbm_gbs"], "unit": "GB/s",
                                           "frac": bw / pk["hbm_gbs"], "peak_kind": kind,
                                           "algorithmic_gb": gb},
                              "data": "synthetic GGML blocks"}), flush=True)
        del W
        torch.cuda.empty_cache()
    # decode attention: B sequences of n cached positions each
    for B, n, nH, nKV, dH in ((64, 4096, 32, 8, 128), (32, 1024, 12, 4, 64), (1, 1024, 12, 4, 64)):
        kvDim = nKV * dH
        kc = torch.randn(B * n, kvDim, device=dev, generator=gen)
        vc = torch.randn(B * n, kvDim, device=dev, generator=gen)
        ld = (nH + 2 * nKV) * dH
        q = torch.randn(B, ld, device=dev, generator=gen)
        out = torch.empty(B, nH * dH, device=dev)
        lens = torch.full((B,), n, dtype=torch.int32, device=dev)
        ms = _time_ms(lambda: call("fcu_attn_decode", h, q.data_ptr(), ld, kc.data_ptr(), vc.data_ptr(), kvDim, None,
                                   1, n, lens.data_ptr(), B, nH, nKV, dH, 1 / math.sqrt(dH), out.data_ptr()),
                      args.steps, args.warmup)
        gb = (2.0 * B * n * kvDim * 4 + B * ld * 4 + B * nH * dH * 4) / 1e9
        bw = gb / (ms / 1e3)
        print(json.dumps({"config": "decode", "kernel": "fcu_attn_decode", "B": B, "n": n, "nH": nH, "nKV": nKV,
                          "dH": dH, "metric": "decode attention GB/s", "value": bw, "unit": "GB/s", "ms": ms,
                          "roofline": {"bound": "hbm", "achieved": bw, "peak": pk["hbm_gbs"], "unit": "GB/s",
                                       "frac": bw / pk["hbm_gbs"], "peak_kind": kind, "algorithmic_gb": gb},
                          "l2": "cache > L2" if gb > 0.126 else "cache fits L2 (latency-bound size)"}),
              flush=True)
        del kc, vc
        torch.cuda.empty_cache()
    # one decode step of the config-5 model (Q4_K matrices, Q8_0 embedding / LM head)
    cfg = F.Config(**C5, maxSeq=1024)
    w = {"tok_emb": I.QuantLinear(I.Q8_0, ggml_bytes(I.Q8_0, cfg.vocabSize, cfg.dim), cfg.vocabSize, cfg.dim),
         "ln_f": torch.ones(cfg.dim)}
    for l in range(cfg.nLayers):
        shapes = {"wqkv": (cfg.qkvOut, cfg.dim), "wo": (cfg.dim, cfg.dim), "ffn_gate": (cfg.hidden, cfg.dim),
                  "ffn_up": (cfg.hidden, cfg.dim), "ffn_down": (cfg.dim, cfg.hidden)}
        L = {k: I.QuantLinear(I.Q4_K, ggml_bytes(I.Q4_K, n_, k_), n_, k_) for k, (n_, k_) in shapes.items()}
        L.update(ln1=torch.ones(cfg.dim), ln2=torch.ones(cfg.dim))
        w[f"layer.{l}"] = L
    tr = F.Transformer(cfg).loadWeights(w)
    wbytes = tr.tokEmb.bytesSize() + sum(q.bytesSize() for L in tr.layers for k, q in L.items()
                                         if isinstance(q, I.QuantLinear))
    for graph in (False, True):
        for B in (1, 32):
            cache = F.KVCache(cfg.nLayers, cfg.maxSeq, cfg.kvDim, batch=B)
            toks = [int(x) for x in F.RNG(5).ints(B, cfg.vocabSize)]
            state = {"pos": 0}

            def step():
                p = state["pos"] % 512 + 256          # positions 256..767: a half-filled cache
                tr.forwardBatch(toks, [p] * B, cache, graph=graph)
                state["pos"] += 1

            for p in range(256):                      # fill the first 256 positions
                tr.forwardBatch(toks, [p] * B, cache, graph=graph)
            ms = _time_ms(step, args.steps, args.warmup)
            note = ("CUDA graph replay of the step (tokens and positions copied in first)" if graph else
                    "eager host loop: 12 layers x 11 launches + embed / head per step")
            print(json.dumps({"config": "decode", "kernel": "Transformer.forwardBatch (config-5 model, Q4_K)",
                              "B": B, "graph": graph, "metric": "decode tokens/s", "value": B / (ms / 1e3),
                              "unit": "tokens/s", "ms_per_step": ms, "weight_bytes": wbytes,
                              "weights_gb_per_s": wbytes / 1e9 / (ms / 1e3), "note": note}), flush=True)


def profile_collectives(F, AD, model, opt, dp, batch):
    """Every collective and join of one op-by-op step (`--comm-profile`),
    timed with CUDA events on the communicator's and the context's streams:
    per bucket its size, how long it queued behind earlier collectives after
    its gradients were ready, and its duration; for each join how long the
    compute stream waited (the exposed communication).  This rank's view."""
    import torch

    def eager_step():
        F.resetTape()
        model.zeroGrad()
        loss = model.lossBatch(batch)
        AD.backward(loss)
        dp.finish()
        opt.step()

    eager_step()
    torch.cuda.synchronize()
    dp.comm.profile(256)
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s0.record()
    eager_step()
    s1.record()
    torch.cuda.synchronize()
    recs = dp.comm.profile_read()
    dp.comm.profile(0)
    colls = [r for r in recs if r["kind"] != "join"]
    joins = [r for r in recs if r["kind"] == "join"]
    return {
        "step_ms": s0.elapsed_time(s1),
        "collectives": [{"kind": r["kind"], "mbytes": round(r["bytes"] / 1e6, 3),
                         "ready_ms": round(r["ready"], 3), "queued_ms": round(r["start"] - r["ready"], 3),
                         "ms": round(r["end"] - r["start"], 3),
                         "gbps": round(r["bytes"] / max(r["end"] - r["start"], 1e-6) / 1e6, 1)}
                        for r in colls],
        "joins_waited_ms": [round(r["end"] - r["ready"], 3) for r in joins],
        "exposed_ms": round(sum(r["end"] - r["ready"] for r in joins), 3),
        "measured": "CUDA events around each NCCL call (communicator stream) and join (compute stream), "
                    "one op-by-op step after one untimed one; times from the first collective's ready time",
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--precision", default=os.environ.get("FORGECU_PRECISION", "bf16"),
                    choices=["fp32", "fp32tc", "bf16"],
                    help="bf16: tensor-core fused step (default); fp32: CUDA-core parity mode; "
                         "fp32tc: parity mode with matmulT on the tensor cores")
    ap.add_argument("--batch", type=int, default=GLOBAL_BATCH)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--eager", action="store_true",
                    help="launch the step op by op instead of replaying its CUDA graph")
    ap.add_argument("--micro", choices=["gemm"], help="time one kernel alone (profiling)")
    ap.add_argument("--zero", action="store_true",
                    help="N > 1: shard Adam's state and update over the ranks (ZeRO-1)")
    ap.add_argument("--comm-profile", action="store_true",
                    help="N > 1: after the timed regions, time every collective of one op-by-op "
                         "step with CUDA events and add them to the line (comm_profile)")
    ap.add_argument("--config", choices=["c1", "c2", "c3", "c4", "decode"],
                    help="time one of the operator configs instead of the C5 train step")
    ap.add_argument("--shape", default="8192,2048,768")
    ap.add_argument("--op", default="fwd", choices=["fwd", "dx", "dw"])
    ap.add_argument("--out", default="f32", choices=["f32", "bf16"], help="--micro gemm output type")
    args = ap.parse_args()
    if args.config == "decode":
        return run_decode(args)
    if args.config:
        return run_config(args)
    if args.micro == "gemm":
        run_micro_gemm(args)
        return
    if args.impl == "reference":
        run_reference(args)
        return

    import numpy as np
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    import forgellm as F
    from forgellm import autograd as AD
    from forgellm import tensor as TS
    from forgellm._lib import lib
    from forgellm.dist import DataParallel, shard_rows
    F.set_precision(args.precision)

    cfg = F.Config(**C5)
    model = F.TrainableTransformer(cfg, seed=SEED)
    if args.zero and world > 1:                 # ZeRO-1: sharded Adam state and update
        from forgellm.dist import ShardedAdam
        dp = DataParallel(model, shard=True)
        opt = ShardedAdam(model, dp, lr=LR)
    else:
        opt = F.Adam(model.paramList, lr=LR)
        dp = DataParallel(model) if world > 1 else None
    toks = F.RNG(SEED).ints(args.batch * (SEQ + 1), C5["vocabSize"]).reshape(args.batch, SEQ + 1)
    local_rows = toks if world == 1 else shard_rows(torch.from_numpy(toks), rank, world).numpy()
    batch_dev = torch.from_numpy(np.ascontiguousarray(local_rows)).cuda()
    batch_host = torch.from_numpy(np.ascontiguousarray(local_rows)).pin_memory()

    use_graph = args.precision == "bf16" and not args.eager
    if use_graph:
        # The whole step (fused fwd + bwd, all-reduces, Adam) as one CUDA graph.
        from forgellm.graph import CapturedStep
        cs = CapturedStep(model, opt, local_rows.shape[0], SEQ, dp=dp)

        def step(batch):
            return cs(batch)
    else:
        cs = None

        def step(batch):
            if batch.device.type != "cuda":
                batch = batch.to("cuda", non_blocking=True)
            F.resetTape()
            model.zeroGrad()
            loss = model.lossBatch(batch)
            AD.backward(loss)
            if dp is not None:
                dp.finish()
            opt.step()
            return loss.data

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    # ---------------- warm-up
    for _ in range(args.warmup):
        step(batch_dev)
    barrier()

    # ---------------- timed region 1: inputs resident in HBM
    sampler = ClockSampler(local)
    sampler.start()
    TS.GEMM_TIMER = None if use_graph else []
    launches0 = lib().fcu_launch_count()
    stream = torch.cuda.current_stream()
    barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(args.steps):
        step(batch_dev)
    ev1.record(stream)
    sampler.mid()
    torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1)
    clocks = sampler.stop()
    if use_graph:
        launches = cs.launches_per_step * args.steps     # kernel nodes replayed
        gemm_ms = gemm_flops = 0.0                       # measured after the e2e region
    else:
        launches = lib().fcu_launch_count() - launches0
        gemm = TS.GEMM_TIMER
        TS.GEMM_TIMER = None
        gemm_ms = sum(a.elapsed_time(b) for _, a, b in gemm)
        gemm_flops = sum(f for f, _, _ in gemm)
    t = torch.tensor([ms, gemm_ms], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t[0])
    tokens_per_step = args.batch * SEQ
    value = tokens_per_step * args.steps / (ms / 1e3)

    # ---------------- timed region 2: end to end through the public API
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        loss = step(batch_host)                  # host -> device copy of the batch inside
        _ = float(loss[0].item())                # device -> host read of the loss
    e1.record(stream)
    torch.cuda.synchronize()
    te = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_value = tokens_per_step * args.steps / (float(te[0]) / 1e3)

    comm_profile = None
    if args.comm_profile and dp is not None and dp.comm is not None:
        comm_profile = profile_collectives(F, AD, model, opt, dp, batch_dev)

    gemm_where = "CUDA events around every matmulT in the timed region"
    gemm_steps = args.steps
    if use_graph:
        # Kernels inside a replayed graph carry no host timing events, so the
        # GEMMs are timed over two op-by-op launches of the same step (the same
        # kernels on the same stream) right after the timed regions.
        TS.GEMM_TIMER = []
        for _ in range(2):
            F.resetTape()
            model.zeroGrad()
            loss = model.lossBatch(batch_dev)
            AD.backward(loss)
            if dp is not None:
                dp.finish()
            opt.step()
        torch.cuda.synchronize()
        gemm, TS.GEMM_TIMER = TS.GEMM_TIMER, None
        gemm_ms = sum(a.elapsed_time(b) for _, a, b in gemm)
        gemm_flops = sum(f for f, _, _ in gemm)
        gemm_steps = 2
        gemm_where = "CUDA events around every GEMM of 2 op-by-op launches of the timed step"

    if rank == 0:
        pk, pk_kind = peaks()
        achieved = gemm_flops / (gemm_ms / 1e3) / 1e12 if gemm_ms > 0 else 0.0
        gb, gl = gemm_algorithmic_bytes(args.batch * SEQ)
        alg_bytes = gb / gl if args.precision == "bf16" else None
        traffic = (gemm_dram_bytes_per_launch_b64()
                   if args.precision == "bf16" and args.batch == GLOBAL_BATCH and world == 1 else None)
        peak = pk["bf16_tflops_sustained"]
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": {"fp32": "f32", "fp32tc": "f32 (matmulT as 3-way bf16 split on tcgen05)",
                      "bf16": "bf16 operands, f32 accumulate/master"}[args.precision],
            "data": "synthetic (RNG(5) tokens, initWeights seed 5)",
            "config": {"workload": "c5-125m-train-step",
                       "model": "llama-125m (forge-llm TrainableTransformer: V32000 D768 L12 H12/4 F2048)",
                       "global_batch": args.batch, "seq_len": SEQ,
                       "parallelism": f"dp{world}" + ("+zero1" if args.zero and world > 1 else ""),
                       "precision": args.precision, "l2": "working set >> L2 (GBs of activations)"},
            "e2e": {"value": e2e_value, "unit": "tokens/s",
                    "h2d_bytes_per_step": int(args.batch * (SEQ + 1) * 4),
                    "d2h_bytes_per_step": 4 * world},
            "gpu_launches": int(launches),
            "roofline": {"kernel": "gemm_bf16_tc_kernel: every matmulT fwd / dX / dW contraction of the step",
                         "bound": "tensor",
                         "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak if peak else None,
                         "peak_kind": f"bf16 dense sustained ({pk_kind})",
                         "traffic": traffic,
                         "traffic_unit": "DRAM bytes per GEMM launch (single-pass ncu capture of the step's 147 GEMM launches, mean per launch)",
                         "algorithmic_bytes_per_launch": alg_bytes,
                         "gemm_share_of_step": (gemm_ms / gemm_steps) / (ms / args.steps) if ms else None,
                         "measured": gemm_where,
                         "model_tflops": FLOP_PER_TOKEN * value / 1e12},
            "clocks": clocks,
        }
        if comm_profile is not None:
            line["comm_profile"] = comm_profile
        if world == 1 and not args.no_cpu_baseline:
            tps, sec = cpu_baseline(1)
            line["cpu_baseline"] = {"value": tps, "unit": "tokens/s", "cores": 1, "kind": "port",
                                    "sample": "1 sequence x 16 tokens of the config-5 model, "
                                              f"fwd+bwd+Adam over all 100M params ({sec:.1f} s)"}
        print(json.dumps(line), flush=True)
    # A CUDA graph that holds NCCL calls must be released before the process
    # group is destroyed, or the exit waits on it forever.
    torch.cuda.synchronize()
    if cs is not None:
        cs.graph.reset()
        del cs
    import gc
    gc.collect()
    if dp is not None:
        dp.detach()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
