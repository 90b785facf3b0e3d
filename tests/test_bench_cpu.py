"""bench.py's contract pieces that need no GPU: the algorithmic work
constants of config 5 and the JSON line of the reference (CPU) arm."""
import importlib.util
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bench():
    spec = importlib.util.spec_from_file_location("bench_mod", os.path.join(ROOT, "bench.py"))
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


def test_config5_algorithmic_work():
    b = _bench()
    # 6 x 100,073,472 matmul parameters + 12 layers x 3 x 2 x 768 x 1024 attention, per token
    assert b.FLOP_PER_TOKEN == 6 * 100_073_472 + 12 * 3 * 2 * 768 * 1024
    # every GEMM operand read once and every output written once, one batch-64 step
    gb, launches = b.gemm_algorithmic_bytes(64 * 1024)
    assert launches == 147
    assert gb == 75_962_515_456
    # the per-launch traffic of the per-shape ncu captures is above the
    # algorithmic bytes (operand re-reads and split-K partials of the weight
    # gradients) and covers every distinct GEMM of the step
    assert b.GEMM_LAUNCHES_B64 == launches
    assert len(b.GEMM_DRAM_BY_SHAPE) == 15
    assert b.gemm_dram_bytes_per_launch_b64() > gb / launches


def test_reference_arm_prints_one_contract_line():
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                          "--steps", "1", "--warmup", "1"], capture_output=True, text=True, timeout=600,
                         cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
              "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["impl"] == "reference" and d["value"] > 0 and d["higher_is_better"] is True
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert d["cpu_baseline"]["kind"] in ("port", "reference") and d["cpu_baseline"]["cores"] >= 1
    assert d["config"]["workload"] == "c5-125m-train-step"
