"""bench.py's reference arm (the reference's own cpu_reference.cpp through
oracle/_ref) runs on the host and prints the contract's JSON line, and the
product ops refuse CPU tensors loudly (no CPU fallback)."""

import json
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def test_reference_arm_prints_the_contract_line():
    from oracle import oracle as O

    if not O.have_ref():
        pytest.skip("oracle/_ref not built")
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference",
                        "--steps", "2", "--warmup", "3"],
                       capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads([l for l in r.stdout.splitlines() if l.startswith("{")][-1])
    assert line["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["value"] > 0 and line["unit"] == "GB/s"
    assert line["cpu_baseline"]["kind"] == "reference" and line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["value"] == line["value"]
    assert "workload" in line["config"]


def test_ops_refuse_cpu_tensors():
    torch = pytest.importorskip("torch")
    from decodebench_b200 import ops

    x = torch.zeros(1, 64, dtype=torch.float16)
    W = torch.zeros(32, 64, dtype=torch.float16)
    g = torch.ones(64, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.rmsnorm_gemv(x, g, W)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.gateup_swiglu(x, W, W)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.gemv(x, W)
    q = torch.zeros(1, 2, 128, dtype=torch.float16)
    kv = torch.zeros(1, 2, 64, 128, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.flashdecode(q, kv, kv)


def _bench_module():
    import importlib.util

    spec = importlib.util.spec_from_file_location("dbk_bench", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_step_graphs_cover_exactly_k_steps():
    """The timed region replays graphs covering exactly K steps: one graph of K
    steps up to the cap, then cap-sized graphs plus one remainder graph."""
    bench = _bench_module()
    sg = bench.StepGraphs.__new__(bench.StepGraphs)
    sg.cap = 4096
    for k in (1, 5, 20, 4096, 4097, 10000):
        chunks = sg._chunks(k)
        assert sum(chunks) == k
        assert all(0 < c <= 4096 for c in chunks)
        assert len(chunks) == (k + 4095) // 4096
    assert sg._chunks(20) == [20]


def test_cpu_sampler_runs_at_least_the_minimum_steps():
    """Both CPU arms use the same time-budgeted sampler: warm-up, then at least
    min_steps measured steps, however short the budget."""
    bench = _bench_module()

    class Fake:
        calls = 0

        def cpu_step(self, threads):
            Fake.calls += 1

    med, n = bench.cpu_time(Fake(), 1, budget_s=0.0, warmup=1, min_steps=10)
    assert n == 10 and med >= 0.0
    assert Fake.calls >= 11
