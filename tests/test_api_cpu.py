"""Behaviour of the kept DecodeBench API on the CPU, restating the reference's
tests (tests/test_bytes_model.py, test_verdict.py, test_report.py,
test_stats.py, test_sequence_bindings.py, test_timing_inputs.py,
test_cost_model.py) against decodebench_b200."""

import csv
import math

import numpy as np
import pytest

from decodebench_b200 import costs
from decodebench_b200.bytes_model import StageTrace, eliminable_bytes, total_bytes
from decodebench_b200.report import Report
from decodebench_b200.sequence import Sequence
from decodebench_b200.stats import bootstrap_diff_ci, summarize
from decodebench_b200.timing import n_weight_replicas, time_callable
from decodebench_b200.verdict import compute_verdict

F1_TRACES = [StageTrace("rmsnorm", [8192, 8192], 8192),
             StageTrace("gemv", [33554432, 8192], 8192, is_final=True)]


# ---------------------------------------------------------------- bytes model
def test_bytes_golden_f1():
    assert total_bytes(F1_TRACES) == 33595392
    assert eliminable_bytes(F1_TRACES) == 16384


def test_bytes_single_final_and_fanout():
    assert total_bytes([F1_TRACES[1]]) == 33570816 and eliminable_bytes([F1_TRACES[1]]) == 0
    tr = [StageTrace("producer", [64], 128, consumers=2),
          StageTrace("final", [128, 128], 32, is_final=True, consumers=0)]
    assert total_bytes(tr) == 480 and eliminable_bytes(tr) == 384


def test_bytes_invalid():
    with pytest.raises(ValueError, match="non-negative"):
        StageTrace("bad", [-1], 1)
    with pytest.raises(ValueError, match="consumers"):
        StageTrace("bad", [], 1, consumers=-1)
    with pytest.raises(ValueError, match="at least one consumer"):
        StageTrace("dead", [], 1, consumers=0)


# ---------------------------------------------------------------- cost model goldens
@pytest.mark.parametrize("d,goldens", [
    (4096, {"F1": (33595392, 16384, 0.000488, "low"), "F2": (180481536, 88064, 0.000488, "low"),
            "F4": (17317888, 524288, 0.030274, "material")}),
    (2048, {"F1": (8409088, 8192, 0.000974, "low"), "F2": (67198976, 65536, 0.000975, "low"),
            "F4": (8658944, 262144, 0.030274, "material")}),
])
def test_cost_model_goldens(d, goldens):
    for c in costs.fusion_costs(d=d, b=1, threshold=0.01):
        tot, el, ratio, kind = goldens[c.name]
        assert (c.total, c.eliminable, round(c.ratio, 6)) == (tot, el, ratio)
        assert c.predicted.startswith(kind)


def test_fused_step_bytes_match_baseline_table():
    assert costs.rmsnorm_gemv_bytes(1, 4096, 4096) == 33579008
    assert costs.gateup_swiglu_bytes(1, 4096, 11008) == 180385280
    assert costs.flashdecode_bytes([4096], 32, 32) == 67125248
    assert costs.mlp_bytes(16, 8192, 28672) == 1409826816


# ---------------------------------------------------------------- verdict
def test_verdict_low_byte_opportunity():
    v = compute_verdict(20.0, 16.0, 33595392, 16384, 0.01)
    assert v.bound == "low-byte-opportunity" and v.delta_launch == 4.0
    assert abs(v.b_bytes_est - 16384 / (33595392 / 16.0)) < 1e-6
    assert v.b_ceiling == v.b_bytes_est and v.dominant == "launch"
    r = v.render()
    for s in ("CUDA Graphs eliminate 4.00 us here", "Eliminable intermediate bytes correspond to",
              "NOT a strict bound", "Verdict: LOW-BYTE-OPPORTUNITY"):
        assert s in r


def test_verdict_threshold_and_f4_regression():
    assert compute_verdict(20, 16, 1000000, 30000, byte_threshold=0.01).bound == "material-byte-opportunity"
    assert compute_verdict(20, 16, 1000000, 30000, byte_threshold=0.05).bound == "low-byte-opportunity"
    v = compute_verdict(20.0, 16.0, 17317888, 524288, 0.01)
    assert v.bound == "material-byte-opportunity" and v.dominant == "launch"
    assert "Caution: measured launch savings exceed the byte estimate" in v.render()


def test_verdict_invalid_inputs():
    with pytest.raises(ValueError, match="t_graph must be positive"):
        compute_verdict(10.0, 0.0, 100, 10)
    with pytest.raises(ValueError, match="t_fused must be finite and positive"):
        compute_verdict(10.0, 8.0, 100, 10, t_fused=-1.0)
    with pytest.raises(ValueError, match="must be finite"):
        compute_verdict(float("nan"), 8.0, 100, 10)
    with pytest.raises(ValueError, match="byte_threshold"):
        compute_verdict(10.0, 8.0, 100, 10, byte_threshold=-0.1)
    with pytest.raises(ValueError, match="ordered bounds"):
        compute_verdict(10.0, 8.0, 100, 10, delta_launch_ci=(2.0, 1.0))


def test_verdict_with_fused_and_roofline():
    v = compute_verdict(20.0, 16.0, 33595392, 16384, 0.01, t_fused=12.0,
                        fused_bytes=33579008, hbm_peak_gbs=6539.5)
    assert abs(v.residual_us - 3.9922) < 1e-3
    r = v.render()
    assert "Measured fused latency: 12.00 us" in r and "unexplained residual 3.99 us" in r
    assert abs(v.fused_gbs - 33579008 / 12.0 / 1e3) < 1e-6
    assert "of 6540 GB/s HBM peak" in r


# ---------------------------------------------------------------- report
def test_report_csv_and_verdict(tmp_path):
    rep = Report("test_f1", [20.0] * 30, [16.0] * 30, F1_TRACES, fused_us=[12.0] * 30)
    v = rep.verdict()
    assert v.bound == "low-byte-opportunity" and v.delta_launch_ci is not None and v.t_fused == 12.0
    p = tmp_path / "r.csv"
    rep.to_csv(str(p))
    rows = list(csv.reader(open(p)))
    assert rows[0] == ["name", "variant", "trial", "us_per_invocation"]
    assert len(rows) == 91
    assert rows[1] == ["test_f1", "stream", "0", "20.0"]
    assert rows[31] == ["test_f1", "graph", "0", "16.0"]
    assert rows[61] == ["test_f1", "fused", "0", "12.0"]


def test_report_capture_failure():
    rep = Report("test_fail", [20.0], [], [], graph_ok=False, graph_skip_reason="Host sync detected")
    with pytest.raises(RuntimeError, match="capture failed for 'test_fail': Host sync detected"):
        rep.verdict()


# ---------------------------------------------------------------- stats
def test_summarize():
    s = summarize([10, 12, 11, 13, 100])
    assert (s.median, s.p25, s.p75, s.iqr, s.n) == (12.0, 11.0, 13.0, 2.0, 5)
    with pytest.raises(ValueError, match="requires at least one sample"):
        summarize([])
    with pytest.raises(ValueError, match="finite"):
        summarize([1.0, np.nan])
    with pytest.raises(ValueError, match="one-dimensional"):
        summarize([[1.0, 2.0]])


def test_bootstrap():
    rng = np.random.default_rng(42)
    a, b = rng.normal(100, 2, 200), rng.normal(90, 2, 200)
    lo, hi, pt = bootstrap_diff_ci(a, b, n_resamples=1000, seed=42)
    assert 0 < lo < pt < hi
    lo2, hi2, _ = bootstrap_diff_ci(a, rng.normal(100, 2, 200), n_resamples=1000, seed=42)
    assert lo2 < 0 < hi2
    for kw, msg in (({"a": [], "b": [1.0]}, "requires non-empty samples"),
                    ({"a": [np.inf], "b": [1.0]}, "finite"),
                    ({"a": [1.0], "b": [1.0], "n_resamples": 0}, "n_resamples"),
                    ({"a": [1.0], "b": [1.0], "ci": 1.0}, "ci must"),
                    ({"a": [[1.0]], "b": [1.0]}, "one-dimensional")):
        with pytest.raises(ValueError, match=msg):
            bootstrap_diff_ci(**kw)


# ---------------------------------------------------------------- sequence bindings
def test_fanin_fanout_counts():
    seq = Sequence("dag")

    @seq.stage
    def source(x):
        return x

    @seq.stage
    def left(source):
        return source

    @seq.stage
    def right(source):
        return source

    @seq.stage
    def merge(left, right):
        return left

    assert seq._dependency_consumer_counts({"x": object()}) == {"source": 2, "left": 1, "right": 1}


def test_unconsumed_and_signature_rules():
    seq = Sequence("bad")

    @seq.stage
    def first(x):
        return x

    @seq.stage
    def second(x):
        return x

    with pytest.raises(ValueError, match="first.*never consumed"):
        seq._dependency_consumer_counts({"x": object()})
    s2 = Sequence("sig")
    with pytest.raises(TypeError, match="plain positional"):
        @s2.stage
        def bad(*args):
            return args

    def same(x):
        return x

    s2.stage(same)
    with pytest.raises(ValueError, match="duplicate stage"):
        s2.stage(same)
    s3 = Sequence("missing")

    @s3.stage
    def only(y):
        return y

    with pytest.raises(KeyError, match="not found"):
        s3._dependency_consumer_counts({"x": 1})


def test_sequence_runs_on_cpu_tensors():
    """The chain machinery itself is device-agnostic (trace on CPU tensors)."""
    import torch

    seq = Sequence("cpu")

    @seq.stage
    def scale(x, g):
        return x * g

    @seq.stage
    def shift(scale):
        return scale + 1.0

    x, g = torch.ones(4, 8), torch.full((8,), 2.0)
    tr = seq.trace({"x": x, "g": g})
    assert [t.name for t in tr] == ["scale", "shift"]
    assert tr[0].reads == [128, 32] and tr[0].consumers == 1 and tr[1].is_final
    assert torch.equal(seq.run({"x": x, "g": g}), torch.full((4, 8), 3.0))


# ---------------------------------------------------------------- timing inputs
def test_replica_sizing_and_timing_validation():
    assert n_weight_replicas(1024, l2_bytes=48 * 1024 * 1024) == 8
    assert n_weight_replicas(180_000_000, l2_bytes=126 * 1024 * 1024) == 4
    with pytest.raises(ValueError, match="weight_bytes"):
        n_weight_replicas(0, l2_bytes=1024)
    with pytest.raises(ValueError, match="l2_bytes"):
        n_weight_replicas(1024, l2_bytes=-1)
    with pytest.raises(ValueError, match="trials"):
        time_callable(lambda: None, trials=0)
    with pytest.raises(ValueError, match="target_ms"):
        time_callable(lambda: None, target_ms=math.nan)
    with pytest.raises(ValueError, match="warmup"):
        time_callable(lambda: None, warmup=-1)
