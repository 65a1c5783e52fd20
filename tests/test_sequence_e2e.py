"""The Sequence / profile / graph / timing API end to end, following the
reference's tests/test_gpu_e2e.py:18-205 test by test.

The hygiene checks (fan-out counts, aliasing, non-contiguous arguments,
closure-captured tensors, replica mismatch) and the fused-output gate are
device-agnostic, so each runs on CPU tensors (always) and on CUDA tensors (gpu
marker). Capture / replay, the temporary-allocation warning, the timing sanity
check and the demo verdicts need the GPU. The demo verdicts run with the fused
arm: the sm_100a kernels of decodebench_b200.ops as the `fused=` callable."""

from __future__ import annotations

import pytest

torch = pytest.importorskip("torch")

from decodebench_b200.graph import try_capture  # noqa: E402
from decodebench_b200.sequence import Sequence  # noqa: E402
from decodebench_b200.timing import n_weight_replicas, time_callable  # noqa: E402

DEVICES = ["cpu", pytest.param("cuda", marks=pytest.mark.gpu)]


@pytest.mark.gpu
def test_n_weight_replicas():
    assert n_weight_replicas(1024, l2_bytes=48 * 1024 * 1024) >= 4
    assert n_weight_replicas(1024) >= 4          # the device's own L2 size


@pytest.mark.parametrize("device", DEVICES)
def test_sequence_trace_bytes(device):
    d = 256
    x = torch.randn(1, d, dtype=torch.float16, device=device)
    g = torch.randn(d, dtype=torch.float16, device=device)
    seq = Sequence("test_trace")

    @seq.stage
    def rmsnorm(x, g):
        return x * g

    traces = seq.trace({"x": x, "g": g})
    assert len(traces) == 1
    assert traces[0].name == "rmsnorm"
    assert traces[0].reads == [x.nbytes, g.nbytes]
    assert traces[0].write == x.nbytes


@pytest.mark.parametrize("device", DEVICES)
def test_sequence_trace_fanout_and_unsafe_tensor_forms(device):
    x = torch.randn(16, device=device)
    seq = Sequence("fanout")

    @seq.stage
    def source(x):
        return x.clone()

    @seq.stage
    def left(source):
        return source + 1

    @seq.stage
    def right(source):
        return source + 2

    @seq.stage
    def merge(left, right):
        return left + right

    traces = seq.trace({"x": x})
    assert traces[0].consumers == 2

    alias = Sequence("alias")

    @alias.stage
    def inplace(x):
        return x.add_(1)

    with pytest.raises(ValueError, match="aliases"):
        alias.trace({"x": x.clone()})

    strided = Sequence("strided")

    @strided.stage
    def copy(x):
        return x.clone()

    with pytest.raises(ValueError, match="non-contiguous"):
        strided.trace({"x": torch.ones(4, 4, device=device).t()})

    hidden_weight = torch.ones(16, device=device)
    closure = Sequence("closure")

    @closure.stage
    def hidden(x):
        return x * hidden_weight

    with pytest.raises(ValueError, match="captures tensor"):
        closure.trace({"x": x})


@pytest.mark.parametrize("device", DEVICES)
def test_replica_shape_mismatch_rejected(device):
    with pytest.raises(ValueError, match="does not match replica 0"):
        Sequence._validate_replicas([
            {"x": torch.ones(2, device=device)},
            {"x": torch.ones(3, device=device)},
        ])


@pytest.mark.parametrize("device", DEVICES)
def test_profile_fused_correctness_mismatch_raises(device):
    """The fused-output gate runs before any timing, so a wrong fused callable is
    refused on any device (reference sequence.py:308-332)."""
    d = 256
    x = torch.randn(1, d, dtype=torch.float16, device=device)
    seq = Sequence("fused_bad")

    @seq.stage
    def double(x):
        return x * 2.0

    def wrong_fused(inputs):
        return inputs["x"] * 3.0   # deliberately wrong

    with pytest.raises(ValueError, match="fused"):
        seq.profile({"x": x}, trials=3, target_ms=2.0, warmup=2, fused=wrong_fused)

    def wrong_shape(inputs):
        return torch.cat([inputs["x"], inputs["x"]])

    with pytest.raises(ValueError, match="shape"):
        seq.profile({"x": x}, trials=3, target_ms=2.0, warmup=2, fused=wrong_shape)


@pytest.mark.gpu
def test_cuda_graph_capture_and_replay():
    x = torch.randn(1, 256, dtype=torch.float16, device="cuda")
    y = torch.zeros(1, 256, dtype=torch.float16, device="cuda")

    def body():
        y.copy_(x * 2.0)

    captured = try_capture(body)
    assert captured.ok is True
    assert captured._graph is not None
    x.fill_(1.0)
    captured.replay()
    assert torch.allclose(y, torch.tensor(2.0, dtype=torch.float16, device="cuda"))


@pytest.mark.gpu
def test_cuda_graph_capture_failure():
    x = torch.tensor([1.0], device="cuda")

    def body():
        _ = x.item()            # a host synchronisation cannot be captured

    captured = try_capture(body)
    assert captured.ok is False
    assert len(captured.reason) > 0
    with pytest.raises(RuntimeError, match="cannot replay: capture failed"):
        captured.replay()
    # the failed capture left nothing behind: random numbers still work
    assert torch.randn(4, device="cuda").isfinite().all()


@pytest.mark.gpu
def test_fused_kernel_captures_and_replays():
    """One of this build's kernels inside a captured graph replays to the eager result."""
    from decodebench_b200 import ops

    gen = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn(1, 4096, generator=gen, device="cuda").half()
    g = torch.randn(4096, generator=gen, device="cuda").half()
    W = (torch.randn(4096, 4096, generator=gen, device="cuda") / 64).half()
    y = torch.empty(1, 4096, dtype=torch.float16, device="cuda")
    eager = ops.rmsnorm_gemv(x, g, W)
    captured = try_capture(lambda: ops.rmsnorm_gemv(x, g, W, out=y))
    assert captured.ok, captured.reason
    y.zero_()
    captured.replay()
    torch.cuda.synchronize()
    assert torch.equal(y, eager)


@pytest.mark.gpu
def test_stage_temporary_allocation_warning():
    seq = Sequence("test_temp_warn")

    @seq.stage
    def alloc_temp(x):
        _temp = torch.randn(100000, dtype=torch.float32, device="cuda")   # > 100 KB, not the output
        return x.clone()

    x = torch.randn(10, dtype=torch.float16, device="cuda")
    with pytest.warns(UserWarning, match="allocated .* MB internally; byte model undercounts"):
        seq.trace({"x": x})


@pytest.mark.gpu
def test_time_callable_sanity():
    x = torch.tensor([0], dtype=torch.int32, device="cuda")

    def increment():
        x.add_(1)

    us_times = time_callable(increment, trials=10, target_ms=5, warmup=5)
    assert len(us_times) == 10
    assert all(t > 0 for t in us_times)
    torch.cuda.synchronize()
    assert int(x.item()) >= 10 * 200          # every trial ran at least _MIN_K calls


@pytest.mark.gpu
@pytest.mark.parametrize("demo_name,expected_bound", [
    ("f1", "low-byte-opportunity"),
    ("f2", "low-byte-opportunity"),
    ("f4", "material-byte-opportunity"),
])
def test_demo_verdicts(demo_name, expected_bound):
    """The reference's demo verdicts, with this build's kernels as the fused arm."""
    from decodebench_b200.cli import _fused_bytes, hbm_peak_gbs
    from decodebench_b200.demos.llama_decode import build_demo

    seq, inputs, replicas, fused = build_demo(demo_name, dim=4096, batch=1)
    report = seq.profile(inputs, trials=10, warmup=10, input_replicas=replicas, fused=fused,
                         fused_bytes=_fused_bytes(demo_name, inputs),
                         hbm_peak_gbs=hbm_peak_gbs())
    assert report.graph_ok is True
    v = report.verdict()
    assert v.bound == expected_bound
    assert v.t_fused is not None and 0 < v.t_fused < v.t_graph, \
        f"{demo_name}: fused {v.t_fused} us not faster than the stage graph {v.t_graph} us"
    assert v.fused_gbs is not None and v.fused_gbs > 0
    print(report.render())


@pytest.mark.gpu
def test_profile_with_fused_callable():
    d = 512
    x = torch.randn(1, d, dtype=torch.float16, device="cuda")
    g = torch.randn(d, dtype=torch.float16, device="cuda")
    seq = Sequence("fused_e2e")

    @seq.stage
    def scale(x, g):
        return (x * g).contiguous()

    @seq.stage
    def shift(scale):
        return scale + 1.0

    def fused_impl(inputs):
        return inputs["x"] * inputs["g"] + 1.0

    report = seq.profile({"x": x, "g": g}, trials=6, target_ms=2.0, warmup=5, fused=fused_impl)
    assert report.fused_us is not None
    assert len(report.fused_us) == 6
    assert len(report.stream_us) == 6 and len(report.graph_us) == 6
    v = report.verdict()
    assert v.t_fused is not None and v.t_fused > 0
