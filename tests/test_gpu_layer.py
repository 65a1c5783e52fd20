"""The whole-decode-layer demo: five fused sm_100a kernels (QKV + RoPE + cache
append -> FlashDecode -> o_proj + residual -> RMSNorm + gate/up + SwiGLU -> down +
residual, chained with programmatic dependent launch) against the unfused PyTorch
stage chain, through the same Sequence / profile / Verdict path as the reference's
demos. The chain rounds to fp16 after every stage, so the comparison uses the
reference's own fused-output gate (fail iff abs >= 5e-2 and rel >= 2e-2,
sequence.py:308-332) plus a loose rel-L2 bound."""

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from tests.helpers import from_torch, reference_gate  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("batch", [1, 4])
def test_layer_fused_matches_chain(batch):
    from decodebench_b200.demos.llama_decode import build_demo

    seq, inputs, reps, fused = build_demo("layer", dim=2048, batch=batch)
    ref = seq.run(inputs)
    got = fused(inputs)
    again = fused(inputs)                 # the cache append is idempotent
    torch.cuda.synchronize()
    assert got.shape == ref.shape
    assert torch.equal(got, again), "fused layer is not deterministic"
    assert reference_gate(from_torch(got), from_torch(ref), 0)
    g, r = got.float(), ref.float()
    assert float((g - r).norm() / r.norm()) < 1e-2


def test_layer_profile_runs_through_the_verdict():
    from decodebench_b200.cli import _run_demo

    report = _run_demo("layer", 2048, 1, 3, 0.2, True)
    v = report.verdict()
    assert np.isfinite(v.t_graph) and v.t_graph > 0
    assert v.t_fused is not None and 0 < v.t_fused < v.t_graph, \
        f"fused layer {v.t_fused} us not faster than the unfused graph {v.t_graph} us"
    assert v.fused_gbs is not None
    print(report.render())
