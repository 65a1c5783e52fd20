"""Host-side helpers of the added rows, on CPU tensors: the pair-interleaved
Wqkv layout for dbk_qkv_rope_append, the rotary frequencies, and the per-row
e4m3 quantisation for the fp8 GEMVs, and the choice between the persistent MLP
block and two launches."""

import pytest

torch = pytest.importorskip("torch")

from decodebench_b200 import ops  # noqa: E402


def test_interleave_rope_rows_is_the_documented_permutation():
    hq, hkv, D = 4, 2, 16
    W = torch.arange((hq + 2 * hkv) * D, dtype=torch.float32)[:, None].repeat(1, 3)
    il = ops.interleave_rope_rows(W, hq, hkv, D)
    assert il.shape == W.shape
    assert sorted(il[:, 0].tolist()) == W[:, 0].tolist()          # a permutation
    for head in range(hq + hkv):                                    # q and k heads
        for i in range(D // 2):
            assert il[head * D + 2 * i, 0] == head * D + i
            assert il[head * D + 2 * i + 1, 0] == head * D + i + D // 2
    v0 = (hq + hkv) * D
    assert torch.equal(il[v0:], W[v0:])                            # v heads unchanged


def test_rope_inv_freq_matches_llama():
    f = ops.rope_inv_freq(128, 500000.0)
    assert f.dtype == torch.float32 and f.shape == (64,)
    ref = 1.0 / (500000.0 ** (torch.arange(0, 128, 2).float() / 128))
    assert torch.equal(f, ref)


def test_quantize_fp8_rows_bounds_the_error():
    g = torch.Generator().manual_seed(0)
    W = torch.randn(64, 256, generator=g) * torch.logspace(-3, 2, 64)[:, None]
    W8, s = ops.quantize_fp8_rows(W)
    assert W8.dtype == torch.float8_e4m3fn and s.dtype == torch.float32
    deq = W8.float() * s[:, None]
    # e4m3: 3 mantissa bits -> relative rounding error <= 2^-4 for normal values;
    # the row maximum maps to 448 exactly
    rel = ((deq - W).abs() / W.abs().amax(dim=1, keepdim=True)).max()
    assert float(rel) <= 2 ** -4
    assert torch.allclose(deq.abs().amax(dim=1), W.abs().amax(dim=1), rtol=2 ** -4)


def test_mlp_block_refuses_cpu_tensors():
    t = lambda *s: torch.zeros(*s, dtype=torch.float16)  # noqa: E731
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        ops.mlp_block(t(1, 256), t(4352, 256), t(4352, 256), t(256, 4352))
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        ops.oproj_mlp_block(t(1, 256), t(256, 256), t(1, 256), t(4352, 256), t(4352, 256),
                            t(256, 4352))


def test_mlp_takes_two_launches_when_the_single_launch_refuses(monkeypatch):
    """ops.mlp: a DBK_ESHAPE answer of the persistent kernel (returned before any
    launch) sends this shape to gate/up + down from then on; other errors raise."""
    from decodebench_b200 import _native as N

    calls = []

    def refuse(*a, **k):
        calls.append("block")
        raise N.DbkError("dbk_mlp_block", N.DBK_ESHAPE)

    monkeypatch.setattr(ops, "_MLP_BLOCK", True)
    monkeypatch.setattr(ops, "_mlp_block_refused", set())
    monkeypatch.setattr(ops, "mlp_block", refuse)
    monkeypatch.setattr(ops, "gateup_swiglu", lambda x, *a, **k: calls.append("gateup") or x)
    monkeypatch.setattr(ops, "gemv", lambda h, *a, **k: calls.append("gemv") or h)
    x = torch.zeros(1, 64)
    for _ in range(2):
        ops.mlp(x, None, torch.zeros(300, 64), None, None)
    assert calls == ["block", "gateup", "gemv", "gateup", "gemv"]

    def broken(*a, **k):
        raise N.DbkError("dbk_mlp_block", -3)       # DBK_EALIGN

    monkeypatch.setattr(ops, "_mlp_block_refused", set())
    monkeypatch.setattr(ops, "mlp_block", broken)
    with pytest.raises(N.DbkError):
        ops.mlp(x, None, torch.zeros(300, 64), None, None)
