"""Host-side helpers of the added rows, on CPU tensors: the pair-interleaved
Wqkv layout for dbk_qkv_rope_append, the rotary frequencies, and the per-row
e4m3 quantisation for the fp8 GEMVs."""

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
