"""The CPU oracle, pinned: the reference's own known-answer tests
(validation/src/tests/test_reference.cpp:32-178), bit-exact agreement with the
reference's compiled cpu_reference.cpp (oracle/_ref, when built), the golden
outputs of the reference's PyTorch stage chains, and the split-KV restatement."""

import math

import numpy as np
import pytest

from oracle import oracle as O

needs_ref = pytest.mark.skipif(not O.have_ref(), reason="oracle/_ref not built (no reference checkout)")


# ---- known-answer tests restated from test_reference.cpp
def test_kat_rmsnorm():
    x = np.array([1, 2, 3, 4], np.float32)
    out = O.rmsnorm_f32(x, np.ones(4, np.float32))
    rms = math.sqrt((1 + 4 + 9 + 16) / 4 + 1e-6)
    np.testing.assert_allclose(out, x / rms, atol=1e-5)


def test_kat_gemv():
    out = O.gemv_f32(np.array([[1, 2], [3, 4]], np.float32), np.ones(2, np.float32))
    np.testing.assert_allclose(out, [3, 7], atol=1e-5)


def test_kat_silu_swiglu():
    assert abs(O.silu(0.0)) < 1e-6
    assert abs(O.silu(1.0) - 0.7310586) < 1e-6
    out = O.swiglu_f32(np.array([0, 1, 2], np.float32), np.ones(3, np.float32))
    np.testing.assert_allclose(out, [0, 0.7310586, O.silu(2.0)], atol=1e-5)


def test_kat_softmax():
    p = O.softmax_f32(np.array([[0, 1, 2], [0, 0, 0]], np.float32))
    e = np.exp([0, 1, 2])
    np.testing.assert_allclose(p[0], e / e.sum(), atol=1e-5)
    np.testing.assert_allclose(p[1], [1 / 3] * 3, atol=1e-6)


def test_kat_attention():
    out = O.attention_f32(np.array([[1, 0]], np.float32), np.array([[[1, 0], [0, 1]]], np.float32),
                          np.array([[[2, 0], [0, 3]]], np.float32))
    e = math.e
    p0, p1 = e / (e + 1), 1 / (e + 1)
    np.testing.assert_allclose(out[0], [2 * p0, 3 * p1], atol=1e-5)


# ---- agreement with the reference's compiled CPU oracle
@needs_ref
def test_primitives_match_reference_binary():
    rng = np.random.default_rng(0)
    x = rng.standard_normal(1000).astype(np.float32)
    g = rng.standard_normal(1000).astype(np.float32)
    assert np.array_equal(O.rmsnorm_f32(x, g, 1e-6), O.rmsnorm_f32(x, g, 1e-6, use_ref=True))
    W = rng.standard_normal((37, 1000)).astype(np.float32)
    assert np.array_equal(O.gemv_f32(W, x), O.gemv_f32(W, x, use_ref=True))
    assert np.array_equal(O.gemv_f32(W, x), O.ref_gemv_threaded(W, x, 4))
    for v in (-3.5, -1.0, 0.0, 0.25, 7.0):
        assert O.silu(v) == O.silu(v, use_ref=True)
    s = rng.standard_normal((4, 300)).astype(np.float32)
    assert np.array_equal(O.softmax_f32(s), O.softmax_f32(s, use_ref=True))
    q = rng.standard_normal((3, 64)).astype(np.float32)
    K = rng.standard_normal((3, 129, 64)).astype(np.float32)
    V = rng.standard_normal((3, 129, 64)).astype(np.float32)
    assert np.array_equal(O.attention_f32(q, K, V), O.attention_f32(q, K, V, use_ref=True))


# ---- 16-bit conversions are IEEE round-to-nearest-even
def test_conversions_bit_exact():
    import torch

    rng = np.random.default_rng(1)
    a = (rng.standard_normal(100000) * np.exp(rng.uniform(-18, 11, 100000))).astype(np.float32)
    a[:6] = [0.0, -0.0, 65504.0, 65519.0, 5.96e-8, 2.98e-8]
    with np.errstate(over="ignore"):
        assert np.array_equal(O.to16(a, O.F16), a.astype(np.float16).view(np.uint16))
    bf = torch.from_numpy(a).bfloat16().view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(O.to16(a, O.BF16), bf)
    h = O.to16(a, O.F16)
    assert np.array_equal(O.from16(h, O.F16), h.view(np.float16).astype(np.float32))


# ---- golden outputs of the reference's PyTorch stages (tests/golden/make_golden.py)
def _g(name):
    from pathlib import Path

    return np.load(Path(__file__).resolve().parent / "golden" / f"golden_{name}.npz")


@pytest.mark.parametrize("name", ["f1", "f1_ragged"])
def test_golden_f1_stage_semantics(name):
    z = _g(name)
    y = O.rmsnorm_gemv(z["x"], z["g"], z["W"], 1e-6, O.F16, O.ROUND_STAGES)
    assert np.array_equal(y, z["y"])


def test_golden_f2_stage_semantics():
    z = _g("f2")
    y = O.gateup_swiglu(z["xh"], z["Wg"], z["Wu"], O.F16, round_mode=O.ROUND_STAGES)
    assert np.array_equal(y, z["y"])


def test_golden_f4_stage_semantics():
    # torch's CPU softmax exp differs from libm's by an ulp now and then, which can
    # flip the fp16 rounding of a probability: agreement is to 2e-4, not bit-exact.
    z = _g("f4")
    y = O.attention(z["q"], z["K"], z["V"], O.F16, 1.0, round_mode=O.ROUND_STAGES)
    a, b = O.from16(y, O.F16), O.from16(z["y"], O.F16)
    assert np.abs(a - b).max() < 2e-4
    assert (y == z["y"]).mean() > 0.95


# ---- split-KV + LSE merge restatement equals direct attention
@pytest.mark.parametrize("L,splits,tile", [(4096, 32, 128), (1000, 7, 128), (130, 5, 64), (64, 9, 128)])
def test_splitkv_merge_equals_direct(L, splits, tile):
    rng = np.random.default_rng(L + splits)
    d = 128
    q = rng.standard_normal(d).astype(np.float32)
    K = rng.standard_normal((L, d)).astype(np.float32)
    V = rng.standard_normal((L, d)).astype(np.float32)
    scale = 1 / math.sqrt(d)
    got = O.splitkv_head(q, K, V, scale, splits, tile)
    s = (K @ q) * scale
    p = np.exp(s - s.max())
    want = (p / p.sum()) @ V
    np.testing.assert_allclose(got, want, atol=1e-5, rtol=1e-4)


def test_paged_oracle_equals_contiguous():
    rng = np.random.default_rng(3)
    dt, d, ps = O.BF16, 128, 16
    K = O.to16(rng.standard_normal((2, 2, 64, d)).astype(np.float32), dt)
    V = O.to16(rng.standard_normal((2, 2, 64, d)).astype(np.float32), dt)
    q = O.to16(rng.standard_normal((2, 8, d)).astype(np.float32), dt)
    perm = rng.permutation(8).astype(np.int32).reshape(2, 4)
    Kp = np.zeros((8, 2, ps, d), np.uint16)
    Vp = np.zeros_like(Kp)
    for b in range(2):
        for p in range(4):
            Kp[perm[b, p]] = K[b, :, p * ps:(p + 1) * ps]
            Vp[perm[b, p]] = V[b, :, p * ps:(p + 1) * ps]
    lens = np.array([64, 37], np.int32)
    a = O.attention(q, K, V, dt, 0.1, seq_lens=lens)
    b = O.attention(q, Kp, Vp, dt, 0.1, seq_lens=lens, page_table=perm)
    assert np.array_equal(a, b)
