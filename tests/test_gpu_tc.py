"""GPU parity of the batch > 8 tensor-core (tcgen05) path: oracle at small and
ragged shapes, and the full Llama-70B-shaped decode MLP (config C4)
against a torch fp32 reference computed on the GPU from the same bf16 inputs
(the C oracle would take minutes at that size)."""

from __future__ import annotations

import math

import numpy as np
import pytest

from oracle import oracle as O
from tests.helpers import assert_close, bits, from_torch, to_torch

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu
F16, BF16 = O.F16, O.BF16


@pytest.fixture(scope="module")
def ops():
    from decodebench_b200 import ops as _ops

    yield _ops
    assert _ops.take_device_error() == 0


@pytest.mark.parametrize("batch,d_in,d_out,dt", [
    (16, 512, 384, BF16), (9, 1024, 200, F16), (33, 256, 130, BF16), (64, 128, 1000, F16),
    (256, 64, 256, BF16), (16, 4096, 2048, BF16)])
def test_tc_rmsnorm_gemv(ops, batch, d_in, d_out, dt):
    rng = np.random.default_rng(batch * 7 + d_in)
    x, g = bits(rng, (batch, d_in), dt), bits(rng, (d_in,), dt)
    W = bits(rng, (d_out, d_in), dt, 1 / math.sqrt(d_in))
    y = ops.rmsnorm_gemv(to_torch(x, dt), to_torch(g, dt), to_torch(W, dt), eps=1e-5)
    assert_close(from_torch(y), O.rmsnorm_gemv(x, g, W, 1e-5, dt), dt, "tc F1")


@pytest.mark.parametrize("batch,d_in,d_ff,dt,norm", [
    (16, 512, 640, BF16, True), (12, 1024, 300, F16, False), (48, 256, 129, BF16, True),
    (16, 8192, 256, BF16, True)])
def test_tc_gateup_swiglu(ops, batch, d_in, d_ff, dt, norm):
    rng = np.random.default_rng(batch + d_ff)
    x = bits(rng, (batch, d_in), dt)
    g = bits(rng, (d_in,), dt) if norm else None
    Wg = bits(rng, (d_ff, d_in), dt, 1 / math.sqrt(d_in))
    Wu = bits(rng, (d_ff, d_in), dt, 1 / math.sqrt(d_in))
    h = ops.gateup_swiglu(to_torch(x, dt), to_torch(Wg, dt), to_torch(Wu, dt),
                          gamma=None if g is None else to_torch(g, dt), eps=1e-5)
    assert_close(from_torch(h), O.gateup_swiglu(x, Wg, Wu, dt, gamma=g, eps=1e-5), dt, "tc F2")


@pytest.mark.parametrize("batch,d_in,d_out,dt,res", [
    (16, 2048, 512, BF16, True), (10, 640, 96, F16, False), (128, 256, 300, BF16, True)])
def test_tc_gemv(ops, batch, d_in, d_out, dt, res):
    rng = np.random.default_rng(batch + d_out)
    x = bits(rng, (batch, d_in), dt)
    W = bits(rng, (d_out, d_in), dt, 1 / math.sqrt(d_in))
    r = bits(rng, (batch, d_out), dt) if res else None
    y = ops.gemv(to_torch(x, dt), to_torch(W, dt), residual=None if r is None else to_torch(r, dt))
    assert_close(from_torch(y), O.gemv(x, W, dt, residual=r), dt, "tc gemv")


def test_tc_deterministic_stream_k(ops):
    """Stream-K partial merges are summed in a fixed order: repeated calls agree bitwise."""
    rng = np.random.default_rng(5)
    dt = BF16
    x = to_torch(bits(rng, (16, 8192), dt), dt)
    W = to_torch(bits(rng, (1024, 8192), dt, 1 / 90.5), dt)
    a = from_torch(ops.gemv(x, W))
    for _ in range(3):
        assert np.array_equal(a, from_torch(ops.gemv(x, W)))


def test_mlp_c4_full_size(ops):
    """config C4: batch 16, d 8192, d_ff 28672, bf16, eps 1e-5."""
    torch.manual_seed(0)
    dev = "cuda"
    B, D, F = 16, 8192, 28672
    x = torch.randn(B, D, device=dev).bfloat16()
    g = torch.ones(D, device=dev).bfloat16()   # RMSNorm weight at its standard init
    Wg = (torch.randn(F, D, device=dev) / math.sqrt(D)).bfloat16()
    Wu = (torch.randn(F, D, device=dev) / math.sqrt(D)).bfloat16()
    Wd = (torch.randn(D, F, device=dev) / math.sqrt(F)).bfloat16()
    h = ops.gateup_swiglu(x, Wg, Wu, gamma=g, eps=1e-5)
    y = ops.gemv(h, Wd)
    # fp32 reference with the same rounding points (h rounded to bf16)
    xf = x.float()
    xn = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-5) * g.float()
    hr = (torch.nn.functional.silu(xn @ Wg.float().T) * (xn @ Wu.float().T)).bfloat16()
    yr = (hr.float() @ Wd.float().T).bfloat16()
    assert_close(from_torch(h), from_torch(hr), BF16, "C4 h")
    assert_close(from_torch(y), from_torch(yr), BF16, "C4 y")
