"""The persistent MLP-block kernel (dbk_mlp_block): gate/up + SwiGLU, a grid-wide
barrier, then down + residual, in one launch.

* against the oracle (oracle/orc_gateup_swiglu then orc_gemv, h rounded to the
  16-bit type in between, as the reference's f2 chain and down projection do) at
  the project's tolerance;
* bit for bit against the two-launch chain dbk_gateup_swiglu -> dbk_gemv, whose
  per-output summation order it keeps;
* the workspace's barrier counters are zero again after every call, so calls
  repeat; shapes outside the single launch are refused with DBK_ESHAPE;
* dbk_oproj_mlp_block (o_proj + residual, then the block: two grid barriers)
  the same way, against dbk_gemv followed by dbk_mlp_block and the oracle."""

from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle as O
from tests.helpers import assert_close, bits, from_torch, to_torch

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _inputs(seed, batch, d, ff, dt, gamma=True, residual=True):
    rng = np.random.default_rng(seed)
    x = bits(rng, (batch, d), dt)
    g = bits(rng, (d,), dt) if gamma else None
    Wg = bits(rng, (ff, d), dt, 1 / 32)
    Wu = bits(rng, (ff, d), dt, 1 / 32)
    # |y| mostly below 2, where one bf16 rounding flip stays within 2e-2
    Wd = bits(rng, (d, ff), dt, 1 / 256)
    r = bits(rng, (batch, d), dt, 0.5) if residual else None
    return x, g, Wg, Wu, Wd, r


def _t(a, dt):
    return None if a is None else to_torch(a, dt)


@pytest.mark.parametrize("batch,d,ff,dt,gamma,residual", [
    (1, 4096, 11008, O.F16, True, True),      # the decode layer's MLP (Llama-2-7B shape)
    (1, 4096, 14336, O.BF16, True, True),     # C2's F2 shape, then its down projection
    (2, 2048, 5632, O.F16, True, False),
    (3, 1024, 4352, O.BF16, False, True),     # no RMSNorm: x is used as is
    (4, 2048, 5632, O.F16, True, True),       # two ring stages
    (2, 1024, 2816, O.F16, True, True),       # d_ff <= 2 chunks: down keeps two chains
])
def test_mlp_block_matches_oracle_and_chain(batch, d, ff, dt, gamma, residual):
    from decodebench_b200 import ops

    x, g, Wg, Wu, Wd, r = _inputs(batch * 7 + d, batch, d, ff, dt, gamma, residual)
    tx, tg, tWg, tWu, tWd, tr = (_t(a, dt) for a in (x, g, Wg, Wu, Wd, r))
    h = torch.empty(batch, ff, dtype=tx.dtype, device="cuda")
    y = ops.mlp_block(tx, tWg, tWu, tWd, gamma=tg, eps=1e-5, residual=tr, h=h)
    ops.check_device_error()

    h2 = ops.gateup_swiglu(tx, tWg, tWu, gamma=tg, eps=1e-5)
    y2 = ops.gemv(h2, tWd, residual=tr)
    torch.cuda.synchronize()
    assert torch.equal(h, h2), "h differs from dbk_gateup_swiglu"
    assert torch.equal(y, y2), "y differs from dbk_gateup_swiglu -> dbk_gemv"

    h_ref = O.gateup_swiglu(x, Wg, Wu, dt, gamma=g, eps=1e-5)
    y_ref = O.gemv(h_ref, Wd, dt, residual=r)
    assert_close(from_torch(h), h_ref, dt, "mlp_block h")
    assert_close(from_torch(y), y_ref, dt, "mlp_block y")


def test_mlp_block_repeats_and_leaves_workspace_zero():
    from decodebench_b200 import ops

    dt = O.F16
    x, g, Wg, Wu, Wd, r = _inputs(5, 1, 4096, 11008, dt)
    tx, tg, tWg, tWu, tWd, tr = (_t(a, dt) for a in (x, g, Wg, Wu, Wd, r))
    ws = torch.zeros(256, dtype=torch.uint8, device="cuda")
    outs = [ops.mlp_block(tx, tWg, tWu, tWd, gamma=tg, residual=tr, workspace=ws)
            for _ in range(5)]
    torch.cuda.synchronize()
    ops.check_device_error()
    assert int(ws.count_nonzero()) == 0
    for o in outs[1:]:
        assert torch.equal(o, outs[0])
    # the same launches captured in a CUDA graph and replayed
    g_ = torch.cuda.CUDAGraph()
    out = torch.empty_like(outs[0])
    with torch.cuda.graph(g_):
        for _ in range(3):
            ops.mlp_block(tx, tWg, tWu, tWd, gamma=tg, residual=tr, out=out, workspace=ws)
    for _ in range(2):
        g_.replay()
    torch.cuda.synchronize()
    ops.check_device_error()
    assert torch.equal(out, outs[0])
    assert int(ws.count_nonzero()) == 0


@pytest.mark.parametrize("batch,d,ff", [(5, 1024, 4352), (1, 128, 4352), (1, 8192, 11008)])
def test_mlp_block_refuses_shapes_outside_one_launch(batch, d, ff):
    from decodebench_b200 import _native as N
    from decodebench_b200 import ops

    t = lambda *s: torch.zeros(*s, dtype=torch.float16, device="cuda")  # noqa: E731
    with pytest.raises(N.DbkError, match="status -2"):
        ops.mlp_block(t(batch, d), t(ff, d), t(ff, d), t(d, ff), gamma=t(d))


@pytest.mark.parametrize("batch,d_attn,d,ff,dt", [
    (1, 4096, 4096, 11008, O.F16),     # the decode layer's tail (Llama-2-7B shape)
    (2, 2048, 2048, 5632, O.BF16),
    (3, 1024, 1024, 4352, O.F16),
])
def test_oproj_mlp_block_matches_chain_and_oracle(batch, d_attn, d, ff, dt):
    from decodebench_b200 import ops

    x, g, Wg, Wu, Wd, _ = _inputs(11 * batch + d, batch, d, ff, dt, True, False)
    rng = np.random.default_rng(d_attn)
    attn = bits(rng, (batch, d_attn), dt)
    Wo = bits(rng, (d, d_attn), dt, 1 / 64)
    tx, tg, tWg, tWu, tWd, ta, tWo = (_t(a, dt) for a in (x, g, Wg, Wu, Wd, attn, Wo))
    ha = torch.empty(batch, d, dtype=tx.dtype, device="cuda")
    h = torch.empty(batch, ff, dtype=tx.dtype, device="cuda")
    y = ops.oproj_mlp_block(ta, tWo, tx, tWg, tWu, tWd, gamma=tg, eps=1e-5, h_attn=ha, h=h)
    ops.check_device_error()

    ha2 = ops.gemv(ta, tWo, residual=tx)
    y2 = ops.mlp_block(ha2, tWg, tWu, tWd, gamma=tg, eps=1e-5, residual=ha2)
    torch.cuda.synchronize()
    assert torch.equal(ha, ha2), "h_attn differs from dbk_gemv"
    assert torch.equal(y, y2), "y differs from dbk_gemv -> dbk_mlp_block"

    ha_ref = O.gemv(attn, Wo, dt, residual=x)
    assert_close(from_torch(ha), ha_ref, dt, "oproj_mlp_block h_attn")
    y_ref = O.mlp(ha_ref, g, Wg, Wu, Wd, 1e-5, dt, residual=ha_ref)
    assert_close(from_torch(y), y_ref, dt, "oproj_mlp_block y")
