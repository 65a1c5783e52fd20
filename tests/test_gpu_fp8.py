"""GEMVs with e4m3 weights and per-row scales (dbk_*_fp8) against a torch fp32
restatement over the dequantised weights (scale * W8, exact in fp32). The
quantisation itself is the caller's choice (ops.quantize_fp8_rows); parity is
about the kernel: same tolerance as the 16-bit paths (per element max(2e-2,
1 ulp), rel-L2 <= 1e-3)."""

import pytest

torch = pytest.importorskip("torch")

from tests.helpers import assert_close, from_torch  # noqa: E402

pytestmark = pytest.mark.gpu

CASES = [(torch.float16, 1, 4096, 4096), (torch.bfloat16, 3, 2048, 1000),
         (torch.float16, 8, 1024, 333), (torch.bfloat16, 2, 8192, 512)]


def _deq(W8, sc):
    return W8.float() * sc[:, None]


@pytest.mark.parametrize("dt,batch,d_in,d_out", CASES)
def test_fp8_gemv_family(dt, batch, d_in, d_out):
    from decodebench_b200 import ops

    g = torch.Generator(device="cuda").manual_seed(d_in + batch)
    code = 0 if dt == torch.float16 else 1
    x = torch.randn(batch, d_in, generator=g, device="cuda").to(dt)
    gam = torch.randn(d_in, generator=g, device="cuda").to(dt)
    W8, s = ops.quantize_fp8_rows(torch.randn(d_out, d_in, generator=g, device="cuda") / d_in ** 0.5)
    Wu8, su = ops.quantize_fp8_rows(torch.randn(d_out, d_in, generator=g, device="cuda") / d_in ** 0.5)
    res = torch.randn(batch, d_out, generator=g, device="cuda").to(dt)
    Wd, Wud = _deq(W8, s), _deq(Wu8, su)
    xf = x.float()
    xn = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-5) * gam.float()

    y = ops.gemv_fp8(x, W8, s, residual=res)
    assert_close(from_torch(y), from_torch((xf @ Wd.t() + res.float()).to(dt)), code, "gemv_fp8")
    y = ops.rmsnorm_gemv_fp8(x, gam, W8, s, eps=1e-5)
    assert_close(from_torch(y), from_torch((xn @ Wd.t()).to(dt)), code, "rmsnorm_gemv_fp8")
    h = ops.gateup_swiglu_fp8(x, W8, s, Wu8, su, gamma=gam, eps=1e-5)
    ref = torch.nn.functional.silu(xn @ Wd.t()) * (xn @ Wud.t())
    assert_close(from_torch(h), from_torch(ref.to(dt)), code, "gateup_swiglu_fp8")
    h = ops.gateup_swiglu_fp8(x, W8, s, Wu8, su)
    ref = torch.nn.functional.silu(xf @ Wd.t()) * (xf @ Wud.t())
    assert_close(from_torch(h), from_torch(ref.to(dt)), code, "gateup_swiglu_fp8 (no norm)")
