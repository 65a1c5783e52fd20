"""QKV projection + RoPE + KV-cache append (dbk_qkv_rope_append) against a torch
fp32 restatement of the Llama attention prologue: RMSNorm (optional), q/k/v
projection, rotate-half RoPE at each sequence's position, the new token's k and
v written to its cache slot. The reference has no such stage (README.md:106), so
the oracle is the fp32 formula; tolerance as everywhere else: per element
max(2e-2, one ulp of the reference), rel-L2 <= 1e-3, one rounding of the output."""

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from tests.helpers import assert_close, from_torch  # noqa: E402

pytestmark = pytest.mark.gpu


def _ref(x, W, gamma, eps, pos, inv_freq, hq, hkv, D):
    xf = x.float()
    if gamma is not None:
        xf = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * gamma.float()
    qkv = xf @ W.float().t()
    B = x.shape[0]
    q = qkv[:, :hq * D].view(B, hq, D)
    k = qkv[:, hq * D:(hq + hkv) * D].view(B, hkv, D)
    v = qkv[:, (hq + hkv) * D:].view(B, hkv, D)
    ang = pos.float()[:, None] * inv_freq[None, :]
    cos, sin = torch.cos(ang)[:, None, :], torch.sin(ang)[:, None, :]

    def rot(t):
        t1, t2 = t[..., :D // 2], t[..., D // 2:]
        return torch.cat([t1 * cos - t2 * sin, t2 * cos + t1 * sin], dim=-1)
    return rot(q), rot(k), v


CASES = [  # dtype, batch, d_in, hq, hkv, paged, gamma
    (torch.float16, 1, 4096, 32, 8, True, True),
    (torch.bfloat16, 3, 1024, 8, 2, False, False),
    (torch.float16, 8, 2048, 16, 4, True, False),
    (torch.bfloat16, 5, 4096, 32, 8, True, True),
]


@pytest.mark.parametrize("dt,batch,d_in,hq,hkv,paged,use_gamma", CASES)
def test_qkv_rope_append(dt, batch, d_in, hq, hkv, paged, use_gamma):
    from decodebench_b200 import ops

    D, ps = 128, 64
    g = torch.Generator(device="cuda").manual_seed(batch * 7 + hq)
    dev = "cuda"
    code = 0 if dt == torch.float16 else 1
    x = torch.randn(batch, d_in, generator=g, device=dev).to(dt)
    gamma = torch.randn(d_in, generator=g, device=dev).to(dt) if use_gamma else None
    W = (torch.randn((hq + 2 * hkv) * D, d_in, generator=g, device=dev) / d_in ** 0.5).to(dt)
    W_il = ops.interleave_rope_rows(W, hq, hkv, D)
    inv_freq = ops.rope_inv_freq(D, 500000.0, device=dev)
    rng = np.random.default_rng(batch + d_in)
    max_pages = 520                                  # up to 33280 positions per sequence
    pos_np = rng.integers(0, max_pages * ps, size=batch).astype(np.int32)
    pos_np[0] = 32767
    if batch > 2:
        pos_np[-1] = max_pages * ps                  # outside the cache: q only
    pos = torch.from_numpy(pos_np).to(dev)
    if paged:
        npages = batch * max_pages
        table = torch.from_numpy(rng.permutation(npages).astype(np.int32).reshape(batch, max_pages)).to(dev)
        kc = torch.full((npages, hkv, ps, D), 7.0, dtype=dt, device=dev)
    else:
        table = None
        kc = torch.full((batch, hkv, max_pages * ps, D), 7.0, dtype=dt, device=dev)
    vc = kc.clone()
    q = ops.qkv_rope_append(x, W_il, pos, inv_freq, kc, vc, hq, hkv, page_table=table,
                            gamma=gamma, eps=1e-5)
    torch.cuda.synchronize()
    rq, rk, rv = _ref(x, W, gamma, 1e-5, pos, inv_freq, hq, hkv, D)
    assert_close(from_torch(q), from_torch(rq.to(dt)), code, "q")
    written = torch.zeros_like(kc, dtype=torch.bool)
    for b in range(batch):
        p = int(pos_np[b])
        if p >= max_pages * ps:
            continue
        if paged:
            page, off = int(table[b, p // ps]), p % ps
        else:
            page, off = b, p
        assert_close(from_torch(kc[page, :, off]), from_torch(rk[b].to(dt)), code, f"k[{b}]")
        assert_close(from_torch(vc[page, :, off]), from_torch(rv[b].to(dt)), code, f"v[{b}]")
        written[page, :, off] = True
    assert bool((kc[~written] == 7.0).all()) and bool((vc[~written] == 7.0).all()), \
        "a cache slot other than the new token's was written"
