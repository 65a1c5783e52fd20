"""Llama decode-chain demos F1, F2, F4 with their fused sm_100a stages.

The unfused chains keep the reference's stage code semantics
(src/decodebench/demos/llama_decode.py:24-161): F1 rmsnorm (eps 1e-6, fp16
roundings) -> gemv; F2 gate, up, swiglu; F4 scores (no scale), softmax, weighted_v.
Unlike the reference, inputs are drawn from a seeded CPU generator (the
reference allocates before its seed call, sequence.py:228) and use
BASELINE-style scaling so fp16 stays far from overflow: W ~ N(0,1)/sqrt(d) and,
for F4, q ~ N(0, 1/128) so the unscaled scores have unit variance.

``build_demo`` returns (seq, inputs, replicas, fused) where ``fused`` is the
B200 kernel for the whole chain, ready for ``seq.profile(fused=fused)``.
"""

from __future__ import annotations

import math

from ..sequence import Sequence
from ..timing import n_weight_replicas

DEMO_NAMES = ("f1", "f2", "f4")
_FFN = {2048: 8192, 4096: 11008}
_L = 1024
_HEAD_DIM = 128


def _randn(gen, *shape, scale=1.0, dtype=None):
    import torch

    t = torch.randn(*shape, generator=gen, dtype=torch.float32) * scale
    return t.to(dtype=dtype or torch.float16, device="cuda")


def _replicas(base: dict, weight_keys: tuple[str, ...]) -> list[dict]:
    nbytes = sum(base[k].nbytes for k in weight_keys)
    reps = []
    for i in range(n_weight_replicas(nbytes)):
        reps.append({k: (v.clone() if (k in weight_keys and i) else v) for k, v in base.items()})
    return reps


def _build_f1(dim: int, batch: int, gen):
    import torch

    from .. import ops

    x = _randn(gen, batch, dim)
    g = _randn(gen, dim)
    W = _randn(gen, dim, dim, scale=1.0 / math.sqrt(dim))
    seq = Sequence("f1")

    @seq.stage
    def rmsnorm(x, g):
        var = x.float().pow(2).mean(dim=-1, keepdim=True)
        return (x.float() * torch.rsqrt(var + 1e-6)).half() * g

    @seq.stage
    def gemv(xh, W):
        return torch.nn.functional.linear(xh, W)

    def fused(inp):
        return ops.rmsnorm_gemv(inp["x"], inp["g"], inp["W"], eps=1e-6)

    inputs = {"x": x, "g": g, "W": W}
    return seq, inputs, _replicas(inputs, ("W",)), fused


def _build_f2(dim: int, batch: int, gen):
    import torch

    from .. import ops

    ff = _FFN[dim]
    xh = _randn(gen, batch, dim)
    Wg = _randn(gen, ff, dim, scale=1.0 / math.sqrt(dim))
    Wu = _randn(gen, ff, dim, scale=1.0 / math.sqrt(dim))
    seq = Sequence("f2")

    @seq.stage
    def gate(xh, Wg):
        return torch.nn.functional.linear(xh, Wg)

    @seq.stage
    def up(xh, Wu):
        return torch.nn.functional.linear(xh, Wu)

    @seq.stage
    def swiglu(up, gate):
        return torch.nn.functional.silu(gate) * up

    def fused(inp):
        return ops.gateup_swiglu(inp["xh"], inp["Wg"], inp["Wu"])

    inputs = {"xh": xh, "Wg": Wg, "Wu": Wu}
    return seq, inputs, _replicas(inputs, ("Wg", "Wu")), fused


def _build_f4(dim: int, batch: int, gen):
    import torch

    from .. import ops

    H, D, L = dim // _HEAD_DIM, _HEAD_DIM, _L
    q = _randn(gen, batch, H, D, scale=D ** -0.5)
    K = _randn(gen, batch, H, L, D)
    V = _randn(gen, batch, H, L, D)
    seq = Sequence("f4")

    @seq.stage
    def scores(q, K):
        return torch.einsum("bhd,bhld->bhl", q, K).float()

    @seq.stage
    def softmax(s):
        return torch.softmax(s, dim=-1)

    @seq.stage
    def weighted_v(p, V):
        return torch.einsum("bhl,bhld->bhd", p.half(), V)

    def fused(inp):
        # The reference chain applies no 1/sqrt(D) scale (llama_decode.py:120-125).
        return ops.flashdecode(inp["q"], inp["K"], inp["V"], scale=1.0)

    inputs = {"q": q, "K": K, "V": V}
    return seq, inputs, _replicas(inputs, ("K", "V")), fused


_BUILDERS = {"f1": _build_f1, "f2": _build_f2, "f4": _build_f4}


def build_demo(name: str, dim: int = 4096, batch: int = 1, seed: int = 42):
    """Build a named demo: returns (seq, inputs, input_replicas, fused_callable)."""
    if name not in _BUILDERS:
        raise ValueError(f"unknown demo '{name}'; choose from {list(_BUILDERS)}")
    import torch

    gen = torch.Generator().manual_seed(seed)
    return _BUILDERS[name](dim, batch, gen)
