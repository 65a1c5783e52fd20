"""Llama decode-chain demos F1, F2, F4 with their fused sm_100a stages.

The unfused chains keep the reference's stage code semantics
(src/decodebench/demos/llama_decode.py:24-161): F1 rmsnorm (eps 1e-6, fp16
roundings) -> gemv; F2 gate, up, swiglu; F4 scores (no scale), softmax, weighted_v.
Unlike the reference, inputs are drawn from a seeded CPU generator (the
reference allocates before its seed call, sequence.py:228) and use
benchmark-style scaling so fp16 stays far from overflow: W ~ N(0,1)/sqrt(d) and,
for F4, q ~ N(0, 1/128) so the unscaled scores have unit variance.

``build_demo`` returns (seq, inputs, replicas, fused) where ``fused`` is the
B200 kernel for the whole chain, ready for ``seq.profile(fused=fused)``.
"""

from __future__ import annotations

import math

from ..sequence import Sequence
from ..timing import n_weight_replicas

DEMO_NAMES = ("f1", "f2", "f4", "layer")
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


def _build_layer(dim: int, batch: int, gen):
    """One whole Llama decode layer for a single new token per sequence (the
    reference's demos stop at single fused ops; README.md:7-14 frames the layer as
    the unit whose launch overhead matters).

    Unfused: the stage chain below in PyTorch (each stage one tensor; attention
    rotates and attends to the new token's k/v next to the cached ones without
    writing the cache). Fused: five sm_100a kernels chained with programmatic
    dependent launch: QKV + RoPE + cache append, FlashDecode over the cache,
    o_proj + residual, RMSNorm + gate/up + SwiGLU, down + residual."""
    import torch

    from .. import ops

    ff = _FFN[dim]
    H, Hkv, D, L = dim // _HEAD_DIM, max(1, dim // _HEAD_DIM // 4), _HEAD_DIM, _L
    sc = 1.0 / math.sqrt(dim)
    x = _randn(gen, batch, dim)
    g1 = _randn(gen, dim, scale=0.5)
    g2 = _randn(gen, dim, scale=0.5)
    Wqkv = _randn(gen, (H + 2 * Hkv) * D, dim, scale=sc)
    Wo = _randn(gen, dim, H * D, scale=1.0 / math.sqrt(H * D))
    Wg = _randn(gen, ff, dim, scale=sc)
    Wu = _randn(gen, ff, dim, scale=sc)
    Wd = _randn(gen, dim, ff, scale=1.0 / math.sqrt(ff))
    cap = L + 64                                   # cache slots; the new token goes to slot L
    Kc = _randn(gen, batch, Hkv, cap, D)
    Vc = _randn(gen, batch, Hkv, cap, D)
    pos = torch.full((batch,), L, dtype=torch.int32, device="cuda")
    lens = torch.full((batch,), L + 1, dtype=torch.int32, device="cuda")
    inv_freq = ops.rope_inv_freq(D, 500000.0, device="cuda")
    ang = pos.float()[:, None] * inv_freq[None, :]
    cos, sin = torch.cos(ang), torch.sin(ang)      # [batch, D/2] fp32
    Wqkv_il = ops.interleave_rope_rows(Wqkv, H, Hkv, D)
    seq = Sequence("layer")

    def _rms(t, g):
        var = t.float().pow(2).mean(dim=-1, keepdim=True)
        return (t.float() * torch.rsqrt(var + 1e-5)).half() * g

    def _rot(t, c, s):                             # t [B, heads, D]
        t1, t2 = t[..., :D // 2].float(), t[..., D // 2:].float()
        c, s = c[:, None, :], s[:, None, :]
        return torch.cat([t1 * c - t2 * s, t2 * c + t1 * s], dim=-1).half()

    @seq.stage
    def attn_norm(x, g1):
        return _rms(x, g1)

    @seq.stage
    def qkv(attn_norm, Wqkv):
        return torch.nn.functional.linear(attn_norm, Wqkv)

    @seq.stage
    def q_rot(qkv, cos, sin):
        return _rot(qkv[:, :H * D].reshape(-1, H, D), cos, sin).contiguous()

    # Attention over the cache plus the new token, one op per stage so the byte
    # model sees every tensor (the grouped einsums read each kv head once for its
    # G = H / Hkv query heads, as the fused kernel does).
    G = H // Hkv

    @seq.stage
    def k_rot(qkv, cos, sin):
        return _rot(qkv[:, H * D:(H + Hkv) * D].reshape(-1, Hkv, D), cos, sin).contiguous()

    @seq.stage
    def v_new(qkv):
        return qkv[:, (H + Hkv) * D:].reshape(-1, Hkv, D).clone()

    def _append(cache, new):                       # [B, Hkv, L+1, D], no temporaries
        out = torch.empty(cache.shape[0], Hkv, L + 1, D, dtype=cache.dtype, device=cache.device)
        out[:, :, :L].copy_(cache[:, :, :L])
        out[:, :, L].copy_(new)
        return out

    @seq.stage
    def K_all(k_rot, Kc):
        return _append(Kc, k_rot)

    @seq.stage
    def V_all(v_new, Vc):
        return _append(Vc, v_new)

    @seq.stage
    def scores(q_rot, K_all):
        qg = q_rot.reshape(q_rot.shape[0], Hkv, G, D)
        return torch.einsum("bkgd,bkld->bkgl", qg, K_all).contiguous()  # fp16, fp32 accumulate

    @seq.stage
    def logits(scores):
        return scores.to(torch.float32).mul_(1.0 / math.sqrt(D))

    @seq.stage
    def probs(logits):
        return torch.softmax(logits, dim=-1)

    @seq.stage
    def p_half(probs):
        return probs.half()

    @seq.stage
    def attn(p_half, V_all):
        o = torch.einsum("bkgl,bkld->bkgd", p_half, V_all)
        return o.reshape(o.shape[0], H * D)

    @seq.stage
    def o_proj(attn, Wo):
        return torch.nn.functional.linear(attn, Wo)

    @seq.stage
    def resid1(o_proj, x):
        return o_proj + x

    @seq.stage
    def mlp_norm(resid1, g2):
        return _rms(resid1, g2)

    @seq.stage
    def gate(mlp_norm, Wg):
        return torch.nn.functional.linear(mlp_norm, Wg)

    @seq.stage
    def up(mlp_norm, Wu):
        return torch.nn.functional.linear(mlp_norm, Wu)

    @seq.stage
    def swiglu(up, gate):
        return torch.nn.functional.silu(gate) * up

    @seq.stage
    def down(swiglu, Wd):
        return torch.nn.functional.linear(swiglu, Wd)

    @seq.stage
    def resid2(down, resid1):
        return down + resid1

    def fused(inp):
        q = ops.qkv_rope_append(inp["x"], inp["Wqkv_il"], inp["pos"], inp["inv_freq"],
                                inp["Kc"], inp["Vc"], H, Hkv, gamma=inp["g1"], eps=1e-5)
        o = ops.flashdecode(q, inp["Kc"], inp["Vc"], seq_lens=inp["lens"])
        # o_proj + residual, then RMSNorm + gate/up + SwiGLU and down + residual in one
        # persistent launch
        return ops.layer_tail(o.reshape(o.shape[0], -1), inp["Wo"], inp["x"], inp["g2"],
                              inp["Wg"], inp["Wu"], inp["Wd"], eps=1e-5)

    inputs = {"x": x, "g1": g1, "g2": g2, "Wqkv": Wqkv, "Wqkv_il": Wqkv_il, "Wo": Wo, "Wg": Wg,
              "Wu": Wu, "Wd": Wd, "Kc": Kc, "Vc": Vc, "cos": cos, "sin": sin, "pos": pos,
              "lens": lens, "inv_freq": inv_freq}
    return seq, inputs, _replicas(inputs, ("Wqkv", "Wqkv_il", "Wo", "Wg", "Wu", "Wd")), fused


_BUILDERS = {"f1": _build_f1, "f2": _build_f2, "f4": _build_f4, "layer": _build_layer}


def build_demo(name: str, dim: int = 4096, batch: int = 1, seed: int = 42):
    """Build a named demo: returns (seq, inputs, input_replicas, fused_callable)."""
    if name not in _BUILDERS:
        raise ValueError(f"unknown demo '{name}'; choose from {list(_BUILDERS)}")
    import torch

    gen = torch.Generator().manual_seed(seed)
    return _BUILDERS[name](dim, batch, gen)
