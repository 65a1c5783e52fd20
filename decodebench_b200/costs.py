"""Analytic byte accounting for the decode hot path.

* Unfused stage traces of F1/F2/F4, restating the reference's cost model
  (model/cost_model.py:18-44): golden totals at d=4096 are 33,595,392 /
  180,481,536 / 17,317,888 bytes.
* Algorithmic bytes of one fused step for each benchmark configuration
  (C1..C5): every weight / cache byte read once, activations read once,
  outputs written once. These are the numerators of achieved GB/s.
"""

from __future__ import annotations

from dataclasses import dataclass

from .bytes_model import StageTrace, eliminable_bytes, total_bytes

FFN = {2048: 8192, 4096: 11008}


def f1_traces(d: int, b: int = 1) -> list[StageTrace]:
    return [StageTrace("rmsnorm", [2 * b * d, 2 * d], 2 * b * d),
            StageTrace("gemv", [2 * d * d, 2 * b * d], 2 * b * d, is_final=True, consumers=0)]


def f2_traces(d: int, b: int = 1) -> list[StageTrace]:
    ff = FFN[d]
    return [StageTrace("gate", [2 * b * d, 2 * ff * d], 2 * b * ff),
            StageTrace("up", [2 * b * d, 2 * ff * d], 2 * b * ff),
            StageTrace("swiglu", [2 * b * ff, 2 * b * ff], 2 * b * ff, is_final=True, consumers=0)]


def f4_traces(d: int, b: int = 1, L: int = 1024, head_dim: int = 128) -> list[StageTrace]:
    h = d // head_dim
    kv = 2 * b * h * L * head_dim
    return [StageTrace("scores", [2 * b * d, kv], 4 * b * h * L),
            StageTrace("softmax", [4 * b * h * L], 4 * b * h * L),
            StageTrace("weighted_v", [4 * b * h * L, kv], 2 * b * d, is_final=True, consumers=0)]


@dataclass(frozen=True)
class FusionCost:
    name: str
    total: int
    eliminable: int
    ratio: float
    predicted: str


def fusion_costs(d: int = 4096, b: int = 1, threshold: float = 0.01) -> list[FusionCost]:
    out = []
    for name, fn in (("F1", f1_traces), ("F2", f2_traces), ("F4", f4_traces)):
        tr = fn(d, b)
        tot, el = total_bytes(tr), eliminable_bytes(tr)
        r = el / tot
        out.append(FusionCost(name, tot, el, r, "material-byte-opportunity" if r >= threshold
                              else "low-byte-opportunity"))
    return out


# ------------------------------------------------------------------ fused-step bytes
def rmsnorm_gemv_bytes(batch: int, d_in: int, d_out: int, elem: int = 2) -> int:
    """W once + x + gamma + y."""
    return elem * (d_out * d_in + batch * d_in + d_in + batch * d_out)


def gateup_swiglu_bytes(batch: int, d_in: int, d_ff: int, elem: int = 2,
                        with_gamma: bool = False) -> int:
    return elem * (2 * d_ff * d_in + batch * d_in + (d_in if with_gamma else 0) + batch * d_ff)


def gemv_bytes(batch: int, d_in: int, d_out: int, elem: int = 2, residual: bool = False) -> int:
    return elem * (d_out * d_in + batch * d_in + batch * d_out * (2 if residual else 1))


def mlp_bytes(batch: int, d: int, d_ff: int, elem: int = 2) -> int:
    """RMSNorm -> gate/up -> SwiGLU -> down, intermediates never leave the fused
    path: 3 weight matrices + x + gamma + y (C4: 1,409,826,816 B)."""
    return elem * (3 * d * d_ff + batch * d + d + batch * d)


def flashdecode_bytes(seq_lens, n_q_heads: int, n_kv_heads: int, head_dim: int = 128,
                      elem: int = 2, page_table_bytes: int = 0) -> int:
    """K and V of every cached token once + q + out (+ the page table)."""
    toks = int(sum(int(x) for x in seq_lens))
    batch = len(seq_lens)
    return (elem * (2 * toks * n_kv_heads * head_dim + 2 * batch * n_q_heads * head_dim)
            + page_table_bytes)
