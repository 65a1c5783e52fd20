"""Shared helpers for the parity tests: seeded 16-bit inputs and the tolerance.

Tolerance (the project's stated bar for fp16/bf16 outputs with fp32
accumulation): every element within max(2e-2, one unit in the last place of the
reference value) AND ||kernel - oracle||_2 / ||oracle||_2 <= 1e-3, the oracle
being the C restatement in oracle/ computing the same roundings as the fused
kernel (ROUND_FUSED). The one-ulp allowance only matters above |x| = 4 (bf16)
or 32 (fp16), where one rounding flip caused by a different fp32 summation
order already exceeds 2e-2. The allowance is itself bounded: at most
ULP_FRACTION of the elements (and at least one) may pass only through it, so a
kernel that is off by one ulp on many large outputs still fails.
"""

from __future__ import annotations

import numpy as np

from oracle import oracle as O

MAX_ABS = 2e-2
REL_L2 = 1e-3
ULP_FRACTION = 1e-3


def bits(rng: np.random.Generator, shape, dt: int, scale: float = 1.0) -> np.ndarray:
    """N(0, scale^2) values rounded to fp16 / bf16, as uint16 bit patterns."""
    return O.to16((rng.standard_normal(shape) * scale).astype(np.float32), dt)


def to_torch(a: np.ndarray, dt: int, device="cuda"):
    import torch

    t = torch.from_numpy(np.ascontiguousarray(a, dtype=np.uint16).view(np.int16))
    return t.view(torch.float16 if dt == O.F16 else torch.bfloat16).to(device)


def from_torch(t) -> np.ndarray:
    import torch

    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def ulp(r: np.ndarray, dt: int) -> np.ndarray:
    """Spacing of 16-bit values at |r| (fp16: 11-bit, bf16: 8-bit significand)."""
    bits_ = 10 if dt == O.F16 else 7
    e = np.floor(np.log2(np.maximum(np.abs(r), 1e-30)))
    return np.exp2(e - bits_)


def errors(got: np.ndarray, ref: np.ndarray, dt: int) -> tuple[float, float]:
    """(largest error in units of the per-element bound scaled to MAX_ABS, rel-L2)."""
    g = O.from16(got, dt).astype(np.float64)
    r = O.from16(ref, dt).astype(np.float64)
    if not np.isfinite(g).all():
        return float("inf"), float("inf")
    bound = np.maximum(MAX_ABS, ulp(r, dt) * 1.0001)
    max_abs = float((np.abs(g - r) / bound).max() * MAX_ABS) if g.size else 0.0
    den = float(np.linalg.norm(r))
    rel = float(np.linalg.norm(g - r) / den) if den > 0 else float(np.linalg.norm(g - r))
    return max_abs, rel


def ulp_only(got: np.ndarray, ref: np.ndarray, dt: int) -> int:
    """Elements whose error exceeds MAX_ABS (they pass only through the one-ulp
    allowance, if at all)."""
    g = O.from16(got, dt).astype(np.float64)
    r = O.from16(ref, dt).astype(np.float64)
    return int(np.count_nonzero(np.abs(g - r) > MAX_ABS))


def assert_close(got: np.ndarray, ref: np.ndarray, dt: int, what: str = "") -> None:
    assert got.shape == ref.shape, f"{what}: shape {got.shape} != {ref.shape}"
    max_abs, rel = errors(got, ref, dt)
    n_ulp = ulp_only(got, ref, dt) if np.isfinite(max_abs) else got.size
    allowed = max(1, int(ULP_FRACTION * got.size))
    assert max_abs <= MAX_ABS and rel <= REL_L2 and n_ulp <= allowed, (
        f"{what}: max_abs={max_abs:.3e} (<= {MAX_ABS}), rel_l2={rel:.3e} (<= {REL_L2}), "
        f"{n_ulp} of {got.size} elements beyond {MAX_ABS} within one ulp (<= {allowed})")


def reference_gate(got: np.ndarray, ref: np.ndarray, dt: int) -> bool:
    """The reference's fused-output gate (sequence.py:308-332): fail where
    abs >= 5e-2 AND rel >= 2e-2."""
    g = O.from16(got, dt).astype(np.float64)
    r = O.from16(ref, dt).astype(np.float64)
    a = np.abs(g - r)
    rel = a / np.maximum(np.abs(r), 1e-12)
    return bool(np.all((a < 5e-2) | (rel < 2e-2)))
