"""Launch-overhead vs eliminable-byte verdict.

Follows decodebench/verdict.py:17-114.

* delta_launch = t_stream - t_graph (measured)
* B = eliminable_bytes / (total_bytes / t_graph): the time the eliminable bytes
  would take at the chain's average byte throughput (an estimate, not a bound)
* bound = "material-byte-opportunity" when B >= byte_threshold * t_graph
* residual = (t_graph - t_fused) - B when a fused time is known

The B200 build adds optional roofline fields: when the caller knows the HBM peak
(GB/s) and the fused kernel's algorithmic bytes, ``fused_gbs`` and
``fused_frac`` report the fused path against that roofline.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional

DEFAULT_BYTE_THRESHOLD = 0.01

LOW = "low-byte-opportunity"
MATERIAL = "material-byte-opportunity"


@dataclass(frozen=True)
class Verdict:
    t_stream: float
    t_graph: float
    delta_launch: float
    b_bytes_est: float
    achieved_bw: float          # bytes per us of the unfused graph
    total_bytes: int
    eliminable_bytes: int
    byte_threshold: float
    bound: str
    dominant: str               # "launch" or "bytes"
    delta_launch_ci: Optional[tuple[float, float]] = None
    t_fused: Optional[float] = None
    residual_us: Optional[float] = None
    fused_bytes: Optional[int] = None
    hbm_peak_gbs: Optional[float] = None

    @property
    def b_ceiling(self) -> float:
        """Older name of :attr:`b_bytes_est`."""
        return self.b_bytes_est

    @property
    def fused_gbs(self) -> Optional[float]:
        if self.t_fused is None or self.fused_bytes is None:
            return None
        return self.fused_bytes / self.t_fused / 1e3

    @property
    def fused_frac(self) -> Optional[float]:
        g = self.fused_gbs
        if g is None or not self.hbm_peak_gbs:
            return None
        return g / self.hbm_peak_gbs

    def render(self) -> str:
        out = []
        spans_zero = False
        ci_txt = ""
        if self.delta_launch_ci is not None:
            lo, hi = self.delta_launch_ci
            ci_txt = f" (95% CI [{lo:.2f}, {hi:.2f}])"
            spans_zero = lo <= 0.0 <= hi
        if spans_zero:
            out.append(f"Measured launch saving {self.delta_launch:.2f} us{ci_txt} is "
                       "statistically indistinguishable from zero (CI spans 0).")
        else:
            out.append(f"CUDA Graphs eliminate {self.delta_launch:.2f} us here{ci_txt} (measured).")
        out.append(f"Eliminable intermediate bytes correspond to ~{self.b_bytes_est:.2f} us at "
                   "this workload's average byte throughput (analytic proportional "
                   "estimate, NOT a strict bound).")
        out.append(f"Floor with graphs on (t_graph): {self.t_graph:.2f} us.")
        dom = ("launch overhead (measured)" if self.dominant == "launch"
               else "eliminable bytes (estimated)")
        out.append(f"Dominant term: {dom} (delta_launch {self.delta_launch:.2f} us vs "
                   f"B {self.b_bytes_est:.2f} us).")
        if self.t_fused is not None and self.residual_us is not None:
            out.append(f"Measured fused latency: {self.t_fused:.2f} us.")
            total = self.delta_launch + self.b_bytes_est + self.residual_us
            out.append(f"Decomposition: launch overhead {self.delta_launch:.2f} us + "
                       f"eliminable bytes {self.b_bytes_est:.2f} us + unexplained residual "
                       f"{self.residual_us:.2f} us = {total:.2f} us (t_stream - t_fused).")
            g = self.fused_gbs
            if g is not None:
                line = f"Fused path: {g:.1f} GB/s over {self.fused_bytes} algorithmic bytes"
                f = self.fused_frac
                if f is not None:
                    line += f" = {100.0 * f:.1f}% of {self.hbm_peak_gbs:.0f} GB/s HBM peak"
                out.append(line + ".")
        if self.bound == LOW:
            advice = ("enable CUDA Graphs first; the declared byte fraction is below the "
                      "configured fusion threshold.")
        else:
            advice = ("the declared byte fraction clears the threshold; benchmark a "
                      "representative fused kernel before committing.")
        out.append(f"Verdict: {self.bound.upper()} -> {advice}")
        if self.bound == MATERIAL and self.dominant == "launch":
            out.append("Caution: measured launch savings exceed the byte estimate; the "
                       "material-byte-opportunity classification reflects the analytic byte "
                       "fraction, not the empirically dominant source of gain.")
        return "\n".join(out)


def _finite(v: float) -> bool:
    return isinstance(v, (int, float)) and math.isfinite(v)


def compute_verdict(t_stream: float, t_graph: float, total_bytes: int,
                    eliminable_bytes: int, byte_threshold: float = DEFAULT_BYTE_THRESHOLD,
                    delta_launch_ci: Optional[tuple[float, float]] = None,
                    t_fused: Optional[float] = None,
                    fused_bytes: Optional[int] = None,
                    hbm_peak_gbs: Optional[float] = None) -> Verdict:
    if not (_finite(t_stream) and _finite(t_graph)) or t_stream <= 0:
        raise ValueError("t_stream and t_graph must be finite, and t_stream must be positive")
    if t_graph <= 0:
        raise ValueError("t_graph must be positive (us)")
    if t_fused is not None and (not _finite(t_fused) or t_fused <= 0):
        raise ValueError("t_fused must be finite and positive (us) when provided")
    if total_bytes <= 0:
        raise ValueError("total_bytes must be positive")
    if eliminable_bytes < 0 or eliminable_bytes > total_bytes:
        raise ValueError("eliminable_bytes must be in [0, total_bytes]")
    if not _finite(byte_threshold) or byte_threshold < 0 or byte_threshold > 1:
        raise ValueError("byte_threshold must be finite and in [0, 1]")
    if delta_launch_ci is not None:
        lo, hi = delta_launch_ci
        if not (_finite(lo) and _finite(hi)) or lo > hi:
            raise ValueError("delta_launch_ci must contain finite ordered bounds")
    if fused_bytes is not None and fused_bytes <= 0:
        raise ValueError("fused_bytes must be positive when provided")
    if hbm_peak_gbs is not None and (not _finite(hbm_peak_gbs) or hbm_peak_gbs <= 0):
        raise ValueError("hbm_peak_gbs must be finite and positive when provided")

    bw = total_bytes / t_graph
    b_est = eliminable_bytes / bw
    d_launch = t_stream - t_graph
    return Verdict(
        t_stream=t_stream, t_graph=t_graph, delta_launch=d_launch, b_bytes_est=b_est,
        achieved_bw=bw, total_bytes=total_bytes, eliminable_bytes=eliminable_bytes,
        byte_threshold=byte_threshold,
        bound=MATERIAL if b_est >= byte_threshold * t_graph else LOW,
        dominant="launch" if d_launch >= b_est else "bytes",
        delta_launch_ci=delta_launch_ci, t_fused=t_fused,
        residual_us=None if t_fused is None else (t_graph - t_fused) - b_est,
        fused_bytes=fused_bytes, hbm_peak_gbs=hbm_peak_gbs,
    )
