"""Report: raw per-trial timings plus byte traces; renders a verdict, writes CSV.

Follows decodebench/report.py:9-48 (fields, verdict refusal after a failed graph
capture, CSV schema ``name,variant,trial,us_per_invocation``). Adds
``fused_bytes`` / ``hbm_peak_gbs`` so the verdict can state the fused path's
GB/s and fraction of the HBM roofline.
"""

from __future__ import annotations

import csv
from dataclasses import dataclass
from typing import Optional

from .bytes_model import StageTrace, eliminable_bytes, total_bytes
from .stats import bootstrap_diff_ci, summarize
from .verdict import DEFAULT_BYTE_THRESHOLD, Verdict, compute_verdict


@dataclass
class Report:
    name: str
    stream_us: list[float]
    graph_us: list[float]
    traces: list[StageTrace]
    fused_us: Optional[list[float]] = None
    byte_threshold: float = DEFAULT_BYTE_THRESHOLD
    graph_ok: bool = True
    graph_skip_reason: str = ""
    fused_bytes: Optional[int] = None
    hbm_peak_gbs: Optional[float] = None

    def verdict(self) -> Verdict:
        if not self.graph_ok:
            raise RuntimeError(
                f"CUDA graph capture failed for '{self.name}': {self.graph_skip_reason}. "
                "Delta_launch is unknown for this chain; no verdict can be emitted.")
        lo, hi, _ = bootstrap_diff_ci(self.stream_us, self.graph_us)
        t_fused = None if self.fused_us is None else summarize(self.fused_us).median
        return compute_verdict(
            t_stream=summarize(self.stream_us).median,
            t_graph=summarize(self.graph_us).median,
            total_bytes=total_bytes(self.traces),
            eliminable_bytes=eliminable_bytes(self.traces),
            byte_threshold=self.byte_threshold,
            delta_launch_ci=(lo, hi),
            t_fused=t_fused,
            fused_bytes=self.fused_bytes if t_fused is not None else None,
            hbm_peak_gbs=self.hbm_peak_gbs if t_fused is not None else None,
        )

    def render(self) -> str:
        return self.verdict().render()

    def rows(self):
        for variant, samples in (("stream", self.stream_us), ("graph", self.graph_us),
                                 ("fused", self.fused_us)):
            if samples is None:
                continue
            for i, t in enumerate(samples):
                yield [self.name, variant, i, t]

    def to_csv(self, path: str) -> None:
        with open(path, "w", newline="") as fh:
            w = csv.writer(fh)
            w.writerow(["name", "variant", "trial", "us_per_invocation"])
            w.writerows(self.rows())
