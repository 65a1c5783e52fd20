"""CUDA Graph capture with an explicit success/failure result.

Follows decodebench/graph.py:9-88: warm the body on a side stream, capture it
with ``torch.cuda.graph`` (optionally into a shared memory pool), and on failure
return ``Captured(ok=False, reason)``. A failed capture can leave the CUDA RNG
generator registered with the aborted graph; a tiny successful capture clears
that registration, and any error in that clean-up is reported, never raised.
"""

from __future__ import annotations

import warnings
from dataclasses import dataclass, field
from typing import Callable


@dataclass
class Captured:
    ok: bool
    reason: str = ""
    _graph: object = field(default=None, repr=False)

    def replay(self) -> None:
        if not self.ok:
            raise RuntimeError(f"cannot replay: capture failed ({self.reason})")
        self._graph.replay()


def try_capture(body: Callable[[], object], warmup_iters: int = 3, pool=None) -> Captured:
    import torch

    main = torch.cuda.current_stream()
    side = torch.cuda.Stream()
    side.wait_stream(main)
    with torch.cuda.stream(side):
        for _ in range(warmup_iters):
            body()
    main.wait_stream(side)

    g = torch.cuda.CUDAGraph()
    try:
        with torch.cuda.graph(g, pool=pool):
            body()
    except Exception as exc:  # the capture failed: report, clean up, never raise
        reason = f"{type(exc).__name__}: {exc}"
        err = _clear_rng_graph_registration()
        if err:
            reason += (f" [additionally, RNG-registration cleanup failed: {err}; "
                       "torch.randn on this device may raise until the process restarts]")
        return Captured(ok=False, reason=reason)
    return Captured(ok=True, _graph=g)


def _clear_rng_graph_registration() -> str:
    """Run one trivial successful capture; returns '' or a description of the error."""
    import torch

    try:
        if torch.cuda.is_current_stream_capturing():
            return "current stream is still in capture mode; skipped cleanup"
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        scratch = torch.zeros(1, device="cuda")   # allocated before the capture begins
        g = torch.cuda.CUDAGraph()
        with warnings.catch_warnings():
            warnings.simplefilter("ignore")
            with torch.cuda.stream(s):
                g.capture_begin()
                scratch.zero_()
                g.capture_end()
        torch.cuda.current_stream().wait_stream(s)
        del g, scratch
        return ""
    except Exception as exc:
        return f"{type(exc).__name__}: {exc}"
