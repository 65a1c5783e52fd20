"""CUDA-event timing with an adaptive iteration count, and L2-defeating replicas.

Follows decodebench/timing.py:8-65:

* ``n_weight_replicas`` = min(8, max(4, ceil(2 * L2 / weight_bytes))): rotate that
  many copies of the weights so consecutive invocations read HBM, not L2;
* ``time_callable``: ``warmup`` calls, a 5-call probe, then ``trials`` batches of
  K = clamp(ceil(target_ms / t_probe), 200, 1e6) back-to-back calls between two
  CUDA events on the current stream; returns microseconds per call per trial.
"""

from __future__ import annotations

import math
from typing import Callable

_PROBE_CALLS = 5
_MIN_K, _MAX_K = 200, 1_000_000


def device_l2_bytes(device=None) -> int:
    import torch

    props = torch.cuda.get_device_properties(
        torch.cuda.current_device() if device is None else device)
    l2 = getattr(props, "L2_cache_size", None)
    if l2 is None:
        l2 = getattr(props, "l2_cache_size")
    return int(l2)


def n_weight_replicas(weight_bytes: int, l2_bytes: int | None = None) -> int:
    """Copies of the weights needed so that a round-robin over them misses L2."""
    if weight_bytes <= 0:
        raise ValueError("weight_bytes must be positive")
    if l2_bytes is None:
        l2_bytes = device_l2_bytes()
    if l2_bytes is None or l2_bytes < 0:
        raise ValueError("l2_bytes must be non-negative")
    return min(8, max(4, math.ceil(2 * l2_bytes / weight_bytes)))


def time_callable(fn: Callable[[], object], trials: int = 30, target_ms: float = 20.0,
                  warmup: int = 50) -> list[float]:
    """Microseconds per invocation of ``fn`` (one invocation per call), per trial."""
    if trials <= 0:
        raise ValueError("trials must be positive")
    if not (isinstance(target_ms, (int, float)) and math.isfinite(target_ms)) or target_ms <= 0:
        raise ValueError("target_ms must be finite and positive")
    if warmup < 0:
        raise ValueError("warmup must be non-negative")

    import torch

    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()

    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(_PROBE_CALLS):
        fn()
    t1.record()
    torch.cuda.synchronize()
    per_call_ms = max(t0.elapsed_time(t1) / _PROBE_CALLS, 1e-4)
    k = max(_MIN_K, min(_MAX_K, math.ceil(target_ms / per_call_ms)))

    out = []
    for _ in range(trials):
        t0.record()
        for _ in range(k):
            fn()
        t1.record()
        torch.cuda.synchronize()
        out.append(t0.elapsed_time(t1) * 1000.0 / k)
    return out
