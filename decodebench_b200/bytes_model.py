"""Byte accounting for an unfused decode chain.

A chain is a list of :class:`StageTrace` records, one per unfused stage. Fusing
the whole chain removes, for every non-final stage, the write of its output and
one read of that output per consumer; the final stage's write survives.

Follows decodebench/bytes_model.py:20-70 (StageTrace fields, validation rules,
``total_bytes`` and ``eliminable_bytes``). Stage-internal temporaries are not
visible here; :meth:`Sequence.trace` warns when a stage allocates more than it
returns.
"""

from __future__ import annotations

from dataclasses import dataclass, field


@dataclass(frozen=True)
class StageTrace:
    """One unfused stage.

    name       label of the stage (the stage function's name)
    reads      bytes read per tensor argument (weights included)
    write      bytes of the stage's output
    is_final   True for the chain's last stage, whose write is not eliminable
    consumers  number of later stage arguments bound to this output
    """

    name: str
    reads: list[int] = field(default_factory=list)
    write: int = 0
    is_final: bool = False
    consumers: int = 1

    def __post_init__(self) -> None:
        if self.write < 0 or min(self.reads, default=0) < 0:
            raise ValueError("StageTrace byte counts must be non-negative")
        if self.consumers < 0:
            raise ValueError("StageTrace consumers must be non-negative")
        if self.consumers == 0 and not self.is_final:
            raise ValueError("non-final StageTrace must have at least one consumer")

    @property
    def bytes(self) -> int:
        return sum(self.reads) + self.write


def total_bytes(traces: list[StageTrace]) -> int:
    """All bytes the unfused chain moves: every read plus every write."""
    return sum(t.bytes for t in traces)


def eliminable_bytes(traces: list[StageTrace]) -> int:
    """Bytes a full fusion removes: (1 + consumers) x write of each non-final stage."""
    return sum(t.write * (t.consumers + 1) for t in traces if not t.is_final)
