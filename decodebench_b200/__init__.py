"""decodebench_b200: the DecodeBench decode hot path rebuilt for B200 (sm_100a).

CPU-only analysis modules import eagerly; torch and the kernel library load
lazily (``decodebench_b200.ops``).
"""

__version__ = "0.1.0"

from .bytes_model import StageTrace, eliminable_bytes, total_bytes
from .report import Report
from .sequence import Sequence
from .stats import Summary, bootstrap_diff_ci, summarize
from .verdict import Verdict, compute_verdict

__all__ = ["__version__", "StageTrace", "eliminable_bytes", "total_bytes", "Verdict",
           "compute_verdict", "Report", "Summary", "bootstrap_diff_ci", "summarize", "Sequence"]
