"""Sequence: a decode chain of stage functions, traced for bytes and profiled.

Follows decodebench/sequence.py:20-365. The contract a stage must meet:

* ``def name(p1, p2, ...) -> Tensor`` with plain positional parameters and a
  name unique within the chain (sequence.py:27-36);
* each parameter binds, in order of precedence, to an earlier stage's output of
  that name, to the ``inputs`` entry of that name, or (first parameter of a
  non-first stage only) to the previous stage's output (sequence.py:40-59);
* every non-final output is consumed by a later stage (sequence.py:61-93);
* no tensor captured through a closure or global, contiguous tensor arguments,
  one contiguous tensor returned in storage of its own (sequence.py:95-167).

``profile`` times the chain three ways on rotating input replicas: launched
stage by stage (stream), replayed from one CUDA graph per replica (graph), and,
when given, a fused callable (fused) whose output is first checked against the
chain (fail when abs >= 5e-2 AND rel >= 2e-2 anywhere, sequence.py:308-332).
The B200 build's fused stages (:mod:`decodebench_b200.ops`) are such callables.
"""

from __future__ import annotations

import inspect
import warnings
from dataclasses import dataclass
from typing import Any, Callable, Optional

from .bytes_model import StageTrace
from .verdict import DEFAULT_BYTE_THRESHOLD

FUSED_ABS_TOL = 5e-2
FUSED_REL_TOL = 2e-2
_TEMP_WARN_MB = 0.1


def _alloc_counter(torch) -> int:
    """Bytes the stage's tensors asked the caching allocator for, cumulatively.
    Requested bytes, not the rounded block sizes the allocator hands out: a
    block rounded up (or left unsplit) for a stage's own output is not a
    temporary of the stage."""
    st = torch.cuda.memory_stats()
    return st.get("requested_bytes.all.allocated", st["allocated_bytes.all.allocated"])


@dataclass
class _Stage:
    fn: Callable[..., Any]
    name: str
    params: list[str]


class Sequence:
    def __init__(self, name: str):
        self.name = name
        self._stages: list[_Stage] = []

    # ------------------------------------------------------------ registration
    def stage(self, fn):
        params = []
        for p in inspect.signature(fn).parameters.values():
            if p.kind not in (p.POSITIONAL_ONLY, p.POSITIONAL_OR_KEYWORD):
                raise TypeError(
                    f"stage '{fn.__name__}': parameter '{p.name}' is {p.kind.description}; "
                    "stages must use plain positional parameters (no *args/**kwargs/"
                    "keyword-only parameters: arguments are bound by name and position)")
            params.append(p.name)
        if fn.__name__ in (s.name for s in self._stages):
            raise ValueError(f"duplicate stage name '{fn.__name__}'")
        self._stages.append(_Stage(fn, fn.__name__, params))
        return fn

    @property
    def stages(self) -> list[str]:
        return [s.name for s in self._stages]

    # ------------------------------------------------------------ binding
    def _resolve(self, idx: int, j: int, p: str, produced, inputs):
        """Where parameter j of stage idx comes from: ('stage', name) or ('input', name)."""
        if p in produced:
            return "stage", p
        if p in inputs:
            return "input", p
        if idx > 0 and j == 0:
            return "stage", produced[-1] if isinstance(produced, list) else list(produced)[-1]
        raise KeyError(
            f"stage '{self._stages[idx].name}' parameter '{p}' not found in earlier "
            f"stage outputs {list(produced)} or inputs {list(inputs)}")

    def _bind_args(self, stage: _Stage, idx: int, prev_out, inputs, stage_outputs):
        args = []
        for j, p in enumerate(stage.params):
            kind, key = self._resolve(idx, j, p, stage_outputs, inputs)
            if kind == "input":
                args.append(inputs[key])
            elif key == p:
                args.append(stage_outputs[key])
            else:
                args.append(prev_out)
        return args

    def _dependency_consumer_counts(self, inputs) -> dict[str, int]:
        """Validate the static bindings and count the reads of each stage output."""
        produced: list[str] = []
        counts: dict[str, int] = {}
        for idx, st in enumerate(self._stages):
            for j, p in enumerate(st.params):
                kind, key = self._resolve(idx, j, p, produced, inputs)
                if kind == "stage":
                    counts[key] = counts.get(key, 0) + 1
            produced.append(st.name)
        dead = [n for n in produced[:-1] if not counts.get(n)]
        if dead:
            raise ValueError(
                f"non-final stage output(s) {dead} are never consumed by a later stage; "
                "the eliminable-byte model assumes every non-final write has a downstream "
                "read, so this chain is not a valid DecodeBench model")
        return counts

    # ------------------------------------------------------------ execution
    @staticmethod
    def _storage_data_ptr(t) -> int:
        us = getattr(t, "untyped_storage", None)
        return us().data_ptr() if us is not None else t.storage().data_ptr()

    @staticmethod
    def _closure_tensors(fn, torch_module) -> list[str]:
        cv = inspect.getclosurevars(fn)
        return [f"{scope}:{name}"
                for scope, table in (("nonlocal", cv.nonlocals), ("global", cv.globals))
                for name, v in table.items() if isinstance(v, torch_module.Tensor)]

    def _check_stage_io(self, st: _Stage, args, out, torch) -> None:
        if not isinstance(out, torch.Tensor):
            raise TypeError(
                f"stage '{st.name}' must return a single torch.Tensor (got "
                f"{type(out).__name__}). DecodeBench v1 supports linear, single-output "
                "chains only.")
        if not out.is_contiguous():
            raise ValueError(
                f"stage '{st.name}' returned a non-contiguous tensor (shape="
                f"{tuple(out.shape)}, stride={out.stride()}); materialize it explicitly "
                "before using DecodeBench byte accounting")
        if out.nbytes:
            optr = self._storage_data_ptr(out)
            hit = [j for j, a in enumerate(args) if isinstance(a, torch.Tensor)
                   and a.nbytes and self._storage_data_ptr(a) == optr]
            if hit:
                raise ValueError(
                    f"stage '{st.name}' output aliases tensor argument(s) {hit}; "
                    "in-place/view outputs do not represent a materialized stage write")

    def _run_once(self, inputs, _check_temporaries: bool = False):
        import torch

        if not self._stages:
            raise ValueError("Sequence has no stages; register at least one with @seq.stage")
        counts = self._dependency_consumer_counts(inputs)
        watch_alloc = _check_temporaries and torch.cuda.is_available()
        outputs: dict[str, Any] = {}
        io = []
        prev = None
        for idx, st in enumerate(self._stages):
            args = self._bind_args(st, idx, prev, inputs, outputs)
            hidden = self._closure_tensors(st.fn, torch)
            if hidden:
                raise ValueError(
                    f"stage '{st.name}' captures tensor(s) {hidden} outside its declared "
                    "parameters; pass them through inputs so byte accounting can see them")
            for j, a in enumerate(args):
                if isinstance(a, torch.Tensor) and not a.is_contiguous():
                    raise ValueError(
                        f"stage '{st.name}' tensor argument {j} is non-contiguous (shape="
                        f"{tuple(a.shape)}, stride={a.stride()}); materialize it "
                        "explicitly as a declared stage")
            before = _alloc_counter(torch) if watch_alloc else None
            out = st.fn(*args)
            self._check_stage_io(st, args, out, torch)
            if before is not None:
                after = _alloc_counter(torch)
                extra_mb = (after - before - out.nbytes) / 2**20
                if extra_mb > _TEMP_WARN_MB:
                    warnings.warn(
                        f"stage '{st.name}' allocated {extra_mb:.1f} MB internally; byte "
                        "model undercounts — split it into single-op stages", stacklevel=2)
            io.append((st.name, [a for a in args if isinstance(a, torch.Tensor)], out))
            outputs[st.name] = out
            prev = out
        return prev, io, counts

    def _replay_body(self, inp):
        outputs: dict[str, Any] = {}
        prev = None
        for idx, st in enumerate(self._stages):
            prev = st.fn(*self._bind_args(st, idx, prev, inp, outputs))
            outputs[st.name] = prev
        return prev

    def run(self, inputs):
        """Run the chain once (no checks) and return the final output."""
        return self._replay_body(inputs)

    def trace(self, inputs) -> list[StageTrace]:
        _, io, counts = self._run_once(inputs, _check_temporaries=True)
        last = len(io) - 1
        return [StageTrace(name, [t.nbytes for t in reads], out.nbytes, i == last,
                           0 if i == last else counts[name])
                for i, (name, reads, out) in enumerate(io)]

    # ------------------------------------------------------------ profiling
    @staticmethod
    def _validate_replicas(replicas: list[dict]) -> None:
        import torch

        ref = replicas[0]
        for i, rep in enumerate(replicas[1:], start=1):
            if set(rep) != set(ref):
                raise ValueError(
                    f"input replica {i} keys {sorted(rep)} != replica 0 keys {sorted(ref)}")
            for k, a in ref.items():
                b = rep[k]
                if isinstance(a, torch.Tensor) != isinstance(b, torch.Tensor):
                    raise ValueError(f"replica {i}['{k}'] tensor-ness differs from replica 0")
                if isinstance(a, torch.Tensor) and (
                        (b.shape, b.dtype, b.stride(), b.device)
                        != (a.shape, a.dtype, a.stride(), a.device)):
                    raise ValueError(
                        f"replica {i}['{k}'] (shape={tuple(b.shape)}, dtype={b.dtype}, "
                        f"stride={b.stride()}, device={b.device}) does not match replica 0")

    def _check_fused_output(self, fused, inputs, torch) -> None:
        ref = self._replay_body(inputs)
        out = fused(inputs)
        if not isinstance(out, torch.Tensor):
            raise ValueError(f"fused callable must return a single torch.Tensor "
                             f"(got {type(out).__name__})")
        if out.shape != ref.shape:
            raise ValueError(f"fused output shape {tuple(out.shape)} != unfused chain "
                             f"output shape {tuple(ref.shape)}")
        err = (out.float() - ref.float()).abs()
        rel = err / ref.float().abs().clamp_min(1e-12)
        if not bool(((err < FUSED_ABS_TOL) | (rel < FUSED_REL_TOL)).all()):
            raise ValueError(
                f"fused output does not match the unfused chain: max_abs="
                f"{err.max().item():.3e}, max_rel={rel.max().item():.3e} (pass requires "
                f"abs < {FUSED_ABS_TOL:g} or rel < {FUSED_REL_TOL:g} elementwise)")

    def profile(self, inputs, trials: int = 30, target_ms: float = 20.0, warmup: int = 50,
                byte_threshold: float = DEFAULT_BYTE_THRESHOLD, seed: int = 42,
                input_replicas: Optional[list[dict]] = None,
                fused: Optional[Callable[[dict], Any]] = None,
                fused_bytes: Optional[int] = None,
                hbm_peak_gbs: Optional[float] = None):
        """Time stream / graph / fused variants over rotating replicas.

        ``input_replicas``: dicts shaped like ``inputs``; call i uses replica
        i % N so that repeated calls read weights from HBM rather than L2.
        ``fused``: callable(inputs) -> Tensor equal to the chain's output.
        ``fused_bytes`` / ``hbm_peak_gbs``: optional, for the roofline line.
        """
        import torch

        from .graph import try_capture
        from .report import Report
        from .timing import time_callable

        torch.manual_seed(seed)
        reps = list(input_replicas) if input_replicas else [inputs]
        self._validate_replicas(reps)
        # One untraced run first: libraries allocate their workspaces lazily on
        # first use (cuBLAS, for a stage's F.linear or einsum), and the temporary-
        # allocation check would otherwise count that one-time allocation as the
        # stage's own temporaries.
        self._replay_body(reps[0])
        traces = self.trace(reps[0])
        if fused is not None:
            self._check_fused_output(fused, reps[0], torch)

        def rotating(call):
            state = [0]

            def body():
                i = state[0]
                state[0] = i + 1
                return call(i % len(reps))
            return body

        stream_body = rotating(lambda i: self._replay_body(reps[i]))
        # Replica graphs replay strictly one after another, so one private pool serves all.
        make_pool = getattr(torch.cuda, "graph_pool_handle", None)
        pool = make_pool() if make_pool is not None else None
        graphs = [try_capture(lambda r=r: self._replay_body(r), pool=pool) for r in reps]
        failed = next((g for g in graphs if not g.ok), None)
        if failed is not None:
            s = time_callable(stream_body, trials=trials, target_ms=target_ms, warmup=warmup)
            return Report(self.name, s, s, traces, byte_threshold=byte_threshold,
                          graph_ok=False, graph_skip_reason=failed.reason)

        variants = [("stream", stream_body),
                    ("graph", rotating(lambda i: graphs[i].replay()))]
        if fused is not None:
            variants.append(("fused", rotating(lambda i: fused(reps[i]))))
        samples: dict[str, list[float]] = {n: [] for n, _ in variants}
        # Rotate the variant order per round so slow clock/thermal drift is shared.
        rounds = min(3, trials)
        for r in range(rounds):
            n = trials // rounds + (1 if r < trials % rounds else 0)
            k = r % len(variants)
            for name, body in variants[k:] + variants[:k]:
                samples[name] += time_callable(body, trials=n, target_ms=target_ms,
                                               warmup=warmup if r == 0 else min(warmup, 5))
        return Report(self.name, samples["stream"], samples["graph"], traces,
                      fused_us=samples.get("fused"), byte_threshold=byte_threshold,
                      fused_bytes=fused_bytes, hbm_peak_gbs=hbm_peak_gbs)
