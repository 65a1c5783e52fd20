"""``decodebench`` command line: demo, profile, sweep.

Follows src/decodebench/cli.py:16-170 (sub-commands, options, dry-run lines,
exit codes: 2 for a malformed profile target, 1 for a missing GPU or a failed
verdict). The B200 build adds ``--no-fused``: by default ``demo`` and ``sweep``
also time the fused sm_100a kernel for the chain and report its GB/s against
the HBM peak (``MEASURED_PEAKS.json`` when present).
"""

from __future__ import annotations

import argparse
import csv
import importlib.util
import json
import os
import sys
from pathlib import Path

from .verdict import DEFAULT_BYTE_THRESHOLD


def parse_comma_list(s: str) -> list[int]:
    try:
        return [int(v) for v in (p.strip() for p in s.split(",")) if v]
    except ValueError:
        raise argparse.ArgumentTypeError(f"Invalid comma-separated list: '{s}'")


def build_parser() -> argparse.ArgumentParser:
    ap = argparse.ArgumentParser(
        prog="decodebench",
        description="DecodeBench (B200): compare launch overhead with an analytic "
                    "eliminable-byte estimate in LLM decode fusion, and time fused "
                    "sm_100a kernels against the HBM roofline.")
    sub = ap.add_subparsers(dest="command", required=True)

    d = sub.add_parser("demo", help="Run a bundled Llama-decode demo.")
    d.add_argument("name", choices=["f1", "f2", "f4", "layer"], help="Demo name.")
    d.add_argument("--dim", type=int, choices=[2048, 4096], default=4096, help="Hidden dimension.")
    d.add_argument("--batch", type=int, default=1, help="Batch size.")
    d.add_argument("--trials", type=int, default=30, help="Number of timing trials.")
    d.add_argument("--byte-threshold", type=float, default=DEFAULT_BYTE_THRESHOLD,
                   help="Byte ratio threshold.")
    d.add_argument("--csv", type=str, help="Output path for trial CSV.")
    d.add_argument("--no-fused", action="store_true", help="Skip the fused sm_100a kernel.")
    d.add_argument("--dry-run", action="store_true", help="Print plan and exit.")

    p = sub.add_parser("profile", help="Profile a user-defined Sequence chain.")
    p.add_argument("target", help="Target sequence wrapper (path/to/module.py:build_fn).")
    p.add_argument("--trials", type=int, default=30, help="Number of timing trials.")
    p.add_argument("--byte-threshold", type=float, default=DEFAULT_BYTE_THRESHOLD,
                   help="Byte ratio threshold.")
    p.add_argument("--csv", type=str, help="Output path for trial CSV.")
    p.add_argument("--dry-run", action="store_true", help="Print plan and exit.")

    s = sub.add_parser("sweep", help="Sweep batch sizes and hidden dims for a demo.")
    s.add_argument("name", choices=["f1", "f2", "f4", "layer"], help="Demo name.")
    s.add_argument("--batch", type=parse_comma_list, default=[1, 2, 4, 8],
                   help="Comma-separated batch sizes to sweep.")
    s.add_argument("--dim", type=int, choices=[2048, 4096], default=4096, help="Hidden dimension.")
    s.add_argument("--trials", type=int, default=30, help="Number of timing trials.")
    s.add_argument("--csv", type=str, help="Output path for sweep summary CSV.")
    s.add_argument("--no-fused", action="store_true", help="Skip the fused sm_100a kernel.")
    s.add_argument("--dry-run", action="store_true", help="Print plan and exit.")
    return ap


def hbm_peak_gbs() -> float | None:
    """Measured HBM copy bandwidth from MEASURED_PEAKS.json next to the package, if any."""
    for cand in (os.environ.get("DBK_PEAKS"), Path(__file__).resolve().parent.parent /
                 "MEASURED_PEAKS.json"):
        if cand and Path(cand).exists():
            try:
                return float(json.loads(Path(cand).read_text())["hbm_gbs"])
            except (KeyError, ValueError, OSError):
                return None
    return None


def _need_gpu() -> bool:
    import torch

    if not torch.cuda.is_available():
        print("Error: GPU/CUDA is not available.", file=sys.stderr)
        return False
    return True


def _fused_bytes(name: str, inputs: dict) -> int:
    from . import costs

    if name == "f1":
        b, d = inputs["x"].shape
        return costs.rmsnorm_gemv_bytes(b, d, inputs["W"].shape[0])
    if name == "f2":
        b, d = inputs["xh"].shape
        return costs.gateup_swiglu_bytes(b, d, inputs["Wg"].shape[0])
    if name == "layer":
        # every weight once, the cached K/V of each sequence once, x in, y out
        w = sum(inputs[k].nbytes for k in ("Wqkv_il", "Wo", "Wg", "Wu", "Wd"))
        b, hkv, _, dh = inputs["Kc"].shape
        kv = 2 * int(inputs["lens"].sum().item()) * hkv * dh * inputs["Kc"].element_size()
        return w + kv + 2 * inputs["x"].nbytes
    b, h, L, dh = inputs["K"].shape
    return costs.flashdecode_bytes([L] * b, h, h, dh)


def _run_demo(name, dim, batch, trials, threshold, fused_on):
    from .demos.llama_decode import build_demo

    seq, inputs, reps, fused = build_demo(name, dim=dim, batch=batch)
    kw = {}
    if fused_on:
        kw = dict(fused=fused, fused_bytes=_fused_bytes(name, inputs), hbm_peak_gbs=hbm_peak_gbs())
    return seq.profile(inputs, trials=trials, byte_threshold=threshold, input_replicas=reps, **kw)


def main(argv: list[str] | None = None) -> int:
    args = build_parser().parse_args(argv)

    if args.command == "demo":
        if args.dry_run:
            print(f"[dry-run] demo {args.name} with dim={args.dim}, batch={args.batch}, "
                  f"trials={args.trials}, threshold={args.byte_threshold}")
            return 0
        if not _need_gpu():
            return 1
        report = _run_demo(args.name, args.dim, args.batch, args.trials, args.byte_threshold,
                           not args.no_fused)
        try:
            print(report.render())
        except RuntimeError as e:
            print(f"Error: {e}", file=sys.stderr)
            return 1
        if args.csv:
            report.to_csv(args.csv)
            print(f"Saved trials to {args.csv}")
        return 0

    if args.command == "profile":
        if ":" not in args.target:
            print("Error: Target must be in the format 'path/to/module.py:build_fn'", file=sys.stderr)
            return 2
        path, fn_name = args.target.split(":", 1)
        if args.dry_run:
            print(f"[dry-run] profile target {path}:{fn_name} with trials={args.trials}, "
                  f"threshold={args.byte_threshold}")
            return 0
        if not os.path.exists(path):
            print(f"Error: Module path '{path}' does not exist.", file=sys.stderr)
            return 1
        try:
            spec = importlib.util.spec_from_file_location("user_module", path)
            if spec is None or spec.loader is None:
                raise ImportError(f"Cannot load module from {path}")
            mod = importlib.util.module_from_spec(spec)
            spec.loader.exec_module(mod)
            build_fn = getattr(mod, fn_name)
        except Exception as e:
            print(f"Error loading target: {e}", file=sys.stderr)
            return 1
        if not _need_gpu():
            return 1
        seq, inputs = build_fn()[:2]
        report = seq.profile(inputs, trials=args.trials, byte_threshold=args.byte_threshold)
        try:
            print(report.render())
        except RuntimeError as e:
            print(f"Error: {e}", file=sys.stderr)
            return 1
        if args.csv:
            report.to_csv(args.csv)
            print(f"Saved trials to {args.csv}")
        return 0

    # sweep
    if args.dry_run:
        print(f"[dry-run] sweep demo {args.name} with batch={args.batch}, dim={args.dim}, "
              f"trials={args.trials}")
        return 0
    if not _need_gpu():
        return 1
    rows = []
    for b in args.batch:
        print(f"Sweeping {args.name} dim={args.dim} batch={b}...")
        report = _run_demo(args.name, args.dim, b, args.trials, DEFAULT_BYTE_THRESHOLD,
                           not args.no_fused)
        try:
            v = report.verdict()
        except RuntimeError as e:
            print(f"  WARN: {e}", file=sys.stderr)
            continue
        lo, hi = v.delta_launch_ci if v.delta_launch_ci else (0.0, 0.0)
        fused = f" | Fused: {v.t_fused:.2f} us" if v.t_fused is not None else ""
        print(f"  Stream: {v.t_stream:.2f} us | Graph: {v.t_graph:.2f} us{fused} | Bound: {v.bound}")
        rows.append([args.name, args.dim, b, args.trials, f"{v.t_stream:.2f}", f"{v.t_graph:.2f}",
                     f"{v.delta_launch:.2f}", f"{v.b_bytes_est:.2f}", v.bound, v.total_bytes,
                     v.eliminable_bytes, f"{lo:.2f}", f"{hi:.2f}",
                     "" if v.t_fused is None else f"{v.t_fused:.2f}",
                     "" if v.fused_gbs is None else f"{v.fused_gbs:.1f}"])
    if args.csv:
        with open(args.csv, "w", newline="") as fh:
            w = csv.writer(fh)
            w.writerow(["demo", "dim", "batch", "trials", "t_stream_us", "t_graph_us",
                        "delta_launch_us", "b_bytes_est_us", "bound", "total_bytes",
                        "eliminable_bytes", "ci_lo", "ci_hi", "t_fused_us", "fused_gbs"])
            w.writerows(rows)
        print(f"Saved sweep results to {args.csv}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
