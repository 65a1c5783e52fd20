"""Generate golden fixtures from the reference's own PyTorch stage code (CPU).

Run where the reference checkout is present ($DBK_REFERENCE_ROOT, else a
``reference`` directory beside this repository):

    python tests/golden/make_golden.py [--ref /path/to/Decodebench]

It imports ``decodebench.demos.llama_decode`` from the reference, builds the F1,
F2 and F4 chains on the CPU (``torch.randn`` device argument dropped, replicas
stubbed), takes the registered stage functions -- rmsnorm/gemv
(llama_decode.py:36-43), gate/up/swiglu (:77-87), scores/softmax/weighted_v
(:120-134) -- and runs them through ``Sequence._replay_body`` on small seeded
inputs. Inputs and outputs are stored as raw 16-bit patterns in
``golden_<name>.npz`` beside this script. The GPU box never needs the reference.
"""

from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def _load_reference(ref: Path):
    import torch

    sys.path.insert(0, str(ref / "src"))
    import decodebench.demos.llama_decode as ld  # the reference module

    real_randn = torch.randn

    def cpu_randn(*shape, dtype=None, device=None, **kw):
        return real_randn(*shape, dtype=dtype, **kw)

    torch.randn = cpu_randn
    ld.n_weight_replicas = lambda nbytes: 1
    try:
        chains = {name: ld.build_demo(name, dim=2048, batch=1)[0] for name in ("f1", "f2", "f4")}
    finally:
        torch.randn = real_randn
    return chains


def _h(rng, shape, scale=1.0):
    return (rng.standard_normal(shape) * scale).astype(np.float16)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=None,
                    help="reference checkout (default: $DBK_REFERENCE_ROOT, else ../reference "
                         "beside this repository)")
    args = ap.parse_args()
    import torch

    ref = args.ref or os.environ.get("DBK_REFERENCE_ROOT") or str(
        Path(__file__).resolve().parents[3] / "reference")
    chains = _load_reference(Path(ref))
    rng = np.random.default_rng(42)
    T = torch.from_numpy
    cases = {}

    # F1 rmsnorm(eps 1e-6, two fp16 roundings) -> linear
    for name, (b, din, dout) in {"f1": (2, 256, 384), "f1_ragged": (1, 72, 37)}.items():
        x, g, W = _h(rng, (b, din)), _h(rng, (din,)), _h(rng, (dout, din), 1 / 16)
        y = chains["f1"]._replay_body({"x": T(x), "g": T(g), "W": T(W)})
        cases[name] = dict(x=x, g=g, W=W, y=y.numpy())

    # F2 gate, up, silu(gate) * up
    b, din, dff = 2, 256, 192
    xh, Wg, Wu = _h(rng, (b, din)), _h(rng, (dff, din), 1 / 16), _h(rng, (dff, din), 1 / 16)
    h = chains["f2"]._replay_body({"xh": T(xh), "Wg": T(Wg), "Wu": T(Wu)})
    cases["f2"] = dict(xh=xh, Wg=Wg, Wu=Wu, y=h.numpy())

    # F4 unscaled scores -> fp32 softmax -> p.half() @ V ; q ~ N(0, 1/128) so that
    # the unscaled scores have unit variance.
    b, H, L, D = 2, 2, 200, 128
    q, K, V = _h(rng, (b, H, D), 128 ** -0.5), _h(rng, (b, H, L, D)), _h(rng, (b, H, L, D))
    o = chains["f4"]._replay_body({"q": T(q), "K": T(K), "V": T(V)})
    cases["f4"] = dict(q=q, K=K, V=V, y=o.numpy())

    for name, arrs in cases.items():
        np.savez_compressed(HERE / f"golden_{name}.npz",
                            **{k: np.ascontiguousarray(v).view(np.uint16) for k, v in arrs.items()})
        print(name, {k: v.shape for k, v in arrs.items()})


if __name__ == "__main__":
    main()
