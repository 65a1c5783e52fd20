"""numpy front end of the CPU oracle (TEST INFRASTRUCTURE ONLY).

Loads ``oracle/_lib/libdbk_oracle.so`` (this repo's C restatement, dbk_oracle.c)
and, when it was built, ``oracle/_ref/libdbref.so`` (the reference's own
cpu_reference.cpp). Only tests/, ``__graft_entry__.smoke()`` and bench.py's
CPU-baseline leg import this module; the product path never does.

16-bit arrays are passed as numpy ``uint16`` bit patterns; helpers convert
between float32 and fp16/bf16 with round-to-nearest-even.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "_lib" / "libdbk_oracle.so"
REF_SO = HERE / "_ref" / "libdbref.so"

F16, BF16 = 0, 1
ROUND_FUSED, ROUND_HARNESS, ROUND_STAGES = 0, 1, 2

_P = ctypes.c_void_p
_I = ctypes.c_int
_F = ctypes.c_float
_SZ = ctypes.c_size_t

_ORC_SIGS = {
    "orc_f16_to_f32": (_F, [ctypes.c_uint16]),
    "orc_f32_to_f16": (ctypes.c_uint16, [_F]),
    "orc_bf16_to_f32": (_F, [ctypes.c_uint16]),
    "orc_f32_to_bf16": (ctypes.c_uint16, [_F]),
    "orc_rmsnorm_f32": (None, [_P, _P, _P, _I, _F]),
    "orc_gemv_f32": (None, [_P, _P, _P, _I, _I]),
    "orc_silu": (_F, [_F]),
    "orc_swiglu_f32": (None, [_P, _P, _P, _I]),
    "orc_softmax_f32": (None, [_P, _P, _I, _I]),
    "orc_attention_f32": (None, [_P, _P, _P, _P, _I, _I, _I]),
    "orc_rmsnorm_gemv": (None, [_P, _P, _P, _P, _I, _I, _I, _F, _I, _I]),
    "orc_gateup_swiglu": (None, [_P, _P, _P, _P, _P, _I, _I, _I, _F, _I, _I]),
    "orc_gemv": (None, [_P, _P, _P, _P, _I, _I, _I, _I]),
    "orc_attention": (None, [_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _F, _I, _I]),
    "orc_splitkv_head": (None, [_P, _P, _P, _P, _I, _I, _F, _I, _I]),
    "orc_to16": (None, [_P, _P, _SZ, _I]),
    "orc_from16": (None, [_P, _P, _SZ, _I]),
}

_REF_SIGS = {
    "ref_rmsnorm": (None, [_P, _P, _P, _I, _F]),
    "ref_gemv": (None, [_P, _P, _P, _I, _I]),
    "ref_silu": (_F, [_F]),
    "ref_swiglu": (None, [_P, _P, _P, _I]),
    "ref_softmax": (None, [_P, _P, _I, _I]),
    "ref_attention": (None, [_P, _P, _P, _P, _I, _I, _I]),
    "ref_gemv_threaded": (None, [_P, _P, _P, _I, _I, _I]),
}

_orc = None
_ref = None


def _bind(path: Path, sigs: dict) -> ctypes.CDLL:
    lib = ctypes.CDLL(str(path))
    for name, (res, args) in sigs.items():
        f = getattr(lib, name)
        f.restype = res
        f.argtypes = args
    return lib


def reference_root() -> Path:
    """The reference checkout: $DBK_REFERENCE_ROOT, else a `reference` directory
    beside this repository's root."""
    env = os.environ.get("DBK_REFERENCE_ROOT")
    return Path(env) if env else HERE.parent.parent / "reference"


def build(ref: bool = True) -> None:
    """Compile the oracle (and the reference's CPU library when its sources exist)."""
    targets = ["oracle"]
    root = reference_root()
    ref_src = root / "validation/src/reference/cpu_reference.cpp"
    if ref and ref_src.exists():
        targets.append("ref")
    subprocess.run(["make", "-s", "-C", str(HERE), *targets, f"REF={root}"], check=True)


def lib() -> ctypes.CDLL:
    global _orc
    if _orc is None:
        if not ORACLE_SO.exists():
            build(ref=False)
        _orc = _bind(ORACLE_SO, _ORC_SIGS)
    return _orc


def have_ref() -> bool:
    return REF_SO.exists()


def ref_lib() -> ctypes.CDLL:
    global _ref
    if _ref is None:
        if not REF_SO.exists():
            raise FileNotFoundError(f"{REF_SO} not built (needs the reference checkout)")
        _ref = _bind(REF_SO, _REF_SIGS)
    return _ref


def _p(a: np.ndarray | None):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


# ------------------------------------------------------------------ conversions
def to16(a: np.ndarray, dt: int) -> np.ndarray:
    src = np.ascontiguousarray(a, dtype=np.float32)
    out = np.empty(src.shape, dtype=np.uint16)
    lib().orc_to16(_p(src), _p(out), src.size, dt)
    return out


def from16(a: np.ndarray, dt: int) -> np.ndarray:
    src = np.ascontiguousarray(a, dtype=np.uint16)
    out = np.empty(src.shape, dtype=np.float32)
    lib().orc_from16(_p(src), _p(out), src.size, dt)
    return out


def _c16(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.uint16)


# ------------------------------------------------------------------ fused ops
def rmsnorm_gemv(x, gamma, W, eps: float, dt: int, round_mode: int = ROUND_FUSED) -> np.ndarray:
    x, gamma, W = _c16(x), _c16(gamma), _c16(W)
    batch, d_in = x.reshape(-1, x.shape[-1]).shape
    d_out = W.shape[0]
    y = np.empty((batch, d_out), dtype=np.uint16)
    lib().orc_rmsnorm_gemv(_p(x), _p(gamma), _p(W), _p(y), batch, d_in, d_out, eps, dt, round_mode)
    return y


def gateup_swiglu(x, Wg, Wu, dt: int, gamma=None, eps: float = 1e-6,
                  round_mode: int = ROUND_FUSED) -> np.ndarray:
    x, Wg, Wu = _c16(x), _c16(Wg), _c16(Wu)
    g = None if gamma is None else _c16(gamma)
    batch, d_in = x.reshape(-1, x.shape[-1]).shape
    d_ff = Wg.shape[0]
    h = np.empty((batch, d_ff), dtype=np.uint16)
    lib().orc_gateup_swiglu(_p(x), _p(g), _p(Wg), _p(Wu), _p(h), batch, d_in, d_ff, eps, dt,
                            round_mode)
    return h


def gemv(x, W, dt: int, residual=None) -> np.ndarray:
    x, W = _c16(x), _c16(W)
    r = None if residual is None else _c16(residual)
    batch, d_in = x.reshape(-1, x.shape[-1]).shape
    d_out = W.shape[0]
    y = np.empty((batch, d_out), dtype=np.uint16)
    lib().orc_gemv(_p(x), _p(W), _p(r), _p(y), batch, d_in, d_out, dt)
    return y


def mlp(x, gamma, Wg, Wu, Wd, eps: float, dt: int, residual=None) -> np.ndarray:
    """gate/up + SwiGLU with RMSNorm prologue (h rounded to dt), then down (+ residual)."""
    h = gateup_swiglu(x, Wg, Wu, dt, gamma=gamma, eps=eps)
    return gemv(h, Wd, dt, residual=residual)


def attention(q, K, V, dt: int, scale: float, seq_lens=None, page_table=None,
              round_mode: int = ROUND_FUSED) -> np.ndarray:
    """q [batch, Hq, D]; contiguous K/V [batch, Hkv, max_len, D] or paged
    [pages, Hkv, page_size, D] with page_table int32 [batch, max_pages]."""
    q, K, V = _c16(q), _c16(K), _c16(V)
    batch, hq, d = q.shape
    if page_table is None:
        _, hkv, max_len, _ = K.shape
        ps, mp, pt = 0, 0, None
    else:
        pt = np.ascontiguousarray(page_table, dtype=np.int32)
        _, hkv, ps, _ = K.shape
        mp = pt.shape[1]
        max_len = ps * mp
    sl = None if seq_lens is None else np.ascontiguousarray(seq_lens, dtype=np.int32)
    out = np.empty_like(q)
    lib().orc_attention(_p(q), _p(K), _p(V), _p(pt), _p(sl), _p(out), batch, hq, hkv, d, max_len,
                        ps, mp, scale, dt, round_mode)
    return out


def splitkv_head(q, K, V, scale: float, splits: int, tile: int = 128) -> np.ndarray:
    q = np.ascontiguousarray(q, dtype=np.float32)
    K = np.ascontiguousarray(K, dtype=np.float32)
    V = np.ascontiguousarray(V, dtype=np.float32)
    L, d = K.shape
    out = np.empty(d, dtype=np.float32)
    lib().orc_splitkv_head(_p(q), _p(K), _p(V), _p(out), L, d, scale, splits, tile)
    return out


# ------------------------------------------------------------------ fp32 primitives
def rmsnorm_f32(x, gamma, eps: float = 1e-6, use_ref: bool = False) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    gamma = np.ascontiguousarray(gamma, np.float32)
    out = np.empty_like(x)
    (ref_lib().ref_rmsnorm if use_ref else lib().orc_rmsnorm_f32)(_p(x), _p(gamma), _p(out),
                                                                   x.size, eps)
    return out


def gemv_f32(W, x, use_ref: bool = False) -> np.ndarray:
    W = np.ascontiguousarray(W, np.float32)
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty(W.shape[0], np.float32)
    (ref_lib().ref_gemv if use_ref else lib().orc_gemv_f32)(_p(W), _p(x), _p(out), W.shape[0],
                                                             W.shape[1])
    return out


def silu(v: float, use_ref: bool = False) -> float:
    return (ref_lib().ref_silu if use_ref else lib().orc_silu)(v)


def swiglu_f32(g, u, use_ref: bool = False) -> np.ndarray:
    g = np.ascontiguousarray(g, np.float32)
    u = np.ascontiguousarray(u, np.float32)
    out = np.empty_like(g)
    (ref_lib().ref_swiglu if use_ref else lib().orc_swiglu_f32)(_p(g), _p(u), _p(out), g.size)
    return out


def softmax_f32(s, use_ref: bool = False) -> np.ndarray:
    s = np.ascontiguousarray(s, np.float32)
    rows, n = s.reshape(-1, s.shape[-1]).shape
    out = np.empty_like(s)
    (ref_lib().ref_softmax if use_ref else lib().orc_softmax_f32)(_p(s), _p(out), rows, n)
    return out


def attention_f32(q, K, V, use_ref: bool = False) -> np.ndarray:
    """Unscaled attention: q [H, D], K/V [H, L, D] (cpu_reference.h attention_ref)."""
    q = np.ascontiguousarray(q, np.float32)
    K = np.ascontiguousarray(K, np.float32)
    V = np.ascontiguousarray(V, np.float32)
    H, L, D = K.shape
    out = np.empty((H, D), np.float32)
    (ref_lib().ref_attention if use_ref else lib().orc_attention_f32)(
        _p(q), _p(K), _p(V), _p(out), H, L, D)
    return out


def ref_gemv_threaded(W, x, threads: int) -> np.ndarray:
    W = np.ascontiguousarray(W, np.float32)
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty(W.shape[0], np.float32)
    ref_lib().ref_gemv_threaded(_p(W), _p(x), _p(out), W.shape[0], W.shape[1], threads)
    return out
