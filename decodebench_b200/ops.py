"""PyTorch-facing fused decode operations (the drop-in fused stages).

Each function validates tensors, allocates the output (and, once per shape, a
zero-filled workspace), and calls the C ABI on the current CUDA stream. No
host synchronisation happens, so every op can be captured in a CUDA graph and
used as a ``Sequence`` stage or as ``Sequence.profile(fused=...)``.

There is deliberately no CPU path: a tensor that is not on a CUDA device, or a
missing kernel library, raises.
"""

from __future__ import annotations

import math
import os
import threading

import torch

from . import _native as N

_DTYPES = {torch.float16: N.DBK_F16, torch.bfloat16: N.DBK_BF16}
_ws_lock = threading.Lock()
_ws_cache: dict[tuple, torch.Tensor] = {}


def _dtype_code(t: torch.Tensor) -> int:
    try:
        return _DTYPES[t.dtype]
    except KeyError:
        raise TypeError(f"decodebench_b200 kernels take float16 or bfloat16, got {t.dtype}")


def _need_cuda(*ts: torch.Tensor) -> torch.device:
    dev = None
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError("decodebench_b200 ops run on CUDA tensors only (no CPU fallback)")
        if not t.is_contiguous():
            raise ValueError("decodebench_b200 ops need contiguous tensors")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError("all tensors must be on the same device")
    return dev


def _check_out(out: torch.Tensor | None, dev: torch.device) -> None:
    """``out`` may be a CUDA tensor on ``dev`` or a pinned CPU tensor: the kernel then
    writes the result straight into host memory (through its unified address), which
    saves the separate copy-out of a decode step. Any other CPU tensor is refused."""
    if out is None:
        return
    if not out.is_contiguous():
        raise ValueError("out must be contiguous")
    if out.is_cuda:
        if out.device != dev:
            raise ValueError("all tensors must be on the same device")
    elif not out.is_pinned():
        raise RuntimeError("out must be a CUDA tensor or a pinned CPU tensor (no CPU fallback)")


def _ptr(t):
    return None if t is None else t.data_ptr()


def workspace_bytes_flashdecode(batch: int, n_q_heads: int, n_kv_heads: int, max_len: int,
                                split_tokens: int = 0) -> int:
    return N.load().dbk_flashdecode_workspace_bytes(batch, n_q_heads, n_kv_heads, max_len,
                                                    split_tokens)


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream(dev: torch.device) -> int:
    """The current CUDA stream of ``dev`` as a raw handle (no Stream object built)."""
    if _raw_stream is not None:
        return _raw_stream(dev.index)
    return torch.cuda.current_stream(dev).cuda_stream


_ws_bytes_cache: dict[tuple, int] = {}


def _ws_bytes(key: tuple, query) -> int:
    """Workspace bytes of an op shape (a pure function of the shape: cached)."""
    nb = _ws_bytes_cache.get(key)
    if nb is None:
        nb = int(query())
        _ws_bytes_cache[key] = nb
    return nb


def _workspace(key: tuple, nbytes: int, device: torch.device,
              given: torch.Tensor | None = None) -> torch.Tensor | None:
    """Zero-filled workspace for one call.

    ``given`` (a caller-owned uint8 CUDA tensor, zero-filled before its first
    use) wins; otherwise one cached workspace per (device, op shape) is reused:
    every kernel leaves its workspace zero-filled again, so calls ordered on one
    stream (or replayed from one graph) may share it. Calls that can run
    concurrently on different streams must each pass their own ``workspace=``.
    """
    if nbytes == 0:
        return None
    if given is not None:
        if given.dtype != torch.uint8 or not given.is_cuda or given.numel() < nbytes:
            raise ValueError(f"workspace must be a uint8 CUDA tensor of >= {nbytes} bytes")
        return given
    full_key = (device.index,) + key
    with _ws_lock:
        ws = _ws_cache.get(full_key)
        if ws is None or ws.numel() < nbytes:
            ws = torch.zeros(nbytes, dtype=torch.uint8, device=device)
            _ws_cache[full_key] = ws
        return ws


def _sharded(name: str, comm, x2: torch.Tensor, d_local: int, out, fused_call, local_call):
    """Column-sharded op followed by the all-gather: [batch, world * d_local].

    ``fused_call(y_full)`` runs the kernel with the exchange in its epilogue; a
    DBK_ESHAPE answer (shape outside the fused variant) falls back to the local
    op plus ``comm.all_gather_rows``."""
    batch = x2.shape[0]
    y = out if out is not None else torch.empty(batch, comm.world * d_local, dtype=x2.dtype,
                                                device=x2.device)
    if tuple(y.shape) != (batch, comm.world * d_local) or not y.is_contiguous():
        raise ValueError(f"out must be contiguous [{batch}, {comm.world * d_local}]")
    st = fused_call(y)
    if st == N.DBK_ESHAPE:
        return comm.all_gather_rows(local_call(), y)
    N.check(name, st)
    return y


def rmsnorm_gemv(x: torch.Tensor, gamma: torch.Tensor, W: torch.Tensor, eps: float = 1e-6,
                 out: torch.Tensor | None = None,
                 workspace: torch.Tensor | None = None, comm=None) -> torch.Tensor:
    """F1: ``linear(rmsnorm(x) * gamma, W)`` for x [batch, d_in], W [d_out, d_in].

    With ``comm`` (a :class:`decodebench_b200.comm.PeerComm`), W holds this rank's
    d_out rows and the result is all-gathered over the ranks inside the kernel:
    [batch, world * d_out], rank p's columns at p * d_out."""
    if comm is not None and comm.world > 1:
        _need_cuda(x, gamma, W, out)
        x2 = x.reshape(-1, x.shape[-1])
        return _sharded("dbk_rmsnorm_gemv_allgather", comm, x2, W.shape[0], out,
                        lambda y: N.load().dbk_rmsnorm_gemv_allgather(
                            comm.handle, x2.data_ptr(), gamma.data_ptr(), W.data_ptr(),
                            y.data_ptr(), x2.shape[0], x2.shape[1], W.shape[0], float(eps),
                            _dtype_code(x), _stream(x.device)),
                        lambda: rmsnorm_gemv(x2, gamma, W, eps=eps, workspace=workspace))
    dev = _need_cuda(x, gamma, W)
    _check_out(out, dev)
    dt = _dtype_code(x)
    if gamma.dtype != x.dtype or W.dtype != x.dtype:
        raise TypeError("x, gamma and W must share one dtype")
    x2 = x.reshape(-1, x.shape[-1])
    batch, d_in = x2.shape
    d_out = W.shape[0]
    if W.shape != (d_out, d_in) or gamma.numel() != d_in:
        raise ValueError(f"shape mismatch: x {tuple(x.shape)}, gamma {tuple(gamma.shape)}, "
                         f"W {tuple(W.shape)}")
    y = out if out is not None else torch.empty(*x.shape[:-1], d_out, dtype=x.dtype, device=dev)
    lib = N.load()
    nb = _ws_bytes(("f1", batch, d_in, d_out),
                   lambda: lib.dbk_workspace_bytes(N.DBK_OP_RMSNORM_GEMV, batch, d_in, d_out))
    ws = _workspace(("f1", batch, d_in, d_out), nb, dev, workspace)
    N.check("dbk_rmsnorm_gemv", lib.dbk_rmsnorm_gemv(
        x2.data_ptr(), gamma.data_ptr(), W.data_ptr(), y.data_ptr(), batch, d_in, d_out,
        float(eps), dt, _ptr(ws), nb, _stream(dev)))
    return y


def gateup_swiglu(x: torch.Tensor, Wg: torch.Tensor, Wu: torch.Tensor,
                  gamma: torch.Tensor | None = None, eps: float = 1e-6,
                  out: torch.Tensor | None = None,
                  workspace: torch.Tensor | None = None, comm=None) -> torch.Tensor:
    """F2: ``silu(x Wg^T) * (x Wu^T)``; with ``gamma``, x is RMS-normalised first.

    With ``comm``, Wg/Wu hold this rank's rows and the result is all-gathered
    inside the kernel ([batch, world * d_ff_local], as rmsnorm_gemv)."""
    if comm is not None and comm.world > 1:
        _need_cuda(x, Wg, Wu, gamma, out)
        x2 = x.reshape(-1, x.shape[-1])
        return _sharded("dbk_gateup_swiglu_allgather", comm, x2, Wg.shape[0], out,
                        lambda y: N.load().dbk_gateup_swiglu_allgather(
                            comm.handle, x2.data_ptr(), _ptr(gamma), Wg.data_ptr(),
                            Wu.data_ptr(), y.data_ptr(), x2.shape[0], x2.shape[1], Wg.shape[0],
                            float(eps), _dtype_code(x), _stream(x.device)),
                        lambda: gateup_swiglu(x2, Wg, Wu, gamma=gamma, eps=eps,
                                              workspace=workspace))
    dev = _need_cuda(x, Wg, Wu, gamma)
    _check_out(out, dev)
    dt = _dtype_code(x)
    x2 = x.reshape(-1, x.shape[-1])
    batch, d_in = x2.shape
    d_ff = Wg.shape[0]
    if Wg.shape != (d_ff, d_in) or Wu.shape != (d_ff, d_in):
        raise ValueError(f"shape mismatch: x {tuple(x.shape)}, Wg {tuple(Wg.shape)}, "
                         f"Wu {tuple(Wu.shape)}")
    if Wg.dtype != x.dtype or Wu.dtype != x.dtype or (gamma is not None and gamma.dtype != x.dtype):
        raise TypeError("all operands must share one dtype")
    h = out if out is not None else torch.empty(*x.shape[:-1], d_ff, dtype=x.dtype, device=dev)
    lib = N.load()
    nb = _ws_bytes(("f2", batch, d_in, d_ff),
                   lambda: lib.dbk_workspace_bytes(N.DBK_OP_GATEUP_SWIGLU, batch, d_in, d_ff))
    ws = _workspace(("f2", batch, d_in, d_ff), nb, dev, workspace)
    N.check("dbk_gateup_swiglu", lib.dbk_gateup_swiglu(
        x2.data_ptr(), _ptr(gamma), Wg.data_ptr(), Wu.data_ptr(), h.data_ptr(), batch, d_in,
        d_ff, float(eps), dt, _ptr(ws), nb, _stream(dev)))
    return h


def gemv(x: torch.Tensor, W: torch.Tensor, residual: torch.Tensor | None = None,
         out: torch.Tensor | None = None, workspace: torch.Tensor | None = None,
         comm=None) -> torch.Tensor:
    """``linear(x, W) (+ residual)`` for x [batch, d_in], W [d_out, d_in].

    With ``comm``, W holds this rank's rows, ``residual`` (optional) is the full
    [batch, world * d_out] tensor, and the result is all-gathered inside the kernel."""
    if comm is not None and comm.world > 1:
        _need_cuda(x, W, residual, out)
        x2 = x.reshape(-1, x.shape[-1])
        d_local = W.shape[0]

        def local():
            r = None
            if residual is not None:
                r = residual.reshape(x2.shape[0], -1)[:, comm.rank * d_local:(comm.rank + 1) * d_local]
                r = r.contiguous()
            return gemv(x2, W, residual=r, workspace=workspace)
        return _sharded("dbk_gemv_allgather", comm, x2, d_local, out,
                        lambda y: N.load().dbk_gemv_allgather(
                            comm.handle, x2.data_ptr(), W.data_ptr(), _ptr(residual),
                            y.data_ptr(), x2.shape[0], x2.shape[1], d_local, _dtype_code(x),
                            _stream(x.device)),
                        local)
    dev = _need_cuda(x, W, residual)
    _check_out(out, dev)
    dt = _dtype_code(x)
    x2 = x.reshape(-1, x.shape[-1])
    batch, d_in = x2.shape
    d_out = W.shape[0]
    if W.shape != (d_out, d_in):
        raise ValueError(f"shape mismatch: x {tuple(x.shape)}, W {tuple(W.shape)}")
    if residual is not None and residual.numel() != batch * d_out:
        raise ValueError("residual must have the output's shape")
    y = out if out is not None else torch.empty(*x.shape[:-1], d_out, dtype=x.dtype, device=dev)
    lib = N.load()
    nb = _ws_bytes(("gemv", batch, d_in, d_out),
                   lambda: lib.dbk_workspace_bytes(N.DBK_OP_GEMV, batch, d_in, d_out))
    ws = _workspace(("gemv", batch, d_in, d_out), nb, dev, workspace)
    N.check("dbk_gemv", lib.dbk_gemv(
        x2.data_ptr(), W.data_ptr(), _ptr(residual), y.data_ptr(), batch, d_in, d_out, dt,
        _ptr(ws), nb, _stream(dev)))
    return y


_MLP_BLOCK = os.environ.get("DBK_MLP_BLOCK", "1") != "0"
_mlp_block_refused: set = set()


def mlp(x: torch.Tensor, gamma: torch.Tensor, Wg: torch.Tensor, Wu: torch.Tensor,
        Wd: torch.Tensor, eps: float = 1e-5, residual: torch.Tensor | None = None) -> torch.Tensor:
    """Decode MLP block: down(silu(gate(rmsnorm(x))) * up(rmsnorm(x))) (+ residual).

    One persistent launch (:func:`mlp_block`) where its shape rules allow, else
    :func:`gateup_swiglu` then :func:`gemv`; the results are bit-identical.
    ``DBK_MLP_BLOCK=0`` in the environment always takes the two launches."""
    key = (x.device.index, x.dtype, x.numel() // x.shape[-1], x.shape[-1], Wg.shape[0])
    if _MLP_BLOCK and key not in _mlp_block_refused:
        try:
            return mlp_block(x, Wg, Wu, Wd, gamma=gamma, eps=eps, residual=residual)
        except N.DbkError as e:
            if e.status != N.DBK_ESHAPE:
                raise
            _mlp_block_refused.add(key)      # refused before any launch
    h = gateup_swiglu(x, Wg, Wu, gamma=gamma, eps=eps)
    return gemv(h, Wd, residual=residual)


def mlp_block(x: torch.Tensor, Wg: torch.Tensor, Wu: torch.Tensor, Wd: torch.Tensor,
              gamma: torch.Tensor | None = None, eps: float = 1e-5,
              residual: torch.Tensor | None = None, out: torch.Tensor | None = None,
              h: torch.Tensor | None = None,
              workspace: torch.Tensor | None = None) -> torch.Tensor:
    """The decode MLP block in one persistent launch (batch 1..4):
    ``Wd @ (silu(Wg x') * (Wu x')) (+ residual)``, x' = RMSNorm(x) with ``gamma``.

    Bit-identical to :func:`gateup_swiglu` followed by :func:`gemv`; the two
    GEMVs meet at a grid-wide barrier inside the kernel instead of a kernel
    boundary. ``h`` (optional, [batch, d_ff]) receives the intermediate
    activation. Raises DbkError (DBK_ESHAPE) for shapes the single launch
    does not cover (see ``dbk_mlp_block`` in dbk.h); :func:`mlp` covers all."""
    dev = _need_cuda(x, Wg, Wu, Wd, gamma, residual)
    _check_out(out, dev)
    _check_out(h, dev)
    dt = _dtype_code(x)
    x2 = x.reshape(-1, x.shape[-1])
    batch, d_model = x2.shape
    d_ff = Wg.shape[0]
    if (Wg.shape != (d_ff, d_model) or Wu.shape != (d_ff, d_model)
            or Wd.shape != (d_model, d_ff)):
        raise ValueError(f"shape mismatch: x {tuple(x.shape)}, Wg {tuple(Wg.shape)}, "
                         f"Wu {tuple(Wu.shape)}, Wd {tuple(Wd.shape)}")
    for t in (Wg, Wu, Wd, gamma, residual):
        if t is not None and t.dtype != x.dtype:
            raise TypeError("all operands must share one dtype")
    if residual is not None and residual.numel() != batch * d_model:
        raise ValueError("residual must have x's shape")
    lib = N.load()
    hbuf = h if h is not None else torch.empty(batch, d_ff, dtype=x.dtype, device=dev)
    if hbuf.numel() != batch * d_ff or not hbuf.is_contiguous():
        raise ValueError("h must be a contiguous [batch, d_ff] tensor")
    y = out if out is not None else torch.empty_like(x)
    ws = _workspace(("mlp_block",), lib.dbk_mlp_block_workspace_bytes(), dev, workspace)
    x2 = x2.contiguous()
    r = residual.contiguous() if residual is not None else None
    N.check("dbk_mlp_block", lib.dbk_mlp_block(
        x2.data_ptr(), _ptr(gamma), Wg.data_ptr(), Wu.data_ptr(), Wd.data_ptr(), _ptr(r),
        hbuf.data_ptr(), y.data_ptr(), batch, d_model, d_ff, float(eps), dt, ws.data_ptr(),
        ws.numel(), _stream(dev)))
    return y


def oproj_mlp_block(attn: torch.Tensor, Wo: torch.Tensor, x: torch.Tensor, Wg: torch.Tensor,
                    Wu: torch.Tensor, Wd: torch.Tensor, gamma: torch.Tensor | None = None,
                    eps: float = 1e-5, out: torch.Tensor | None = None,
                    h_attn: torch.Tensor | None = None, h: torch.Tensor | None = None,
                    workspace: torch.Tensor | None = None) -> torch.Tensor:
    """The rest of a decode layer after attention, in one persistent launch:
    ``h_attn = attn Wo^T + x``, then :func:`mlp_block` on h_attn with h_attn as
    the residual. Bit-identical to :func:`gemv` followed by :func:`mlp_block`.
    ``h_attn`` / ``h`` (optional) receive the two intermediate activations.
    Raises DbkError (DBK_ESHAPE) outside the single launch's shape rules;
    :func:`layer_tail` covers all shapes."""
    dev = _need_cuda(attn, Wo, x, Wg, Wu, Wd, gamma)
    _check_out(out, dev)
    dt = _dtype_code(x)
    a2 = attn.reshape(x.numel() // x.shape[-1], -1)
    batch, d_attn = a2.shape
    d_model = x.shape[-1]
    d_ff = Wg.shape[0]
    if (Wo.shape != (d_model, d_attn) or Wg.shape != (d_ff, d_model)
            or Wu.shape != (d_ff, d_model) or Wd.shape != (d_model, d_ff)):
        raise ValueError(f"shape mismatch: attn {tuple(attn.shape)}, Wo {tuple(Wo.shape)}, "
                         f"x {tuple(x.shape)}, Wg {tuple(Wg.shape)}, Wd {tuple(Wd.shape)}")
    for t in (attn, Wo, Wg, Wu, Wd, gamma):
        if t is not None and t.dtype != x.dtype:
            raise TypeError("all operands must share one dtype")
    lib = N.load()
    ha = h_attn if h_attn is not None else torch.empty(batch, d_model, dtype=x.dtype, device=dev)
    hb = h if h is not None else torch.empty(batch, d_ff, dtype=x.dtype, device=dev)
    for t, n in ((ha, batch * d_model), (hb, batch * d_ff)):
        if t.numel() != n or not t.is_contiguous() or not t.is_cuda:
            raise ValueError("h_attn / h must be contiguous CUDA tensors of [batch, d_model] / "
                             "[batch, d_ff] elements")
    y = out if out is not None else torch.empty_like(x)
    ws = _workspace(("mlp_block",), lib.dbk_mlp_block_workspace_bytes(), dev, workspace)
    N.check("dbk_oproj_mlp_block", lib.dbk_oproj_mlp_block(
        a2.data_ptr(), Wo.data_ptr(), x.data_ptr(), _ptr(gamma), Wg.data_ptr(), Wu.data_ptr(),
        Wd.data_ptr(), ha.data_ptr(), hb.data_ptr(), y.data_ptr(), batch, d_attn, d_model, d_ff,
        float(eps), dt, ws.data_ptr(), ws.numel(), _stream(dev)))
    return y


_LAYER_TAIL = os.environ.get("DBK_LAYER_TAIL", "0") == "1"


def layer_tail(attn: torch.Tensor, Wo: torch.Tensor, x: torch.Tensor, gamma: torch.Tensor,
               Wg: torch.Tensor, Wu: torch.Tensor, Wd: torch.Tensor,
               eps: float = 1e-5) -> torch.Tensor:
    """o_proj + residual, then the MLP block with that result as its residual.

    By default :func:`gemv` then :func:`mlp` (two launches: on one B200 the
    decode layer measured faster this way than with o_proj inside the
    persistent kernel, whose launch then waits for the attention kernel's SMs
    before any Wo byte moves). ``DBK_LAYER_TAIL=1`` in the environment takes
    the single launch (:func:`oproj_mlp_block`) where its shape rules allow. The
    results are bit-identical either way."""
    if _LAYER_TAIL and _MLP_BLOCK:
        key = ("tail", x.device.index, x.dtype, tuple(attn.shape), tuple(x.shape), Wg.shape[0])
        if key not in _mlp_block_refused:
            try:
                return oproj_mlp_block(attn, Wo, x, Wg, Wu, Wd, gamma=gamma, eps=eps)
            except N.DbkError as e:
                if e.status != N.DBK_ESHAPE:
                    raise
                _mlp_block_refused.add(key)      # refused before any launch
    h = gemv(attn.reshape(x.numel() // x.shape[-1], -1), Wo, residual=x)
    return mlp(h, gamma, Wg, Wu, Wd, eps=eps, residual=h)


def flashdecode(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                seq_lens: torch.Tensor | None = None, page_table: torch.Tensor | None = None,
                scale: float | None = None, split_tokens: int = 0,
                out: torch.Tensor | None = None,
                workspace: torch.Tensor | None = None) -> torch.Tensor:
    """F4 split-KV FlashDecode for one query token per sequence.

    q [batch, Hq, 128]. Contiguous caches: k/v [batch, Hkv, max_len, 128].
    Paged caches (``page_table`` int32 [batch, max_pages]): k/v [pages, Hkv, page_size, 128].
    ``seq_lens`` int32 [batch] (device) or None for full length. ``scale``
    defaults to 1/sqrt(128).
    """
    dev = _need_cuda(q, k_cache, v_cache, seq_lens, page_table)
    _check_out(out, dev)
    dt = _dtype_code(q)
    if k_cache.dtype != q.dtype or v_cache.dtype != q.dtype:
        raise TypeError("q, k_cache and v_cache must share one dtype")
    if k_cache.shape != v_cache.shape:
        raise ValueError("k_cache and v_cache must have the same shape")
    q3 = q.reshape(q.shape[0], -1, q.shape[-1])
    batch, hq, d = q3.shape
    if page_table is None:
        if k_cache.dim() != 4 or k_cache.shape[0] != batch:
            raise ValueError("contiguous cache must be [batch, Hkv, max_len, head_dim]")
        _, hkv, max_len, _ = k_cache.shape
        page_size, max_pages = 0, 0
    else:
        if page_table.dtype != torch.int32 or page_table.dim() != 2 or page_table.shape[0] != batch:
            raise ValueError("page_table must be int32 [batch, max_pages]")
        _, hkv, page_size, _ = k_cache.shape
        max_pages = page_table.shape[1]
        max_len = page_size * max_pages
    if seq_lens is not None and (seq_lens.dtype != torch.int32 or seq_lens.numel() != batch):
        raise ValueError("seq_lens must be int32 [batch]")
    if scale is None:
        scale = 1.0 / math.sqrt(d)
    o = out if out is not None else torch.empty_like(q)
    lib = N.load()
    nb = _ws_bytes(("f4", batch, hq, hkv, max_len, split_tokens),
                   lambda: lib.dbk_flashdecode_workspace_bytes(batch, hq, hkv, max_len, split_tokens))
    ws = _workspace(("f4", batch, hq, hkv, max_len, split_tokens), nb, dev, workspace)
    N.check("dbk_flashdecode", lib.dbk_flashdecode(
        q3.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), _ptr(page_table),
        _ptr(seq_lens), o.data_ptr(), batch, hq, hkv, d, max_len, page_size, max_pages,
        float(scale), int(split_tokens), dt, _ptr(ws), nb, _stream(dev)))
    return o


def interleave_rope_rows(Wqkv: torch.Tensor, n_q_heads: int, n_kv_heads: int,
                         head_dim: int = 128) -> torch.Tensor:
    """Wqkv in the usual layout ([q heads | k heads | v heads] x head_dim rows, natural
    dim order) -> the layout qkv_rope_append streams: inside each q and k head, row
    2i = dim i and row 2i + 1 = dim i + head_dim/2 (v heads unchanged). Done once
    when the weights are loaded."""
    h = head_dim // 2
    perm = torch.stack([torch.arange(h), torch.arange(h) + h], dim=1).reshape(-1)
    idx = [perm + head * head_dim for head in range(n_q_heads + n_kv_heads)]
    idx.append(torch.arange((n_q_heads + n_kv_heads) * head_dim,
                            (n_q_heads + 2 * n_kv_heads) * head_dim))
    return Wqkv[torch.cat(idx).to(Wqkv.device)].contiguous()


def rope_inv_freq(head_dim: int = 128, theta: float = 10000.0, device=None) -> torch.Tensor:
    """theta^(-2i/head_dim), i < head_dim/2, in fp32 (as Llama's rotary embedding)."""
    return 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64,
                                         device=device).float() / head_dim))


def qkv_rope_append(x: torch.Tensor, Wqkv_il: torch.Tensor, positions: torch.Tensor,
                    inv_freq: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                    n_q_heads: int, n_kv_heads: int, page_table: torch.Tensor | None = None,
                    gamma: torch.Tensor | None = None, eps: float = 1e-5,
                    out: torch.Tensor | None = None) -> torch.Tensor:
    """QKV projection + RoPE + KV-cache append for one decode token per sequence.

    x [batch, d_in]; Wqkv_il from :func:`interleave_rope_rows`; positions int32
    [batch] (the new token's index = its cache slot); inv_freq fp32 [head_dim/2].
    Paged caches (``page_table`` int32 [batch, max_pages]): [pages, Hkv, page_size, D];
    contiguous: [batch, Hkv, max_len, D]. k and v are written into the caches in
    place; returns q [batch, Hq, D] (rotated). With ``gamma``, x is RMS-normalised
    first."""
    dev = _need_cuda(x, Wqkv_il, positions, inv_freq, k_cache, v_cache, page_table, gamma, out)
    dt = _dtype_code(x)
    x2 = x.reshape(-1, x.shape[-1])
    batch, d_in = x2.shape
    D = k_cache.shape[-1]
    if Wqkv_il.shape != ((n_q_heads + 2 * n_kv_heads) * D, d_in):
        raise ValueError(f"Wqkv must be [{(n_q_heads + 2 * n_kv_heads) * D}, {d_in}]")
    if positions.dtype != torch.int32 or positions.numel() != batch:
        raise ValueError("positions must be int32 [batch]")
    if inv_freq.dtype != torch.float32 or inv_freq.numel() != D // 2:
        raise ValueError(f"inv_freq must be float32 [{D // 2}]")
    if k_cache.shape != v_cache.shape or k_cache.dtype != x.dtype or k_cache.shape[1] != n_kv_heads:
        raise ValueError("k_cache / v_cache must share x's dtype and be [*, Hkv, slots, D]")
    if page_table is None:
        ps, maxp = k_cache.shape[2], 1
    else:
        if page_table.dtype != torch.int32 or page_table.dim() != 2 or page_table.shape[0] != batch:
            raise ValueError("page_table must be int32 [batch, max_pages]")
        ps, maxp = k_cache.shape[2], page_table.shape[1]
    q = out if out is not None else torch.empty(batch, n_q_heads, D, dtype=x.dtype, device=dev)
    N.check("dbk_qkv_rope_append", N.load().dbk_qkv_rope_append(
        x2.data_ptr(), _ptr(gamma), Wqkv_il.data_ptr(), positions.data_ptr(), inv_freq.data_ptr(),
        q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), _ptr(page_table), batch, d_in,
        n_q_heads, n_kv_heads, D, ps, maxp, float(eps), dt, _stream(dev)))
    return q


def quantize_fp8_rows(W: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-row e4m3 quantisation for the fp8 GEMVs: returns (W8, scale) with
    W ~= scale[:, None] * W8.float(); scale = amax(|row|) / 448 (fp32)."""
    Wf = W.float()
    scale = (Wf.abs().amax(dim=1) / 448.0).clamp_min(1e-30)
    W8 = (Wf / scale[:, None]).to(torch.float8_e4m3fn).contiguous()
    return W8, scale.contiguous()


def gemv_fp8(x: torch.Tensor, W8: torch.Tensor, w_scale: torch.Tensor,
             residual: torch.Tensor | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """``linear(x, scale * W8) (+ residual)``, e4m3 weights with per-row scales, batch <= 8."""
    dev = _need_cuda(x, W8, w_scale, residual, out)
    x2, d_out = x.reshape(-1, x.shape[-1]), W8.shape[0]
    _check_fp8(x2, W8, w_scale)
    y = out if out is not None else torch.empty(*x.shape[:-1], d_out, dtype=x.dtype, device=dev)
    N.check("dbk_gemv_fp8", N.load().dbk_gemv_fp8(
        x2.data_ptr(), W8.data_ptr(), w_scale.data_ptr(), _ptr(residual), y.data_ptr(),
        x2.shape[0], x2.shape[1], d_out, _dtype_code(x), _stream(dev)))
    return y


def rmsnorm_gemv_fp8(x: torch.Tensor, gamma: torch.Tensor, W8: torch.Tensor,
                     w_scale: torch.Tensor, eps: float = 1e-6,
                     out: torch.Tensor | None = None) -> torch.Tensor:
    """F1 with e4m3 weights: ``linear(rmsnorm(x) * gamma, scale * W8)``."""
    dev = _need_cuda(x, gamma, W8, w_scale, out)
    x2, d_out = x.reshape(-1, x.shape[-1]), W8.shape[0]
    _check_fp8(x2, W8, w_scale)
    y = out if out is not None else torch.empty(*x.shape[:-1], d_out, dtype=x.dtype, device=dev)
    N.check("dbk_rmsnorm_gemv_fp8", N.load().dbk_rmsnorm_gemv_fp8(
        x2.data_ptr(), gamma.data_ptr(), W8.data_ptr(), w_scale.data_ptr(), y.data_ptr(),
        x2.shape[0], x2.shape[1], d_out, float(eps), _dtype_code(x), _stream(dev)))
    return y


def gateup_swiglu_fp8(x: torch.Tensor, Wg8: torch.Tensor, g_scale: torch.Tensor,
                      Wu8: torch.Tensor, u_scale: torch.Tensor,
                      gamma: torch.Tensor | None = None, eps: float = 1e-6,
                      out: torch.Tensor | None = None) -> torch.Tensor:
    """F2 with e4m3 weights: ``silu(x (sg Wg8)^T) * (x (su Wu8)^T)``, optional RMSNorm."""
    dev = _need_cuda(x, Wg8, g_scale, Wu8, u_scale, gamma, out)
    x2, d_ff = x.reshape(-1, x.shape[-1]), Wg8.shape[0]
    _check_fp8(x2, Wg8, g_scale)
    _check_fp8(x2, Wu8, u_scale)
    h = out if out is not None else torch.empty(*x.shape[:-1], d_ff, dtype=x.dtype, device=dev)
    N.check("dbk_gateup_swiglu_fp8", N.load().dbk_gateup_swiglu_fp8(
        x2.data_ptr(), _ptr(gamma), Wg8.data_ptr(), g_scale.data_ptr(), Wu8.data_ptr(),
        u_scale.data_ptr(), h.data_ptr(), x2.shape[0], x2.shape[1], d_ff, float(eps),
        _dtype_code(x), _stream(dev)))
    return h


def _check_fp8(x2, W8, scale):
    if W8.dtype != torch.float8_e4m3fn:
        raise TypeError(f"fp8 weights must be torch.float8_e4m3fn, got {W8.dtype}")
    if scale.dtype != torch.float32 or scale.numel() != W8.shape[0]:
        raise ValueError("scale must be float32 with one value per weight row")
    if W8.dim() != 2 or W8.shape[1] != x2.shape[1]:
        raise ValueError(f"shape mismatch: x {tuple(x2.shape)}, W8 {tuple(W8.shape)}")


def stage(dst: torch.Tensor, src: torch.Tensor) -> torch.Tensor:
    """Copy a decode step's input in, or its result out, with a small kernel.

    One side is a CUDA tensor, the other a pinned CPU tensor (or CUDA too); both
    contiguous with the same byte size. Runs on the CUDA side's current stream,
    like ``dst.copy_(src, non_blocking=True)``, but without a copy-engine
    transfer's fixed latency, and a following decode kernel can start streaming
    its weights while the input arrives. Read a host ``dst`` only after the
    stream has completed."""
    dev = dst.device if dst.is_cuda else src.device
    if dev.type != "cuda":
        raise RuntimeError("stage: one side must be a CUDA tensor")
    if not (dst.is_contiguous() and src.is_contiguous()):
        raise ValueError("stage: tensors must be contiguous")
    nb = dst.numel() * dst.element_size()
    if nb != src.numel() * src.element_size():
        raise ValueError("stage: byte sizes differ")
    st = N.load().dbk_copy(dst.data_ptr(), src.data_ptr(), nb, _stream(dev))
    if st != 0:
        for t in (dst, src):     # the usual cause: pageable host memory
            if not t.is_cuda and not t.is_pinned():
                raise ValueError("stage: a CPU tensor must be pinned (pin_memory())")
        N.check("dbk_copy", st)
    return dst


def take_device_error() -> int:
    """Error code a kernel recorded after a bounded wait gave up (0 = none); clears it.

    A kernel that gave up may have left arrival counters of its workspace
    non-zero (a partial it never merged), so on a non-zero code the cached
    workspaces are dropped: later calls start from fresh zero-filled ones.
    Synchronises the current device."""
    code = N.load().dbk_take_device_error()
    if code != 0:
        with _ws_lock:
            _ws_cache.clear()
    return code


def check_device_error() -> None:
    """Raise RuntimeError if a kernel recorded a bounded-wait failure since the last
    check (see :func:`take_device_error`); synchronises the current device."""
    code = take_device_error()
    if code > 0 and code < 16:
        raise RuntimeError(f"a decodebench_b200 kernel gave up a bounded wait (device error {code}); "
                           "its outputs are not valid")
    if code != 0:
        raise RuntimeError(f"dbk_take_device_error failed: {N.load().dbk_status_string(code)!r}")


def set_spin_limit(polls: int = 0) -> None:
    """Poll budget of the kernels' bounded waits on the current device (0 = default)."""
    N.check("set_spin_limit", N.load().dbk_set_spin_limit(int(polls)))
