"""Sharding of the decode hot path over the GPUs of one node.

One process per GPU (``torch.distributed``, NCCL over NVLink; gloo on CPU for
tests). The path partitions with a single exchange at the shard boundary:

* F1 / F2 / GEMV: weight rows (output features) are split into contiguous,
  balanced ranges; every rank computes its output columns from the replicated
  activation; one all-gather reassembles the output in rank order.
* Decode MLP: gate/up rows sharded -> all-gather of h -> down rows sharded ->
  all-gather of y.
* FlashDecode: kv heads are split (each with its query heads), so every rank
  sees every sequence and the load stays balanced; one all-gather of the output.

The reference (animeshsri14/Decodebench) is single-GPU and has no collective;
this module is the B200 build's multi-GPU layer.
"""

from __future__ import annotations

from typing import Callable


def row_range(n: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous, balanced [start, stop) of n items for rank (sizes differ by <= 1)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} for world {world}")
    return n * rank // world, n * (rank + 1) // world


def shard_rows(W, rank: int, world: int):
    """Rows [row_range] of a [rows, ...] tensor (a view; contiguous for row-major W)."""
    a, b = row_range(W.shape[0], rank, world)
    return W[a:b]


def shard_heads(q, k_cache, v_cache, rank: int, world: int, paged: bool = False):
    """Split kv heads (and their query heads): q [batch, Hq, D];
    contiguous caches [batch, Hkv, L, D] or paged [pages, Hkv, ps, D]."""
    hkv = k_cache.shape[1]
    if hkv % world:
        raise ValueError(f"{hkv} kv heads do not split over {world} ranks")
    g = q.shape[1] // hkv
    a, b = row_range(hkv, rank, world)
    return (q[:, a * g:b * g].contiguous(), k_cache[:, a:b].contiguous(),
            v_cache[:, a:b].contiguous())


def gather_last_dim(local, group=None, sizes: list[int] | None = None):
    """All-gather rank-local column blocks [..., n_r] into [..., sum n_r] in rank order.

    ``sizes`` (every rank's block width) avoids a size handshake, which would
    synchronise the host and break CUDA-graph capture; without it the widths are
    exchanged first. Blocks are padded to the widest and gathered in one call.
    """
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    if world == 1:
        return local
    if sizes is None:
        n = torch.tensor([local.shape[-1]], device=local.device)
        got = [torch.zeros_like(n) for _ in range(world)]
        dist.all_gather(got, n, group=group)
        sizes = [int(s.item()) for s in got]
    width = max(sizes)
    lead = local.shape[:-1]
    buf = local
    if local.shape[-1] != width:
        buf = torch.zeros(*lead, width, dtype=local.dtype, device=local.device)
        buf[..., :local.shape[-1]] = local
    flat = buf.reshape(-1, width).contiguous()
    out = torch.empty(world, *flat.shape, dtype=flat.dtype, device=flat.device)
    if hasattr(dist, "all_gather_into_tensor") and dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, flat, group=group)
    else:
        dist.all_gather(list(out.unbind(0)), flat, group=group)
    parts = [out[r][:, :sizes[r]] for r in range(world)]
    return torch.cat(parts, dim=1).reshape(*lead, sum(sizes))


def gather_heads(local, group=None):
    """All-gather [batch, H_r, D] head blocks into [batch, sum H_r, D] in rank order."""
    b, h, d = local.shape
    full = gather_last_dim(local.permute(0, 2, 1).contiguous(), group)   # [b, d, H]
    return full.permute(0, 2, 1).contiguous()


class ShardedMLP:
    """Decode MLP over `world` ranks: rmsnorm -> gate/up (rows sharded) -> SwiGLU ->
    all-gather h -> down (rows sharded) -> all-gather y.

    ``gateup`` and ``down`` are the per-rank compute functions (the sm_100a ops on
    GPUs; any torch function with the same contract in CPU tests).
    """

    def __init__(self, Wg, Wu, Wd, gamma, rank: int, world: int, eps: float = 1e-5,
                 gateup: Callable | None = None, down: Callable | None = None, group=None):
        self.Wg, self.Wu = shard_rows(Wg, rank, world), shard_rows(Wu, rank, world)
        self.Wd = shard_rows(Wd, rank, world)
        self.gamma, self.eps, self.group = gamma, eps, group
        self._gateup = gateup
        self._down = down

    def __call__(self, x):
        h = self._gateup(x, self.Wg, self.Wu, self.gamma, self.eps)
        h = gather_last_dim(h, self.group)
        y = self._down(h, self.Wd)
        return gather_last_dim(y, self.group)
