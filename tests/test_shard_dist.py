"""Multi-rank logic of the sharded decode path, on CPU with the gloo backend
(world size 2): partitioning, all-gather reassembly in rank order, the sharded
MLP pipeline, head sharding, and failure of a rank surfacing as an error on the
others instead of a hang."""

import math
import os
import socket
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from decodebench_b200 import shard


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(fn, world=2, timeout_s=30):
    port = _port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_entry, args=(fn, r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout_s)
    results = {}
    while not q.empty():
        r, v = q.get()
        results[r] = v
    for p in procs:
        if p.is_alive():
            p.kill()
    return results


def _entry(fn, rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=timedelta(seconds=5))
        q.put((rank, fn(rank, world)))
    except Exception as e:  # reported to the test, never swallowed
        q.put((rank, f"ERROR {type(e).__name__}: {e}"))
    finally:
        if dist.is_initialized():
            try:
                dist.destroy_process_group()
            except Exception:
                pass


def test_row_range_partitions():
    for n in (1, 7, 11008, 28672):
        for world in (1, 2, 3, 4, 8):
            spans = [shard.row_range(n, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard.row_range(8, 2, 2)


# ---- world-2 workers (module-level so spawn can pickle them)
def _w_gather(rank, world):
    width = 3 + rank                         # unequal blocks: 3 and 4 columns
    local = torch.full((2, width), float(rank))
    out = shard.gather_last_dim(local)
    return out.tolist()


def _w_f2(rank, world):
    g = torch.Generator().manual_seed(0)
    x = torch.randn(3, 64, generator=g)
    Wg, Wu = torch.randn(48, 64, generator=g), torch.randn(48, 64, generator=g)
    h_local = torch.nn.functional.silu(x @ shard.shard_rows(Wg, rank, world).T) * \
        (x @ shard.shard_rows(Wu, rank, world).T)
    h = shard.gather_last_dim(h_local)
    ref = torch.nn.functional.silu(x @ Wg.T) * (x @ Wu.T)
    return float((h - ref).abs().max())


def _w_mlp(rank, world):
    g = torch.Generator().manual_seed(1)
    x = torch.randn(4, 32, generator=g)
    gamma = torch.randn(32, generator=g)
    Wg, Wu, Wd = (torch.randn(40, 32, generator=g), torch.randn(40, 32, generator=g),
                  torch.randn(32, 40, generator=g))

    def gateup(x, Wg, Wu, gamma, eps):
        xn = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * gamma
        return torch.nn.functional.silu(xn @ Wg.T) * (xn @ Wu.T)

    def down(h, Wd):
        return h @ Wd.T

    y = shard.ShardedMLP(Wg, Wu, Wd, gamma, rank, world, gateup=gateup, down=down)(x)
    ref = down(gateup(x, Wg, Wu, gamma, 1e-5), Wd)
    return float((y - ref).abs().max())


def _w_heads(rank, world):
    g = torch.Generator().manual_seed(2)
    q = torch.randn(2, 8, 16, generator=g)          # 8 q heads over 4 kv heads
    K, V = torch.randn(2, 4, 10, 16, generator=g), torch.randn(2, 4, 10, 16, generator=g)

    def attend(q, K, V):
        gq = q.shape[1] // K.shape[1]
        Kx, Vx = K.repeat_interleave(gq, 1), V.repeat_interleave(gq, 1)
        p = torch.softmax(torch.einsum("bhd,bhld->bhl", q, Kx) / 4.0, -1)
        return torch.einsum("bhl,bhld->bhd", p, Vx)

    ql, Kl, Vl = shard.shard_heads(q, K, V, rank, world)
    out = shard.gather_heads(attend(ql, Kl, Vl))
    return float((out - attend(q, K, V)).abs().max())


def _w_rank_fails(rank, world):
    if rank == 1:
        raise RuntimeError("injected failure on rank 1 before the exchange")
    shard.gather_last_dim(torch.zeros(2, 2))        # rank 0 must error out, not hang
    return "completed"


def test_gather_unequal_blocks_in_rank_order():
    res = _run(_w_gather)
    assert res[0] == res[1] == [[0.0] * 3 + [1.0] * 4] * 2


@pytest.mark.parametrize("worker", [_w_f2, _w_mlp, _w_heads])
def test_sharded_equals_unsharded(worker):
    res = _run(worker)
    assert set(res) == {0, 1}, res
    for r, v in res.items():
        assert isinstance(v, float), v
        assert v < 1e-4, (r, v)


def test_rank_failure_surfaces_as_error():
    res = _run(_w_rank_fails, timeout_s=60)
    assert str(res.get(1, "")).startswith("ERROR RuntimeError"), res
    assert str(res.get(0, "")).startswith("ERROR"), res
