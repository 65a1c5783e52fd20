"""dbk_allgather (NVLink peer-store all-gather) against NCCL's all-gather on 2 GPUs.

Two processes, one per GPU (the exchange waits on the other rank, so both ranks
must own a GPU each; the test is skipped with fewer than 2 GPUs). Checked:
the [world, block] and the column-block [rows, world * n] layouts, a strided
source, repeated exchanges with new data (staging parity), alternating shapes
(cumulative counters), replay inside a CUDA graph, and no device error recorded.
"""

import os
import socket

import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, errq):
    try:
        import torch.distributed as dist

        from decodebench_b200 import ops
        from decodebench_b200.comm import PeerComm

        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world, device_id=torch.device("cuda", rank))
        dev = torch.device("cuda", rank)
        comm = PeerComm(4 << 20)
        g = torch.Generator(device=dev).manual_seed(rank)
        for it in range(6):
            # block layout (F2 at batch 1: h [1, d_ff / world])
            a = torch.randn(1, 5504, generator=g, device=dev).half()
            got = comm.all_gather_blocks(a)
            ref = torch.empty(world, 1, 5504, dtype=a.dtype, device=dev)
            dist.all_gather_into_tensor(ref, a)
            assert torch.equal(got, ref), f"blocks differ at iteration {it}"
            # column-block layout (MLP h: [16, d_ff / world] -> [16, d_ff])
            b = torch.randn(16, 7168, generator=g, device=dev).bfloat16()
            got = comm.all_gather_rows(b)
            full = torch.empty(world, 16, 7168, dtype=b.dtype, device=dev)
            dist.all_gather_into_tensor(full, b)
            assert torch.equal(got, full.permute(1, 0, 2).reshape(16, world * 7168)), \
                f"rows differ at iteration {it}"
            # strided source rows (a slice of a wider tensor)
            w = torch.randn(8, 512, generator=g, device=dev).bfloat16()
            got = comm.all_gather_rows(w[:, :256])
            full = torch.empty(world, 8, 256, dtype=w.dtype, device=dev)
            dist.all_gather_into_tensor(full, w[:, :256].contiguous())
            assert torch.equal(got, full.permute(1, 0, 2).reshape(8, world * 256))
        # inside a CUDA graph, replayed with new inputs
        src = torch.zeros(4, 1024, dtype=torch.float16, device=dev)
        out = torch.empty(4, world * 1024, dtype=torch.float16, device=dev)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            comm.all_gather_rows(src, out)
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            comm.all_gather_rows(src, out)
        for it in range(4):
            src.copy_(torch.randn(4, 1024, generator=g, device=dev).half())
            graph.replay()
            full = torch.empty(world, 4, 1024, dtype=src.dtype, device=dev)
            dist.all_gather_into_tensor(full, src)
            assert torch.equal(out, full.permute(1, 0, 2).reshape(4, world * 1024)), \
                f"graph replay {it} differs"
        torch.cuda.synchronize()
        assert ops.take_device_error() == 0, "a bounded wait gave up"
        dist.barrier()
        comm.close()
        dist.destroy_process_group()
    except BaseException as e:          # report to the parent, never hang it
        import traceback

        errq.put(f"rank {rank}: {e!r}\n{traceback.format_exc()}")
        os._exit(1)
    os._exit(0)


def test_peer_allgather_matches_nccl():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    errq = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, errq)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    errors = []
    while not errq.empty():
        errors.append(errq.get())
    assert not alive, "a rank did not finish within 240 s"
    assert not errors, "\n".join(errors)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
