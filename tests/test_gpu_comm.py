"""dbk_allgather (NVLink peer-store all-gather) and the GEMVs with the all-gather
fused in (dbk_*_allgather) against NCCL's all-gather on 2 GPUs.

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
        # GEMVs with the all-gather fused into the kernel, against the same op
        # unfused + NCCL (bit-identical: same kernel arithmetic per CTA)
        def nccl_rows(t):
            full = torch.empty(world, *t.shape, dtype=t.dtype, device=dev)
            dist.all_gather_into_tensor(full, t.contiguous())
            return full.permute(1, 0, 2).reshape(t.shape[0], world * t.shape[1])

        for it in range(3):
            for dt, batch, d_in, d_loc in ((torch.float16, 1, 1024, 688),
                                           (torch.bfloat16, 3, 2048, 512),
                                           (torch.float16, 8, 512, 200)):
                x = torch.randn(batch, d_in, generator=g, device=dev).to(dt)
                gam = torch.randn(d_in, generator=g, device=dev).to(dt)
                Wg = (torch.randn(d_loc, d_in, generator=g, device=dev) / 32).to(dt)
                Wu = (torch.randn(d_loc, d_in, generator=g, device=dev) / 32).to(dt)
                got = ops.gateup_swiglu(x, Wg, Wu, gamma=gam, eps=1e-5, comm=comm)
                ref = nccl_rows(ops.gateup_swiglu(x, Wg, Wu, gamma=gam, eps=1e-5))
                assert torch.equal(got, ref), f"fused F2 differs ({dt}, batch {batch}, it {it})"
                got = ops.rmsnorm_gemv(x, gam, Wg, eps=1e-6, comm=comm)
                ref = nccl_rows(ops.rmsnorm_gemv(x, gam, Wg, eps=1e-6))
                assert torch.equal(got, ref), f"fused F1 differs ({dt}, batch {batch}, it {it})"
                res = torch.randn(batch, world * d_loc, generator=g, device=dev).to(dt)
                dist.broadcast(res, 0)
                got = ops.gemv(x, Wu, residual=res, comm=comm)
                loc = res[:, rank * d_loc:(rank + 1) * d_loc].contiguous()
                ref = nccl_rows(ops.gemv(x, Wu, residual=loc))
                assert torch.equal(got, ref), f"fused GEMV differs ({dt}, batch {batch}, it {it})"
                # the standalone exchange interleaved with the fused ones
                got = comm.all_gather_rows(x)
                assert torch.equal(got, nccl_rows(x))
        # fused op inside a CUDA graph
        x = torch.zeros(1, 1024, dtype=torch.float16, device=dev)
        Wg = (torch.randn(344, 1024, generator=g, device=dev) / 32).half()
        Wu = (torch.randn(344, 1024, generator=g, device=dev) / 32).half()
        h = torch.empty(1, world * 344, dtype=torch.float16, device=dev)
        with torch.cuda.stream(s):
            ops.gateup_swiglu(x, Wg, Wu, out=h, comm=comm)
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            ops.gateup_swiglu(x, Wg, Wu, out=h, comm=comm)
        for it in range(3):
            x.copy_(torch.randn(1, 1024, generator=g, device=dev).half())
            dist.broadcast(x, 0)
            graph.replay()
            ref = nccl_rows(ops.gateup_swiglu(x, Wg, Wu))
            assert torch.equal(h, ref), f"fused graph replay {it} differs"
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
