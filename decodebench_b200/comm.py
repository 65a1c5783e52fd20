"""Shard-boundary all-gather over NVLink peer memory (``dbk_allgather``).

One process per GPU. :class:`PeerComm` sets up, once per process group, a comm
buffer on every GPU and maps the peers' buffers (CUDA IPC; the records are
exchanged with ``torch.distributed.all_gather_object``). After that,
:meth:`PeerComm.all_gather_rows` / :meth:`PeerComm.all_gather_blocks` replace
``all_gather_into_tensor`` at the end of a sharded op: a single kernel stores
this rank's block into every peer and waits (bounded) for theirs,
stream-ordered and without host synchronisation.

The reference (animeshsri14/Decodebench) is single-GPU; this module has no
counterpart there. Every rank must issue the same exchanges in the same order.
"""

from __future__ import annotations

import ctypes

import torch

from . import _native as N


class PeerComm:
    def __init__(self, capacity_bytes: int, group=None):
        import torch.distributed as dist

        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.device = torch.device("cuda", torch.cuda.current_device())
        lib = N.load()
        self._lib = lib
        buf = ctypes.c_void_p()
        rec = (ctypes.c_ubyte * N.DBK_COMM_RECORD_BYTES)()
        N.check("dbk_comm_alloc", lib.dbk_comm_alloc(int(capacity_bytes), self.world,
                                                     ctypes.byref(buf), ctypes.addressof(rec)))
        self._buf = buf
        records = [None] * self.world
        dist.all_gather_object(records, bytes(rec), group=group)
        blob = b"".join(records)
        if len(blob) != self.world * N.DBK_COMM_RECORD_BYTES:
            raise RuntimeError("peer records of unexpected size")
        arr = (ctypes.c_ubyte * len(blob)).from_buffer_copy(blob)
        comm = ctypes.c_void_p()
        st = lib.dbk_comm_open(self.rank, self.world, buf, ctypes.addressof(arr),
                               ctypes.byref(comm))
        if st != 0:
            lib.dbk_comm_free(buf)
            self._buf = None
            N.check("dbk_comm_open", st)
        self._comm = comm
        self.capacity = int(capacity_bytes)
        dist.barrier(group=group)

    @property
    def handle(self):
        """The ``dbk_comm*`` for the C-ABI entry points that take one."""
        if not getattr(self, "_comm", None):
            raise RuntimeError("PeerComm is closed")
        return self._comm

    def _stream(self) -> int:
        return torch.cuda.current_stream(self.device).cuda_stream

    def _check(self, *ts):
        for t in ts:
            if not t.is_cuda or t.device != self.device:
                raise ValueError("PeerComm tensors must be on this rank's CUDA device")

    def all_gather_blocks(self, local: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """[*shape] on every rank -> [world, *shape] in rank order."""
        self._check(local)
        if not local.is_contiguous():
            raise ValueError("local block must be contiguous")
        if out is None:
            out = torch.empty(self.world, *local.shape, dtype=local.dtype, device=local.device)
        self._check(out)
        if out.numel() != self.world * local.numel() or not out.is_contiguous():
            raise ValueError("out must be contiguous with world * local.numel() elements")
        nb = local.numel() * local.element_size()
        N.check("dbk_allgather", self._lib.dbk_allgather(
            self._comm, local.data_ptr(), out.data_ptr(), 1, nb, nb, nb, nb, self._stream()))
        return out

    def all_gather_rows(self, local: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """[rows, n] on every rank -> [rows, world * n], rank p's block in columns
        [p * n, (p + 1) * n) (the layout of a column-sharded GEMV output)."""
        self._check(local)
        if local.dim() != 2 or local.stride(1) != 1:
            raise ValueError("local must be [rows, n] with unit column stride")
        rows, n = local.shape
        es = local.element_size()
        if out is None:
            out = torch.empty(rows, self.world * n, dtype=local.dtype, device=local.device)
        self._check(out)
        if out.shape != (rows, self.world * n) or not out.is_contiguous():
            raise ValueError("out must be contiguous [rows, world * n]")
        N.check("dbk_allgather", self._lib.dbk_allgather(
            self._comm, local.data_ptr(), out.data_ptr(), rows, n * es, local.stride(0) * es,
            self.world * n * es, n * es, self._stream()))
        return out

    def close(self) -> None:
        """Unmap the peers, wait until every rank has done so, then free (collective)."""
        import torch.distributed as dist

        if getattr(self, "_comm", None):
            torch.cuda.synchronize(self.device)
            self._lib.dbk_comm_close(self._comm)
            self._comm = None
            dist.barrier(group=self.group)
        if getattr(self, "_buf", None):
            self._lib.dbk_comm_free(self._buf)
            self._buf = None
