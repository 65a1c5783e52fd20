"""The C-ABI library: it loads, exports every symbol include/dbk.h declares with
the signatures the ctypes binding uses, and answers host-only queries without a GPU."""

import re
from pathlib import Path

import pytest

from decodebench_b200 import _native as N

HEADER = Path(__file__).resolve().parent.parent / "include" / "dbk.h"


def declared_functions() -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(dbk_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = N.load()
    names = declared_functions()
    assert len(names) >= 9
    for name in names:
        assert hasattr(lib, name), f"libdbk.so does not export {name}"
    assert set(names) == set(N.SIGNATURES), "ctypes signatures out of sync with include/dbk.h"


def test_host_queries():
    lib = N.load()
    assert lib.dbk_abi_version() == 1
    assert N.status_string(0) == "ok"
    assert "supported range" in N.status_string(-2)
    assert "workspace" in N.status_string(-4)
    assert lib.dbk_workspace_bytes(N.DBK_OP_RMSNORM_GEMV, 1, 4096, 4096) == 0
    assert lib.dbk_flashdecode_workspace_bytes(1, 32, 32, 4096, 0) > 0
    assert lib.dbk_flashdecode_workspace_bytes(0, 32, 32, 4096, 0) == 0


def test_null_and_shape_errors_before_any_device_work():
    lib = N.load()
    assert lib.dbk_rmsnorm_gemv(None, None, None, None, 1, 64, 64, 1e-6, 0, None, 0, None) == -1
    assert lib.dbk_gemv(8, 16, None, 32, 1, 12, 4, 0, None, 0, None) == -2     # d_in % 8
    assert lib.dbk_gemv(8, 16, None, 32, 1, 16, 4, 7, None, 0, None) == -5     # dtype
    assert lib.dbk_gemv(8, 24, None, 32, 1, 16, 4, 0, None, 0, None) == -3     # misaligned W
    assert lib.dbk_flashdecode(16, 16, 16, None, None, 16, 1, 3, 2, 128, 64, 0, 0, 1.0, 0, 0,
                               None, 0, None) == -2                              # 3 % 2
    assert lib.dbk_flashdecode(16, 16, 16, None, None, 16, 1, 2, 2, 64, 64, 0, 0, 1.0, 0, 0,
                               None, 0, None) == -2                              # head_dim
    # dbk_mlp_block: x, Wg, Wu, Wd, residual, h, y ... workspace, bytes, stream
    assert lib.dbk_mlp_block_workspace_bytes() >= 8
    assert lib.dbk_mlp_block(16, None, 16, None, 16, None, 16, 16, 1, 1024, 4352, 1e-5, 0,
                             16, 256, None) == -1                               # Wu
    assert lib.dbk_mlp_block(16, None, 16, 16, 24, None, 16, 16, 1, 1024, 4352, 1e-5, 0,
                             16, 256, None) == -3                               # misaligned Wd
    assert lib.dbk_mlp_block(16, None, 16, 16, 16, None, 16, 16, 1, 1024, 4352, 1e-5, 0,
                             None, 0, None) == -4                               # no workspace


def test_ops_refuse_cpu_tensors():
    torch = pytest.importorskip("torch")
    from decodebench_b200 import ops

    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        ops.gemv(torch.zeros(1, 16, dtype=torch.float16), torch.zeros(4, 16, dtype=torch.float16))


def test_comm_host_checks():
    lib = N.load()
    assert lib.dbk_comm_buffer_bytes(1000, 2) == 10496 + 2 * 2 * 1024
    assert lib.dbk_comm_buffer_bytes(1000, 9) == 0               # at most 8 ranks
    assert lib.dbk_allgather(None, 16, 16, 1, 16, 16, 16, 16, None) == -1
    assert lib.dbk_comm_open(0, 2, None, None, None) == -1
    assert lib.dbk_comm_close(None) == -1
