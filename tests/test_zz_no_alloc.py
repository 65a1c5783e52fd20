"""GPU test of dbk_flashdecode_noalloc, the entry point for callers that cannot
allocate device memory (for example a plugin whose host process owns the GPU's
allocator). It must give the same results as dbk_flashdecode, which takes a
caller workspace, on two calls in a row (the shared scratch array keeps the
previous call's contents). Collected last on purpose."""

import math

import numpy as np
import pytest

from oracle import oracle as O
from tests.helpers import assert_close, bits, from_torch, to_torch

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _noalloc(lib, q, K, V, out, lens=None, table=None, page_size=0, scale=1.0):
    batch, hq, d = q.shape
    if table is None:
        _, hkv, max_len, _ = K.shape
        mp = 0
    else:
        _, hkv, page_size, _ = K.shape
        mp = table.shape[1]
        max_len = page_size * mp
    dt = 0 if q.dtype == torch.float16 else 1
    return lib.dbk_flashdecode_noalloc(
        q.data_ptr(), K.data_ptr(), V.data_ptr(), None if table is None else table.data_ptr(),
        None if lens is None else lens.data_ptr(), out.data_ptr(), batch, hq, hkv, d, max_len,
        page_size, mp, scale, dt, torch.cuda.current_stream().cuda_stream)


def test_noalloc_matches_workspace_entry_point():
    from decodebench_b200 import _native, ops

    lib = _native.load()
    rng = np.random.default_rng(77)
    scale = 1 / math.sqrt(128)
    cases = []
    # GQA, paged, ragged lengths (bf16)
    dt = O.BF16
    lens = np.array([700, 1, 333], np.int32)
    ps, maxp = 64, 11
    table = rng.permutation(3 * maxp).astype(np.int32).reshape(3, maxp)
    cases.append(dict(q=to_torch(bits(rng, (3, 16, 128), dt), dt),
                      K=to_torch(bits(rng, (3 * maxp, 2, ps, 128), dt), dt),
                      V=to_torch(bits(rng, (3 * maxp, 2, ps, 128), dt), dt),
                      lens=torch.from_numpy(lens).cuda(), table=torch.from_numpy(table).cuda(), dt=dt))
    # MHA, contiguous (fp16)
    dt = O.F16
    cases.append(dict(q=to_torch(bits(rng, (1, 32, 128), dt), dt),
                      K=to_torch(bits(rng, (1, 32, 1024, 128), dt), dt),
                      V=to_torch(bits(rng, (1, 32, 1024, 128), dt), dt), lens=None, table=None, dt=dt))
    for c in cases:
        ref = from_torch(ops.flashdecode(c["q"], c["K"], c["V"], seq_lens=c["lens"],
                                         page_table=c["table"], scale=scale))
        for _ in range(2):
            out = torch.full_like(c["q"], float("nan"))
            assert _noalloc(lib, c["q"], c["K"], c["V"], out, c["lens"], c["table"],
                            scale=scale) == 0
            torch.cuda.synchronize()
            assert_close(from_torch(out), ref, c["dt"], "noalloc vs workspace entry point")


def test_noalloc_rejects_oversized_problem():
    from decodebench_b200 import _native

    lib = _native.load()
    q = torch.zeros(1, 8, 128, dtype=torch.bfloat16, device="cuda")
    # 200k sequences x 8 kv heads of arrival counters do not fit in the 2 MiB array
    rc = lib.dbk_flashdecode_noalloc(q.data_ptr(), q.data_ptr(), q.data_ptr(), None, None,
                                     q.data_ptr(), 200000, 8, 8, 128, 64, 0, 0, 1.0, 1,
                                     torch.cuda.current_stream().cuda_stream)
    assert rc == -4
