"""A bounded device wait that runs out, on one GPU, without faulting anything.

Every spin-wait in the library's kernels (mbarrier waits on the copy ring, the
peer-flag waits of the fused all-gather, the stream-K merge waits) gives up
after a poll budget, records an error code and returns. Here the budget is
lowered (dbk_set_spin_limit) and a one-CTA probe kernel waits on events that
never happen, using the library's own mbar_wait / wait_flag helpers. The test
checks that the kernel returns, that dbk_take_device_error reports the code,
and that the context stays usable: a normal FlashDecode call afterwards still
matches the oracle."""

from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle as O
from tests.helpers import assert_close, bits, from_torch, to_torch

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

K_TIMEOUT_FULL, K_TIMEOUT_PEER = 1, 5


@pytest.fixture()
def lib():
    from decodebench_b200 import _native as N
    from decodebench_b200 import ops

    L = N.load()
    assert ops.take_device_error() == 0
    yield L
    N.check("set_spin_limit", L.dbk_set_spin_limit(0))     # restore the default budget
    assert ops.take_device_error() == 0


@pytest.mark.parametrize("which,code", [(0, K_TIMEOUT_FULL), (1, K_TIMEOUT_PEER)])
def test_wait_runs_out_and_reports(lib, which, code):
    from decodebench_b200 import _native as N
    from decodebench_b200 import ops

    N.check("set_spin_limit", lib.dbk_set_spin_limit(2000))
    s = torch.cuda.current_stream().cuda_stream
    N.check("test_bounded_wait", lib.dbk_test_bounded_wait(which, s))
    assert lib.dbk_take_device_error() == code
    assert lib.dbk_take_device_error() == 0            # taking it cleared it
    # ops.check_device_error raises on a recorded failure
    N.check("test_bounded_wait", lib.dbk_test_bounded_wait(which, s))
    with pytest.raises(RuntimeError, match="bounded wait"):
        ops.check_device_error()
    N.check("set_spin_limit", lib.dbk_set_spin_limit(0))

    # the context is intact: a real kernel with the default budget matches the oracle
    rng = np.random.default_rng(77)
    H, L, D = 4, 700, 128
    q = bits(rng, (1, H, D), O.F16)
    K = bits(rng, (1, H, L, D), O.F16)
    V = bits(rng, (1, H, L, D), O.F16)
    out = ops.flashdecode(to_torch(q, O.F16), to_torch(K, O.F16), to_torch(V, O.F16))
    ref = O.attention(q, K, V, O.F16, 1.0 / np.sqrt(D))
    assert_close(from_torch(out), ref, O.F16, "flashdecode after a timed-out wait")
    ops.check_device_error()


def test_spin_limit_rejects_nothing_and_restores(lib):
    from decodebench_b200 import _native as N

    for v in (1, 5000, 0):
        N.check("set_spin_limit", lib.dbk_set_spin_limit(v))
