"""GPU parity of the sm_100a kernels (through the C ABI via decodebench_b200.ops)
against the CPU oracle, the reference's golden stage outputs, and
size-independent properties at the benchmark sizes."""

from __future__ import annotations

import math
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O
from tests.helpers import assert_close, bits, from_torch, reference_gate, to_torch

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"
F16, BF16 = O.F16, O.BF16


@pytest.fixture(scope="module")
def ops():
    from decodebench_b200 import ops as _ops

    yield _ops
    assert _ops.take_device_error() == 0, "a kernel recorded a bounded-wait timeout"


# ---------------------------------------------------------------- F1
F1_CASES = [
    (1, 4096, 4096, F16),     # C1
    (1, 4096, 4096, BF16),
    (1, 256, 384, F16),
    (2, 256, 384, F16),
    (3, 72, 37, F16),         # ragged: d_in not a multiple of 256, d_out < SMs
    (1, 8, 1, BF16),          # smallest legal shape
    (8, 512, 300, BF16),
    (5, 1040, 777, F16),
    (1, 28672, 64, BF16),     # long rows
]


@pytest.mark.parametrize("batch,d_in,d_out,dt", F1_CASES)
def test_rmsnorm_gemv_parity(ops, batch, d_in, d_out, dt):
    rng = np.random.default_rng(1000 + d_in + d_out + batch)
    x, g = bits(rng, (batch, d_in), dt), bits(rng, (d_in,), dt)
    W = bits(rng, (d_out, d_in), dt, 1 / math.sqrt(d_in))
    y = ops.rmsnorm_gemv(to_torch(x, dt), to_torch(g, dt), to_torch(W, dt), eps=1e-6)
    ref = O.rmsnorm_gemv(x, g, W, 1e-6, dt, O.ROUND_FUSED)
    assert_close(from_torch(y), ref, dt, f"F1 {batch}x{d_in}->{d_out}")


# ---------------------------------------------------------------- F2
F2_CASES = [
    (1, 4096, 11008, F16, False),   # C2
    (1, 4096, 11008, BF16, True),
    (2, 256, 192, F16, False),
    (3, 72, 37, BF16, True),
    (4, 1024, 513, F16, True),
    (8, 2048, 160, BF16, False),
]


@pytest.mark.parametrize("batch,d_in,d_ff,dt,norm", F2_CASES)
def test_gateup_swiglu_parity(ops, batch, d_in, d_ff, dt, norm):
    rng = np.random.default_rng(2000 + d_in + d_ff + batch)
    x = bits(rng, (batch, d_in), dt)
    g = bits(rng, (d_in,), dt) if norm else None
    Wg = bits(rng, (d_ff, d_in), dt, 1 / math.sqrt(d_in))
    Wu = bits(rng, (d_ff, d_in), dt, 1 / math.sqrt(d_in))
    h = ops.gateup_swiglu(to_torch(x, dt), to_torch(Wg, dt), to_torch(Wu, dt),
                          gamma=None if g is None else to_torch(g, dt), eps=1e-5)
    ref = O.gateup_swiglu(x, Wg, Wu, dt, gamma=g, eps=1e-5)
    assert_close(from_torch(h), ref, dt, f"F2 {batch}x{d_in}->{d_ff}")


# ---------------------------------------------------------------- plain GEMV
@pytest.mark.parametrize("batch,d_in,d_out,dt,res", [
    (1, 11008, 4096, F16, False), (2, 4096, 1000, BF16, True), (7, 264, 99, F16, True)])
def test_gemv_parity(ops, batch, d_in, d_out, dt, res):
    rng = np.random.default_rng(3000 + d_in)
    x = bits(rng, (batch, d_in), dt)
    W = bits(rng, (d_out, d_in), dt, 1 / math.sqrt(d_in))
    r = bits(rng, (batch, d_out), dt) if res else None
    y = ops.gemv(to_torch(x, dt), to_torch(W, dt),
                 residual=None if r is None else to_torch(r, dt))
    assert_close(from_torch(y), O.gemv(x, W, dt, residual=r), dt, "gemv")


# ---------------------------------------------------------------- F4 / GQA
def _paged(rng, K, V, page_size):
    """Scatter contiguous [batch, hkv, max_len, D] caches into randomly permuted pages."""
    b, hkv, L, d = K.shape
    per = L // page_size
    npages = b * per
    perm = rng.permutation(npages).astype(np.int32)
    table = perm.reshape(b, per)
    Kp = np.zeros((npages, hkv, page_size, d), np.uint16)
    Vp = np.zeros_like(Kp)
    for s in range(b):
        for p in range(per):
            Kp[table[s, p]] = K[s, :, p * page_size:(p + 1) * page_size]
            Vp[table[s, p]] = V[s, :, p * page_size:(p + 1) * page_size]
    return Kp, Vp, table


FD_CASES = [
    # batch, hq, hkv, max_len, lens, page, split, dt
    (1, 32, 32, 4096, None, 0, 0, F16),                    # C3
    (1, 32, 32, 4096, None, 0, 0, BF16),
    (2, 2, 2, 200, None, 0, 0, F16),
    (3, 16, 2, 768, [1, 100, 700], 64, 0, BF16),           # GQA G=8, paged, ragged
    (3, 16, 2, 768, [768, 65, 64], 16, 128, F16),          # small pages
    (2, 8, 4, 512, [300, 0], 0, 64, BF16),                 # empty sequence
    (4, 8, 2, 1024, [1024, 1, 513, 777], 128, 0, F16),     # G=4
    (2, 64, 8, 4096, [4096, 2500], 64, 0, BF16),           # C5 head layout
    (2, 4, 2, 300, [300, 77], 20, 0, F16),                 # page size not a multiple of 16:
    (2, 2, 2, 300, [1, 299], 12, 0, BF16),                 #   CUDA-core path
]


@pytest.mark.parametrize("batch,hq,hkv,max_len,lens,page,split,dt", FD_CASES)
def test_flashdecode_parity(ops, batch, hq, hkv, max_len, lens, page, split, dt):
    rng = np.random.default_rng(4000 + max_len + hq + batch)
    d = 128
    q = bits(rng, (batch, hq, d), dt)
    K = bits(rng, (batch, hkv, max_len, d), dt)
    V = bits(rng, (batch, hkv, max_len, d), dt)
    scale = 1 / math.sqrt(d)
    sl = None if lens is None else np.array(lens, np.int32)
    ref = O.attention(q, K, V, dt, scale, seq_lens=sl)
    tl = None if sl is None else torch.from_numpy(sl).cuda()
    if page:
        Kp, Vp, table = _paged(rng, K, V, page)
        out = ops.flashdecode(to_torch(q, dt), to_torch(Kp, dt), to_torch(Vp, dt), seq_lens=tl,
                              page_table=torch.from_numpy(table).cuda(), scale=scale,
                              split_tokens=split)
        ref_p = O.attention(q, Kp, Vp, dt, scale, seq_lens=sl, page_table=table)
        assert np.array_equal(ref_p, ref), "oracle paged/contiguous mismatch"
    else:
        out = ops.flashdecode(to_torch(q, dt), to_torch(K, dt), to_torch(V, dt), seq_lens=tl,
                              scale=scale, split_tokens=split)
    assert_close(from_torch(out), ref, dt, f"F4 b{batch} {hq}/{hkv} L{max_len} page{page}")


def test_flashdecode_c5_full(ops):
    """C5 at full size: batch 8, 64/8 heads, paged (64), lengths ~U[1024, 32768]."""
    dt, d, ps = BF16, 128, 64
    rng = np.random.default_rng(55)
    lens = rng.integers(1024, 32769, size=8).astype(np.int32)
    maxp = (int(lens.max()) + ps - 1) // ps
    pages_per = [(int(n) + ps - 1) // ps for n in lens]
    npages = sum(pages_per)
    perm = rng.permutation(npages).astype(np.int32)
    table = np.zeros((8, maxp), np.int32)
    o = 0
    for b, n in enumerate(pages_per):
        table[b, :n] = perm[o:o + n]
        o += n
    q = bits(rng, (8, 64, d), dt)
    Kp = bits(rng, (npages, 8, ps, d), dt)
    Vp = bits(rng, (npages, 8, ps, d), dt)
    out = ops.flashdecode(to_torch(q, dt), to_torch(Kp, dt), to_torch(Vp, dt),
                          seq_lens=torch.from_numpy(lens).cuda(),
                          page_table=torch.from_numpy(table).cuda(), scale=1 / math.sqrt(d))
    ref = O.attention(q, Kp, Vp, dt, 1 / math.sqrt(d), seq_lens=lens, page_table=table)
    assert_close(from_torch(out), ref, dt, "C5")


# ---------------------------------------------------------------- golden fixtures
def _g(name):
    return np.load(GOLDEN / f"golden_{name}.npz")


@pytest.mark.parametrize("name", ["f1", "f1_ragged"])
def test_golden_f1(ops, name):
    z = _g(name)
    y = from_torch(ops.rmsnorm_gemv(to_torch(z["x"], F16), to_torch(z["g"], F16),
                                    to_torch(z["W"], F16), eps=1e-6))
    assert reference_gate(y, z["y"], F16)
    assert_close(y, z["y"], F16, name)   # the stage chain's extra roundings stay in budget


def test_golden_f2(ops):
    z = _g("f2")
    y = from_torch(ops.gateup_swiglu(to_torch(z["xh"], F16), to_torch(z["Wg"], F16),
                                     to_torch(z["Wu"], F16)))
    assert reference_gate(y, z["y"], F16)
    assert_close(y, O.gateup_swiglu(z["xh"], z["Wg"], z["Wu"], F16), F16, "f2 oracle")


def test_golden_f4(ops):
    z = _g("f4")
    y = from_torch(ops.flashdecode(to_torch(z["q"], F16), to_torch(z["K"], F16),
                                   to_torch(z["V"], F16), scale=1.0))
    assert reference_gate(y, z["y"], F16)
    assert_close(y, O.attention(z["q"], z["K"], z["V"], F16, 1.0), F16, "f4 oracle")


# ---------------------------------------------------------------- properties
def test_determinism_and_split_invariance(ops):
    dt, d = BF16, 128
    rng = np.random.default_rng(7)
    q = to_torch(bits(rng, (2, 16, d), dt), dt)
    K = to_torch(bits(rng, (2, 2, 4096, d), dt), dt)
    V = to_torch(bits(rng, (2, 2, 4096, d), dt), dt)
    a = from_torch(ops.flashdecode(q, K, V))
    b = from_torch(ops.flashdecode(q, K, V))
    assert np.array_equal(a, b), "same inputs must give bit-identical outputs"
    for split in (64, 256, 4096):
        assert_close(from_torch(ops.flashdecode(q, K, V, split_tokens=split)), a, dt,
                     f"split {split}")
    x = to_torch(bits(rng, (1, 4096), dt), dt)
    g = to_torch(bits(rng, (4096,), dt), dt)
    W = to_torch(bits(rng, (4096, 4096), dt, 1 / 64), dt)
    y1 = from_torch(ops.rmsnorm_gemv(x, g, W))
    assert np.array_equal(y1, from_torch(ops.rmsnorm_gemv(x, g, W)))


def test_gemv_linearity(ops):
    """W(x1) + W(x2) == W(x1 + x2) within tolerance at the C2 size (fp32 path)."""
    dt = F16
    rng = np.random.default_rng(8)
    W = to_torch(bits(rng, (11008, 4096), dt, 1 / 64), dt)
    x1 = to_torch(bits(rng, (1, 4096), dt, 0.5), dt)
    x2 = to_torch(bits(rng, (1, 4096), dt, 0.5), dt)
    y = ops.gemv(x1, W).float() + ops.gemv(x2, W).float()
    y12 = ops.gemv((x1.float() + x2.float()).half(), W).float()
    rel = (y - y12).norm() / y12.norm()
    assert rel.item() < 2e-3


def test_cuda_graph_capture_of_ops(ops):
    dt = F16
    rng = np.random.default_rng(9)
    x = to_torch(bits(rng, (1, 1024), dt), dt)
    g = to_torch(bits(rng, (1024,), dt), dt)
    W = to_torch(bits(rng, (2048, 1024), dt, 1 / 32), dt)
    K = to_torch(bits(rng, (1, 4, 512, 128), dt), dt)
    q = to_torch(bits(rng, (1, 4, 128), dt), dt)
    eager_y = ops.rmsnorm_gemv(x, g, W)
    eager_o = ops.flashdecode(q, K, K)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        gy = ops.rmsnorm_gemv(x, g, W)
        go = ops.flashdecode(q, K, K)
    graph.replay()
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(gy, eager_y) and torch.equal(go, eager_o)


def test_argument_errors(ops):
    from decodebench_b200._native import DbkError

    x = torch.zeros(1, 12, dtype=torch.float16, device="cuda")   # d_in % 8 != 0
    W = torch.zeros(4, 12, dtype=torch.float16, device="cuda")
    with pytest.raises(DbkError, match="supported range"):
        ops.gemv(x, W)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        ops.gemv(torch.zeros(1, 16, dtype=torch.float16), torch.zeros(4, 16, dtype=torch.float16))
    q = torch.zeros(1, 3, 128, dtype=torch.float16, device="cuda")
    K = torch.zeros(1, 2, 64, 128, dtype=torch.float16, device="cuda")
    with pytest.raises(DbkError):
        ops.flashdecode(q, K, K)   # 3 q heads over 2 kv heads


@pytest.mark.gpu
def test_stage_copies_between_pinned_host_and_device():
    """ops.stage (dbk_copy): pinned host -> device and back, bit-exact, including
    sizes that are not a multiple of 16 bytes; pageable memory is refused."""
    import torch

    from decodebench_b200 import ops
    from decodebench_b200._native import DbkError

    for n in (8, 4096, 11008, 1000003):
        src = torch.randint(-30000, 30000, (n,), dtype=torch.int16).pin_memory()
        dev = torch.empty(n, dtype=torch.int16, device="cuda")
        back = torch.empty(n, dtype=torch.int16).pin_memory()
        ops.stage(dev, src)
        ops.stage(back, dev)
        torch.cuda.synchronize()
        assert torch.equal(back, src), f"round trip differs at {n} elements"
        assert torch.equal(dev.cpu(), src)
    with pytest.raises(ValueError):
        ops.stage(torch.empty(16, dtype=torch.int16, device="cuda"), torch.zeros(16, dtype=torch.int16))
    with pytest.raises(DbkError):
        big = torch.empty(17, dtype=torch.int8, device="cuda")
        ops.stage(big[1:], torch.zeros(16, dtype=torch.int8).pin_memory())   # misaligned


@pytest.mark.gpu
def test_output_straight_into_pinned_host_memory():
    """out= a pinned CPU tensor: the kernels write the result into host memory
    directly; equal to the device-output result; pageable CPU out is refused."""
    import torch

    from decodebench_b200 import ops

    g = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn(2, 1024, generator=g, device="cuda").half()
    gam = torch.randn(1024, generator=g, device="cuda").half()
    Wg = (torch.randn(700, 1024, generator=g, device="cuda") / 32).half()
    Wu = (torch.randn(700, 1024, generator=g, device="cuda") / 32).half()
    ref = ops.gateup_swiglu(x, Wg, Wu, gamma=gam)
    host = torch.empty(2, 700, dtype=torch.float16).pin_memory()
    ops.gateup_swiglu(x, Wg, Wu, gamma=gam, out=host)
    torch.cuda.synchronize()
    assert torch.equal(host, ref.cpu())
    ref = ops.rmsnorm_gemv(x, gam, Wg)
    ops.rmsnorm_gemv(x, gam, Wg, out=host)
    torch.cuda.synchronize()
    assert torch.equal(host, ref.cpu())
    q = torch.randn(1, 8, 128, generator=g, device="cuda").half()
    K = torch.randn(1, 8, 1000, 128, generator=g, device="cuda").half()
    V = torch.randn(1, 8, 1000, 128, generator=g, device="cuda").half()
    ref = ops.flashdecode(q, K, V)
    hq = torch.empty(1, 8, 128, dtype=torch.float16).pin_memory()
    ops.flashdecode(q, K, V, out=hq)
    torch.cuda.synchronize()
    assert torch.equal(hq, ref.cpu())
    with pytest.raises(RuntimeError, match="pinned"):
        ops.gemv(x, Wg, out=torch.empty(2, 700, dtype=torch.float16))
