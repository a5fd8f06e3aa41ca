"""Linear layer (mlb_linear_f32) vs the reference's LinearWithBlocks / F32
Linear (quant.cc:171-226, matmul_optimized.cc:95-117) through the C ABI.

The vector path sums each block's 32 products before scaling and reduces a
row across a warp, so it is checked within |y - y_ref| <= 1e-5 * sum|w x|
(the magnitude of the dot product's terms); the scalar path (k % 32 != 0)
keeps the reference's sequential order and must match bit for bit.
"""
import numpy as np
import pytest

from conftest import assert_bitexact

import mlb
import workloads as wl

pytestmark = pytest.mark.gpu


def dev(a, device):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


def _check(got, want, wdeq, x, what):
    mag = np.abs(x.astype(np.float64)) @ np.abs(wdeq.astype(np.float64)).T
    err = np.abs(got.astype(np.float64) - want.astype(np.float64))
    bad = err > 1e-5 * mag + 1e-30
    assert not bad.any(), (f"{what}: {bad.sum()} outputs off; worst ratio "
                           f"{float((err / np.maximum(mag, 1e-30)).max()):.2e}")


@pytest.mark.parametrize("qtype", [wl.F32, wl.Q8_0, wl.Q4_0, wl.Q4_1])
@pytest.mark.parametrize("n,k,t", [(37, 96, 1), (300, 4096, 1), (64, 4096, 3),
                                   (129, 1024, 8), (40, 2048, 9), (17, 3584, 17),
                                   (2000, 896, 2)])
def test_linear_vs_oracle(cuda, oracle, qtype, n, k, t):
    import torch
    rng = np.random.default_rng(n * 7 + k + t)
    table = wl.numpy_quant_table(qtype, n, k, seed=n + k)
    x = rng.standard_normal((t, k), dtype=np.float32)
    want = oracle.linear(table, qtype, n, k, x)
    got = mlb.linear(dev(table, cuda), qtype, n, k, dev(x, cuda))
    torch.cuda.synchronize()
    wdeq, _ = oracle.embedding(table, qtype, n, k, np.arange(n, dtype=np.int32))
    _check(got.cpu().numpy(), want, wdeq, x, f"{wl.QNAME[qtype]} n={n} k={k} t={t}")


@pytest.mark.parametrize("qtype", [wl.F32, wl.Q8_0, wl.Q4_0, wl.Q4_1])
def test_linear_scalar_path_bitexact(cuda, oracle, qtype):
    """k not a multiple of 32 (tail block): the reference's order, bit-exact."""
    import torch
    rng = np.random.default_rng(qtype)
    for n, k, t in ((33, 40, 2), (7, 38, 1), (12, 1000, 3)):
        table = wl.numpy_quant_table(qtype, n, k, seed=k)
        x = rng.standard_normal((t, k), dtype=np.float32)
        got = mlb.linear(dev(table, cuda), qtype, n, k, dev(x, cuda))
        torch.cuda.synchronize()
        assert_bitexact(got.cpu().numpy(), oracle.linear(table, qtype, n, k, x),
                        f"{wl.QNAME[qtype]} k={k}")


def test_linear_llama3_ffn_shapes(cuda, oracle):
    """Decode step of the LLaMA-3-8B FFN (Q8_0 gate [14336, 4096] and down
    [4096, 14336]); sampled output rows against the oracle."""
    import torch
    rng = np.random.default_rng(1)
    for n, k in ((14336, 4096), (4096, 14336)):
        table_d = wl.quant_table(wl.Q8_0, n, k, cuda, seed=2)
        x = rng.standard_normal((1, k), dtype=np.float32)
        got = mlb.linear(table_d, wl.Q8_0, n, k, dev(x, cuda)).cpu().numpy()
        rows = np.unique(np.r_[0, n - 1, rng.integers(0, n, 200)])
        rb = wl.row_bytes(wl.Q8_0, k)
        tbl = table_d.view(n, rb)[torch.from_numpy(rows).to(cuda)].cpu().numpy()
        want = oracle.linear(tbl.reshape(-1), wl.Q8_0, rows.size, k, x)
        wdeq, _ = oracle.embedding(tbl.reshape(-1), wl.Q8_0, rows.size, k,
                                   np.arange(rows.size, dtype=np.int32))
        _check(got[:, rows], want, wdeq, x, f"ffn {n}x{k}")


def test_linear_rejects_bad_input(cuda):
    import torch
    w = torch.zeros(64 * 34, dtype=torch.uint8, device=cuda)
    with pytest.raises(ValueError):
        mlb.linear(w, wl.Q8_0, 3, 1024, torch.zeros(1024, device=cuda))
    with pytest.raises(ValueError):
        mlb.linear(w, wl.Q8_0, 1, 64, torch.zeros(63, device=cuda))


@pytest.mark.parametrize("qtype", [wl.F32, wl.Q8_0, wl.Q4_0, wl.Q4_1])
@pytest.mark.parametrize("n,k,t", [(128, 256, 48), (300, 4096, 49), (64, 1024, 128),
                                   (200, 512, 200), (129, 3584, 64), (1000, 4096, 257)])
def test_linear_rows_tensor_cores_vs_oracle(cuda, oracle, qtype, n, k, t):
    """Prompt-sized batches (>= 48 tokens) run on the tensor cores: Q8_0 /
    Q4_0 with d * q and x in exact fp16 pieces, Q4_1 / F32 with TF32 head +
    tail splits; same 1e-5 * sum|w x| bar as the GEMV, every output (ragged
    tiles in both n and t included)."""
    import torch
    rng = np.random.default_rng(n + 3 * k + 7 * t)
    table = wl.numpy_quant_table(qtype, n, k, seed=n + k + t)
    x = rng.standard_normal((t, k), dtype=np.float32)
    want = oracle.linear(table, qtype, n, k, x)
    got = mlb.linear_rows(dev(table, cuda), qtype, n, k, dev(x, cuda))
    torch.cuda.synchronize()
    assert mlb.wait_timeouts() == 0
    wdeq, _ = oracle.embedding(table, qtype, n, k, np.arange(n, dtype=np.int32))
    _check(got.cpu().numpy(), want, wdeq, x, f"rows {wl.QNAME[qtype]} n={n} k={k} t={t}")


@pytest.mark.parametrize("qtype", [wl.Q8_0, wl.Q4_0])
@pytest.mark.parametrize("k", [4160, 6144, 8192, 10240, 12288, 14336, 16384, 16448])
def test_linear_rows_long_rows_vs_oracle(cuda, oracle, qtype, k):
    """Rows long enough for every register width of the x split of the fp16
    prompt path (one float4 per thread of 512 up to eight: k up to 16384,
    k = 14336 being the Llama-3 down projection) and for its two-pass form
    beyond (k = 16448); one row of x spans many binades, so the per-row
    power-of-two scale and the second fp16 piece are exercised at these
    lengths too."""
    import torch
    n, t = 64, 48
    rng = np.random.default_rng(k + qtype)
    table = wl.numpy_quant_table(qtype, n, k, seed=k)
    x = rng.standard_normal((t, k), dtype=np.float32)
    x[5] = (rng.standard_normal(k) * np.exp(rng.uniform(-10, 10, k))).astype(np.float32)
    want = oracle.linear(table, qtype, n, k, x)
    got = mlb.linear_rows(dev(table, cuda), qtype, n, k, dev(x, cuda))
    torch.cuda.synchronize()
    assert mlb.wait_timeouts() == 0
    wdeq, _ = oracle.embedding(table, qtype, n, k, np.arange(n, dtype=np.int32))
    _check(got.cpu().numpy(), want, wdeq, x, f"long rows {wl.QNAME[qtype]} k={k}")


def test_linear_rows_large_values_and_small_batches(cuda, oracle):
    """x spanning many binades (the tail split matters) and batches below the
    tensor-core threshold (the GEMV path) through the same entry."""
    import torch
    rng = np.random.default_rng(9)
    n, k = 256, 1024
    table = wl.numpy_quant_table(wl.Q8_0, n, k, seed=5)
    wdeq, _ = oracle.embedding(table, wl.Q8_0, n, k, np.arange(n, dtype=np.int32))
    for t in (1, 47, 48, 96):
        x = (rng.standard_normal((t, k)) * np.exp(rng.uniform(-8, 8, (t, k)))).astype(np.float32)
        want = oracle.linear(table, wl.Q8_0, n, k, x)
        got = mlb.linear_rows(dev(table, cuda), wl.Q8_0, n, k, dev(x, cuda))
        torch.cuda.synchronize()
        _check(got.cpu().numpy(), want, wdeq, x, f"rows wide-range t={t}")


def _set_scale(table, qtype, k, row, block, d):
    bb = wl.BLOCK_BYTES[qtype]
    at = (row * (k // 32) + block) * bb
    table[at:at + 2] = np.array([d], dtype=np.float16).view(np.uint8)


@pytest.mark.parametrize("qtype", [wl.Q8_0, wl.Q4_0])
def test_linear_rows_block_scale_edges(cuda, oracle, qtype):
    """Block scales at the edges of the fp16 split of d * q: the largest
    that keeps it exact (511.75, with code -128 for Q8_0), subnormal ones
    (2^-24, 1e-6), decades apart inside one row, negative; and one of 1000,
    which sends its 128 x 128 tile to the CUDA cores.  Every output within
    the bar, ragged tiles in n and t."""
    import torch
    n, k, t = 300, 1024, 130
    rng = np.random.default_rng(qtype + 11)
    table = wl.numpy_quant_table(qtype, n, k, seed=21)
    _set_scale(table, qtype, k, 5, 3, 511.75)
    if qtype == wl.Q8_0:
        at = (5 * (k // 32) + 3) * 34 + 2
        table[at] = 0x80  # code -128
    for b, d in enumerate([2.0 ** -24, 1e-6, 6e-5, 1e-3, 10.0, 300.0, -0.02, -2.0 ** -20] * 4):
        _set_scale(table, qtype, k, 7, b, d)
    _set_scale(table, qtype, k, 200, 10, 1000.0)
    x = rng.standard_normal((t, k), dtype=np.float32)
    want = oracle.linear(table, qtype, n, k, x)
    got = mlb.linear_rows(dev(table, cuda), qtype, n, k, dev(x, cuda))
    torch.cuda.synchronize()
    assert mlb.wait_timeouts() == 0
    wdeq, _ = oracle.embedding(table, qtype, n, k, np.arange(n, dtype=np.int32))
    _check(got.cpu().numpy(), want, wdeq, x, f"scale edges {wl.QNAME[qtype]}")


@pytest.mark.parametrize("qtype", [wl.Q8_0, wl.Q4_0])
def test_linear_rows_many_tiles(cuda, oracle, qtype):
    """More 128 x 128 tiles than SMs (30 row tiles x 5 token tiles, a second
    wave of CTAs): within the bar, and two calls agree bit for bit."""
    import torch
    n, k, t = 3840, 512, 640
    rng = np.random.default_rng(qtype + 13)
    table = wl.numpy_quant_table(qtype, n, k, seed=23)
    x = rng.standard_normal((t, k), dtype=np.float32)
    want = oracle.linear(table, qtype, n, k, x)
    w, xd = dev(table, cuda), dev(x, cuda)
    a = mlb.linear_rows(w, qtype, n, k, xd)
    b = mlb.linear_rows(w, qtype, n, k, xd)
    torch.cuda.synchronize()
    assert mlb.wait_timeouts() == 0
    assert torch.equal(a, b)
    wdeq, _ = oracle.embedding(table, qtype, n, k, np.arange(n, dtype=np.int32))
    _check(a.cpu().numpy(), want, wdeq, x, f"many tiles {wl.QNAME[qtype]}")


def test_linear_rows_many_tiles_cuda_core(cuda, oracle):
    """Block scales of 1000 in the first stage of even row tiles and the last
    stage of odd ones: those tiles go to the CUDA cores, beside tensor-core
    tiles in the same launch."""
    import torch
    n, k, t = 3840, 512, 640
    rng = np.random.default_rng(14)
    table = wl.numpy_quant_table(wl.Q8_0, n, k, seed=24)
    for rt in range(n // 128):
        if rt % 2 == 0:
            _set_scale(table, wl.Q8_0, k, 128 * rt + 3, 1, 1000.0)
        else:
            _set_scale(table, wl.Q8_0, k, 128 * rt + 7, k // 32 - 1, -1000.0)
    x = rng.standard_normal((t, k), dtype=np.float32)
    want = oracle.linear(table, wl.Q8_0, n, k, x)
    got = mlb.linear_rows(dev(table, cuda), wl.Q8_0, n, k, dev(x, cuda))
    torch.cuda.synchronize()
    assert mlb.wait_timeouts() == 0
    wdeq, _ = oracle.embedding(table, wl.Q8_0, n, k, np.arange(n, dtype=np.int32))
    _check(got.cpu().numpy(), want, wdeq, x, "many tiles, CUDA-core tiles")


@pytest.mark.parametrize("qtype", [wl.Q8_0, wl.Q4_0])
def test_linear_rows_non_finite_block_scale(cuda, oracle, qtype):
    """An Inf or NaN block scale makes that row's outputs non-finite, as in
    the reference's sum; the other rows of its tile (computed on the CUDA
    cores) and of the other tiles stay within the bar."""
    import torch
    n, k, t = 256, 512, 64
    rng = np.random.default_rng(qtype + 12)
    table = wl.numpy_quant_table(qtype, n, k, seed=22)
    _set_scale(table, qtype, k, 40, 4, np.inf)
    _set_scale(table, qtype, k, 170, 0, np.nan)
    x = rng.standard_normal((t, k), dtype=np.float32)
    want = oracle.linear(table, qtype, n, k, x)
    got = mlb.linear_rows(dev(table, cuda), qtype, n, k, dev(x, cuda)).cpu().numpy()
    assert mlb.wait_timeouts() == 0
    assert not np.isfinite(got[:, 40]).any() and not np.isfinite(got[:, 170]).any()
    keep = np.array([r for r in range(n) if r not in (40, 170)])
    wdeq, _ = oracle.embedding(table, qtype, n, k, keep.astype(np.int32))
    _check(got[:, keep], want[:, keep], wdeq, x, f"non-finite scale {wl.QNAME[qtype]}")


@pytest.mark.parametrize("qtype", [wl.Q8_0, wl.Q4_1, wl.F32])
@pytest.mark.parametrize("t", [5, 64, 200])
def test_linear_rows_group_vs_single(cuda, oracle, qtype, t):
    """Three matrices of different heights (a q / k / v shape) in one grouped
    launch: each output within the same bar as the single-matrix entry; below
    48 tokens the group falls back to the GEMV per matrix."""
    import torch
    rng = np.random.default_rng(t + qtype)
    k = 512
    ns = (256, 128, 130)
    tables = [wl.numpy_quant_table(qtype, n, k, seed=n + t) for n in ns]
    x = rng.standard_normal((t, k), dtype=np.float32)
    outs = mlb.linear_rows_group([dev(tb, cuda) for tb in tables], qtype, list(ns), k,
                                 dev(x, cuda))
    torch.cuda.synchronize()
    for tb, n, got in zip(tables, ns, outs):
        want = oracle.linear(tb, qtype, n, k, x)
        wdeq, _ = oracle.embedding(tb, qtype, n, k, np.arange(n, dtype=np.int32))
        _check(got.cpu().numpy(), want, wdeq, x, f"group {wl.QNAME[qtype]} n={n} t={t}")


@pytest.fixture
def tensor_core_gemv():
    """Forces mlb.linear onto the int8 tensor-core GEMV wherever its shape
    rules allow (restores the automatic choice afterwards)."""
    previous = mlb.set_gemv_path(2)
    yield
    mlb.set_gemv_path(previous)


@pytest.mark.parametrize("qtype", [wl.Q8_0, wl.Q4_0, wl.Q4_1])
@pytest.mark.parametrize("n,k,t", [(37, 512, 1), (300, 4096, 1), (129, 1024, 3),
                                   (256, 2048, 4), (200, 4096, 5), (1000, 512, 8),
                                   (128, 4096, 2), (64, 256, 1), (256, 14336, 1),
                                   (300, 7168, 2), (5000, 1536, 1)])
def test_linear_tensor_core_gemv_vs_oracle(cuda, oracle, tensor_core_gemv, qtype, n, k, t):
    """int8 tensor-core GEMV (codes as stored, x as exact int8 digits):
    ragged tiles, 1..8 tokens (passes of 4), every ggml format, k split
    over clusters of 1..8 CTAs (evenly and unevenly)."""
    import torch
    rng = np.random.default_rng(n * 5 + k + t + qtype)
    table = wl.numpy_quant_table(qtype, n, k, seed=n + 3 * k)
    x = rng.standard_normal((t, k), dtype=np.float32)
    want = oracle.linear(table, qtype, n, k, x)
    got = mlb.linear(dev(table, cuda), qtype, n, k, dev(x, cuda))
    torch.cuda.synchronize()
    assert mlb.wait_timeouts() == 0
    wdeq, _ = oracle.embedding(table, qtype, n, k, np.arange(n, dtype=np.int32))
    _check(got.cpu().numpy(), want, wdeq, x, f"tc {wl.QNAME[qtype]} n={n} k={k} t={t}")


@pytest.mark.parametrize("qtype", [wl.Q8_0, wl.Q4_0, wl.Q4_1])
def test_linear_tensor_core_gemv_x_ranges(cuda, oracle, tensor_core_gemv, qtype):
    """Blocks of x that are all zero, tiny (1e-30), huge (1e30), or spread
    over three decades inside one block; a NaN in a block of x makes every
    output of that token NaN, as in the reference's sum."""
    import torch
    n, k = 384, 1024
    rng = np.random.default_rng(qtype + 40)
    table = wl.numpy_quant_table(qtype, n, k, seed=77)
    x = rng.standard_normal((4, k), dtype=np.float32)
    x[0, 0:32] = 0.0
    x[0, 64:96] *= np.float32(1e-30)
    x[1, 128:160] *= np.float32(1e30)
    x[2] *= (10.0 ** rng.uniform(-1.5, 1.5, k)).astype(np.float32)
    x[3, 0:32] = 0.0
    x[3, 32:64] *= np.float32(1e-30)
    want = oracle.linear(table, qtype, n, k, x)
    got = mlb.linear(dev(table, cuda), qtype, n, k, dev(x, cuda))
    torch.cuda.synchronize()
    wdeq, _ = oracle.embedding(table, qtype, n, k, np.arange(n, dtype=np.int32))
    _check(got.cpu().numpy(), want, wdeq, x, f"tc ranges {wl.QNAME[qtype]}")
    xn = x.copy()
    xn[1, 300] = np.nan
    got = mlb.linear(dev(table, cuda), qtype, n, k, dev(xn, cuda)).cpu().numpy()
    assert np.isnan(got[1]).all()
    for t in (0, 2, 3):
        assert np.isfinite(got[t]).all()


def test_linear_tensor_core_gemv_deterministic_and_auto(cuda, oracle):
    """The automatic choice takes the tensor-core GEMV for a wide matrix
    (LLaMA-3-8B FFN up, 14336 x 4096 Q8_0); repeated calls give identical
    bits and agree with the CUDA-core GEMV within the bound."""
    import torch
    n, k = 14336, 4096
    rng = np.random.default_rng(9)
    table_d = wl.quant_table(wl.Q8_0, n, k, cuda, seed=5)
    x = dev(rng.standard_normal((2, k), dtype=np.float32), cuda)
    a = mlb.linear(table_d, wl.Q8_0, n, k, x)
    b = mlb.linear(table_d, wl.Q8_0, n, k, x)
    previous = mlb.set_gemv_path(1)
    try:
        c = mlb.linear(table_d, wl.Q8_0, n, k, x)
    finally:
        mlb.set_gemv_path(previous)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    rows = np.unique(np.r_[0, n - 1, rng.integers(0, n, 200)])
    rb = wl.row_bytes(wl.Q8_0, k)
    tbl = table_d.view(n, rb)[torch.from_numpy(rows).to(cuda)].cpu().numpy()
    xs = x.cpu().numpy()
    want = oracle.linear(tbl.reshape(-1), wl.Q8_0, rows.size, k, xs)
    wdeq, _ = oracle.embedding(tbl.reshape(-1), wl.Q8_0, rows.size, k,
                               np.arange(rows.size, dtype=np.int32))
    _check(a.cpu().numpy()[:, rows], want, wdeq, xs, "auto tensor-core 14336x4096")
    _check(c.cpu().numpy()[:, rows], want, wdeq, xs, "cuda-core 14336x4096")


@pytest.mark.parametrize("qtype", [wl.Q8_0, wl.Q4_0, wl.Q4_1])
@pytest.mark.parametrize("t", [1, 3, 6])
def test_linear_rows_group_tensor_core_gemv(cuda, oracle, tensor_core_gemv, qtype, t):
    """Decode-sized grouped launch on the int8 tensor cores: three matrices
    of different heights (ragged last tiles) in one launch, tiles numbered
    matrix by matrix, k split over a cluster; each output within the bar."""
    import torch
    rng = np.random.default_rng(3 * t + qtype)
    k = 2048
    ns = (512, 130, 257)
    tables = [wl.numpy_quant_table(qtype, n, k, seed=n + t) for n in ns]
    x = rng.standard_normal((t, k), dtype=np.float32)
    outs = mlb.linear_rows_group([dev(tb, cuda) for tb in tables], qtype, list(ns), k,
                                 dev(x, cuda))
    torch.cuda.synchronize()
    assert mlb.wait_timeouts() == 0
    for tb, n, got in zip(tables, ns, outs):
        want = oracle.linear(tb, qtype, n, k, x)
        wdeq, _ = oracle.embedding(tb, qtype, n, k, np.arange(n, dtype=np.int32))
        _check(got.cpu().numpy(), want, wdeq, x, f"tc group {wl.QNAME[qtype]} n={n} t={t}")


def test_linear_rows_group_tensor_core_persistent(cuda, oracle, tensor_core_gemv):
    """More tiles than resident CTAs (two 14336-row matrices, the FFN gate /
    up): persistent clusters walk tiles of both matrices; sampled rows of
    each output against the oracle."""
    import torch
    rng = np.random.default_rng(21)
    n, k = 14336, 4096
    tabs = [wl.quant_table(wl.Q8_0, n, k, cuda, seed=s) for s in (3, 4)]
    x = rng.standard_normal((1, k), dtype=np.float32)
    outs = mlb.linear_rows_group(tabs, wl.Q8_0, [n, n], k, dev(x, cuda))
    torch.cuda.synchronize()
    rows = np.unique(np.r_[0, 127, 128, n - 1, rng.integers(0, n, 100)])
    rb = wl.row_bytes(wl.Q8_0, k)
    for tab, got in zip(tabs, outs):
        tbl = tab.view(n, rb)[torch.from_numpy(rows).to(cuda)].cpu().numpy()
        want = oracle.linear(tbl.reshape(-1), wl.Q8_0, rows.size, k, x)
        wdeq, _ = oracle.embedding(tbl.reshape(-1), wl.Q8_0, rows.size, k,
                                   np.arange(rows.size, dtype=np.int32))
        _check(got.cpu().numpy()[:, rows], want, wdeq, x, "gate/up group")
