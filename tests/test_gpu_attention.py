"""Decode attention and the KV-cache write through the C ABI, against the
reference arithmetic of src/forward.cc:50-95 (restated in the oracle and
pinned against the reference's KvCache + Softmax in tests/test_oracle.py).

Attention sums run in another order (split positions, online softmax), so
each output is checked within 1e-5 * sum_t w_t |v_t[i]| — the size of the
terms it sums; the cache write is a copy and must be bit-exact.
"""
import numpy as np
import pytest

from conftest import assert_bitexact

import mlb

pytestmark = pytest.mark.gpu


def dev(a, device):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


def _magnitude(q, keys, values, position, n_heads, n_kv):
    hd = q.shape[1]
    group = n_heads // n_kv
    out = np.empty((n_heads, hd))
    for h in range(n_heads):
        k = keys[:position + 1, h // group].astype(np.float64)
        v = values[:position + 1, h // group].astype(np.float64)
        s = k @ q[h].astype(np.float64) / np.sqrt(hd)
        w = np.exp(s - s.max())
        w /= w.sum()
        out[h] = w @ np.abs(v)
    return out


@pytest.mark.parametrize("nh,nkv,hd,pos,max_seq", [
    (4, 2, 8, 0, 16), (8, 2, 64, 37, 64), (32, 8, 128, 300, 512),
    (14, 2, 64, 255, 256), (32, 32, 128, 2047, 2048), (28, 4, 128, 4095, 4096),
    (8, 1, 256, 1000, 1024), (16, 2, 32, 9999, 10000), (64, 8, 128, 65, 70),
    # 157 slices whose partials exceed the combine's shared memory
    (8, 1, 128, 20000, 20001)])
def test_attention_decode_vs_oracle(cuda, oracle, nh, nkv, hd, pos, max_seq):
    import torch
    rng = np.random.default_rng(nh * 1000 + pos)
    q = rng.standard_normal((nh, hd), dtype=np.float32)
    keys = rng.standard_normal((max_seq, nkv, hd), dtype=np.float32)
    values = rng.standard_normal((max_seq, nkv, hd), dtype=np.float32)
    want = oracle.attention_decode(q, keys, values, pos, nh, nkv)
    got = mlb.attention_decode(dev(q, cuda), dev(keys, cuda), dev(values, cuda), pos)
    torch.cuda.synchronize()
    got = got.cpu().numpy()
    mag = _magnitude(q, keys, values, pos, nh, nkv)
    err = np.abs(got.astype(np.float64) - want)
    ratio = float((err / np.maximum(mag, 1e-30)).max())
    assert ratio <= 1e-5, f"max error / magnitude {ratio:.2e}"


def test_attention_reuses_scratch_and_rejects_bad_input(cuda, oracle):
    import torch
    rng = np.random.default_rng(4)
    nh, nkv, hd, max_seq = 8, 2, 64, 300
    keys = dev(rng.standard_normal((max_seq, nkv, hd), dtype=np.float32), cuda)
    values = dev(rng.standard_normal((max_seq, nkv, hd), dtype=np.float32), cuda)
    need = mlb.attention_scratch_floats(nh, nkv, hd, max_seq - 1)
    scratch = torch.empty(need, device=cuda)
    for pos in (0, 1, 150, max_seq - 1):
        q = rng.standard_normal((nh, hd), dtype=np.float32)
        got = mlb.attention_decode(dev(q, cuda), keys, values, pos, scratch=scratch)
        want = oracle.attention_decode(q, keys.cpu().numpy(), values.cpu().numpy(),
                                       pos, nh, nkv)
        assert np.allclose(got.cpu().numpy(), want, rtol=0, atol=1e-5)
    # scratch that starts 4 bytes past a 16-byte boundary: the slice
    # combine reads the partials from global memory instead of staging them
    odd = torch.empty(need + 1, device=cuda)[1:]
    got = mlb.attention_decode(dev(q, cuda), keys, values, max_seq - 1, scratch=odd)
    want = oracle.attention_decode(q, keys.cpu().numpy(), values.cpu().numpy(),
                                   max_seq - 1, nh, nkv)
    assert np.allclose(got.cpu().numpy(), want, rtol=0, atol=1e-5)
    with pytest.raises(IndexError):
        mlb.attention_decode(dev(q, cuda), keys, values, max_seq)
    with pytest.raises(ValueError):
        mlb.attention_decode(dev(q, cuda), keys, values, 10,
                             scratch=torch.empty(1, device=cuda))
    with pytest.raises(ValueError):   # 8 heads over 3 kv heads
        bad = torch.zeros((max_seq, 3, hd), device=cuda)
        mlb.attention_decode(dev(q, cuda), bad, bad, 10)


def test_kv_write_is_a_copy(cuda):
    import torch
    rng = np.random.default_rng(5)
    max_seq, nkv, hd = 50, 4, 32
    keys = torch.zeros((max_seq, nkv, hd), device=cuda)
    values = torch.zeros((max_seq, nkv, hd), device=cuda)
    k1 = rng.standard_normal((nkv, hd), dtype=np.float32)
    v1 = rng.standard_normal((nkv, hd), dtype=np.float32)
    mlb.kv_write(keys, values, dev(k1, cuda), dev(v1, cuda), 7)
    kb = rng.standard_normal((5, nkv, hd), dtype=np.float32)
    vb = rng.standard_normal((5, nkv, hd), dtype=np.float32)
    mlb.kv_write(keys, values, dev(kb, cuda), dev(vb, cuda), 45)
    torch.cuda.synchronize()
    kh, vh = keys.cpu().numpy(), values.cpu().numpy()
    assert_bitexact(kh[7], k1)
    assert_bitexact(vh[7], v1)
    assert_bitexact(kh[45:50], kb)
    assert_bitexact(vh[45:50], vb)
    assert not kh[:7].any() and not kh[8:45].any()
    with pytest.raises(IndexError):
        mlb.kv_write(keys, values, dev(kb, cuda), dev(vb, cuda), 46)


@pytest.fixture
def attention_path():
    """Sets mlb_set_attention_path for one test and restores it after."""
    previous = mlb.set_attention_path(0)
    yield mlb.set_attention_path
    mlb.set_attention_path(previous)


@pytest.mark.parametrize("path", [0, 1])
@pytest.mark.parametrize("nh,nkv,hd,pos,rows,max_seq", [
    (4, 2, 8, 0, 1, 16), (8, 2, 64, 0, 37, 64), (32, 8, 128, 100, 64, 512),
    (14, 2, 64, 0, 256, 256), (28, 4, 128, 2000, 48, 4096), (8, 8, 32, 5, 300, 400)])
def test_attention_rows_vs_oracle(cuda, oracle, attention_path, path, nh, nkv, hd, pos, rows,
                                  max_seq):
    """Row r of a prompt chunk equals decode attention at position pos + r
    (the reference's per-token loop, batch.cc:26-41 over forward.cc:50-95),
    with the automatic kernel choice and with the CUDA-core kernels."""
    import torch
    attention_path(path)
    rng = np.random.default_rng(nh * 7 + rows)
    q = rng.standard_normal((rows, nh, hd), dtype=np.float32)
    keys = rng.standard_normal((max_seq, nkv, hd), dtype=np.float32)
    values = rng.standard_normal((max_seq, nkv, hd), dtype=np.float32)
    got = mlb.attention_rows(dev(q, cuda), dev(keys, cuda), dev(values, cuda), pos)
    torch.cuda.synchronize()
    got = got.cpu().numpy()
    for r in sorted({0, rows // 3, rows // 2, rows - 1}):
        want = oracle.attention_decode(q[r], keys, values, pos + r, nh, nkv)
        mag = _magnitude(q[r], keys, values, pos + r, nh, nkv)
        err = np.abs(got[r].astype(np.float64) - want)
        ratio = float((err / np.maximum(mag, 1e-30)).max())
        assert ratio <= 1e-5, f"row {r}: max error / magnitude {ratio:.2e}"


def test_attention_rows_rejects_rows_beyond_cache(cuda):
    nh, nkv, hd, max_seq = 4, 2, 16, 32
    keys = torch_zeros((max_seq, nkv, hd), cuda)
    with pytest.raises(IndexError):
        mlb.attention_rows(torch_zeros((5, nh, hd), cuda), keys, keys, max_seq - 4)
    out = mlb.attention_rows(torch_zeros((4, nh, hd), cuda), keys, keys, max_seq - 4)
    assert out.shape == (4, nh, hd)


def torch_zeros(shape, device):
    import torch
    return torch.zeros(shape, dtype=torch.float32, device=device)


@pytest.mark.parametrize("nh,nkv,hd,pos,rows,max_seq", [
    (32, 8, 128, 0, 512, 600),      # group 4, a prompt from position 0
    (32, 32, 128, 100, 300, 512),   # group 1, partial last tile
    (16, 2, 64, 7, 1000, 1100),     # group 8, head_dim 64
    (64, 32, 128, 1500, 100, 1700), # group 2, chunk after a long context
    (32, 8, 64, 33, 333, 400),      # head_dim 64, ragged everything
    (28, 4, 128, 0, 700, 800),      # group 7 (Qwen2-7B): 9 rows = 63 vectors per tile
    (24, 8, 64, 10, 400, 500)])     # group 3: 21 rows = 63 vectors
@pytest.mark.parametrize("path", [1, 2])
def test_attention_row_tiles_vs_oracle(cuda, oracle, attention_path, path, nh, nkv, hd, pos,
                                       rows, max_seq):
    """Prompt chunks large enough for the query-row tile kernels — the CUDA-core
    one (path 1; n_kv_heads x row tiles >= half the SMs) and the tensor-core
    one (path 2; 128 query vectors per tile, TF32 head + tail splits of Q, K,
    P and V): sampled rows (first, last, tile edges, random) against
    per-position decode attention of the oracle."""
    import torch
    attention_path(path)
    rng = np.random.default_rng(rows + pos)
    q = rng.standard_normal((rows, nh, hd), dtype=np.float32)
    keys = rng.standard_normal((max_seq, nkv, hd), dtype=np.float32)
    values = rng.standard_normal((max_seq, nkv, hd), dtype=np.float32)
    got = mlb.attention_rows(dev(q, cuda), dev(keys, cuda), dev(values, cuda), pos)
    torch.cuda.synchronize()
    got = got.cpu().numpy()
    qr = (64 if path == 1 else 128) // (nh // nkv)
    sample = {0, 1, rows - 1, rows - 2, qr - 1, qr, min(rows - 1, 2 * qr + 1)}
    sample |= set(rng.integers(0, rows, 6).tolist())
    for r in sorted(sample):
        want = oracle.attention_decode(q[r], keys, values, pos + r, nh, nkv)
        mag = _magnitude(q[r], keys, values, pos + r, nh, nkv)
        err = np.abs(got[r].astype(np.float64) - want)
        ratio = float((err / np.maximum(mag, 1e-30)).max())
        assert ratio <= 1e-5, f"row {r}: max error / magnitude {ratio:.2e}"


def _exact_attention(q, keys, values, position, n_heads, n_kv):
    """Decode attention of one row in float64 (the ground truth the fp32
    reference itself only approximates)."""
    hd = q.shape[1]
    group = n_heads // n_kv
    out = np.empty((n_heads, hd))
    for h in range(n_heads):
        k = keys[:position + 1, h // group].astype(np.float64)
        v = values[:position + 1, h // group].astype(np.float64)
        s = (k @ q[h].astype(np.float64)) * (1.0 / np.sqrt(np.float64(hd)))
        w = np.exp(s - s.max())
        out[h] = (w / w.sum()) @ v
    return out


@pytest.mark.parametrize("nh,nkv,hd,pos,rows,max_seq,spread", [
    (32, 8, 128, 0, 2, 64, 1.0),      # two rows: one tile of mostly padding
    (8, 8, 64, 3, 5, 40, 1.0),        # group 1, head_dim 64, a few rows
    (32, 8, 128, 0, 300, 400, 6.0),   # wide score spread: the reference max moves, O rescaled
    (16, 2, 128, 50, 200, 300, 12.0), # group 8, very peaked softmax
    (28, 4, 128, 0, 129, 160, 3.0)])  # group 7 tiles of 18 rows, one row past a tile
def test_attention_rows_tensor_cores_edges(cuda, oracle, attention_path, nh, nkv, hd, pos,
                                           rows, max_seq, spread):
    """The tensor-core prompt kernel on its edges: tiles that are mostly
    padding, head_dim 64, and scores spread widely enough that the softmax's
    reference max moves by more than 8 mid-row (O rescaled in tensor
    memory); every row checked, keys past the last written position left as
    garbage (NaN) to prove they are never read.

    Bar: 1e-5 * sum_t w_t |v_t[i]| as everywhere.  With scores of standard
    deviation 6 or 12 the reference's own fp32 dot products are off by more
    than that (their rounding grows with sum_i |q_i k_i|), so there the
    worst error over all rows, relative to that magnitude, must stay within
    the larger of 1e-5 and twice the reference's own worst error over the
    same rows, both measured against a float64 evaluation (row by row, two
    roundings of this size are noise against noise)."""
    import torch
    attention_path(2)
    rng = np.random.default_rng(rows * 3 + hd)
    q = (rng.standard_normal((rows, nh, hd)) * spread).astype(np.float32)
    keys = rng.standard_normal((max_seq, nkv, hd), dtype=np.float32)
    keys[:, :, :4] *= np.linspace(0.1, 3.0, max_seq, dtype=np.float32)[:, None, None]
    values = rng.standard_normal((max_seq, nkv, hd), dtype=np.float32)
    keys[pos + rows:] = np.nan
    values[pos + rows:] = np.nan
    got = mlb.attention_rows(dev(q, cuda), dev(keys, cuda), dev(values, cuda), pos)
    torch.cuda.synchronize()
    assert mlb.wait_timeouts() == 0
    got = got.cpu().numpy()
    ours = theirs = 0.0
    for r in range(rows):
        want = oracle.attention_decode(q[r], keys, values, pos + r, nh, nkv)
        mag = np.maximum(_magnitude(q[r], keys, values, pos + r, nh, nkv), 1e-30)
        if spread > 3.0:
            exact = _exact_attention(q[r], keys, values, pos + r, nh, nkv)
            ours = max(ours, float((np.abs(got[r].astype(np.float64) - exact) / mag).max()))
            theirs = max(theirs, float((np.abs(want - exact) / mag).max()))
        else:
            ratio = float((np.abs(got[r].astype(np.float64) - want) / mag).max())
            assert ratio <= 1e-5, f"row {r}: max error / magnitude {ratio:.2e}"
    assert ours <= max(1e-5, 2.0 * theirs), \
        f"worst error {ours:.2e}, the reference's own {theirs:.2e}"
