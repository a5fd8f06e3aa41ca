"""The attention entry point that allocates nothing
(mlb_attention_decode_noalloc_f32), through the C ABI.

It exists for callers that cannot give the library device scratch — a
plugin inside a framework that owns every device allocation, or a decode
loop that must not call cudaMalloc / cudaFree because they can synchronise
the device — and keeps its slice partials in a 4 MiB array inside the
library instead.  Its output must match the scratch-taking entry point's
(mlb_attention_decode_f32) within the attention tests' tolerance, 1e-5 of
sum_t w_t |v_t[i]|, on consecutive calls (the shared array keeps the previous
call's contents), and sizes that need more scratch than the array holds must
be refused with a message, not run.

This file sorts last so that a run stopping at the first failure has already
run every other test; it also passes on its own in a fresh process.
"""
import ctypes

import numpy as np
import pytest

import mlb

pytestmark = pytest.mark.gpu


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def _noalloc(lib, q, keys, values, out, position, stream):
    max_seq, n_kv, hd = keys.shape
    return lib.mlb_attention_decode_noalloc_f32(
        _ptr(q), _ptr(keys), _ptr(values), _ptr(out), position, max_seq,
        q.shape[0], n_kv, hd, ctypes.c_void_p(stream))


def _with_scratch(lib, q, keys, values, out, position, stream):
    import torch
    max_seq, n_kv, hd = keys.shape
    need = lib.mlb_attention_scratch_floats(q.shape[0], n_kv, hd, position)
    scratch = torch.empty(need, device=q.device)
    return lib.mlb_attention_decode_f32(
        _ptr(q), _ptr(keys), _ptr(values), _ptr(out), position, max_seq,
        q.shape[0], n_kv, hd, _ptr(scratch), need, ctypes.c_void_p(stream))


def _magnitude(q, keys, values, position, n_kv):
    n_heads, hd = q.shape
    group = n_heads // n_kv
    out = np.empty((n_heads, hd))
    for h in range(n_heads):
        k = keys[:position + 1, h // group].astype(np.float64)
        v = values[:position + 1, h // group].astype(np.float64)
        s = k @ q[h].astype(np.float64) / np.sqrt(hd)
        w = np.exp(s - s.max())
        out[h] = (w / w.sum()) @ np.abs(v)
    return out


def test_noalloc_matches_scratch_entry_on_consecutive_calls():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    lib = mlb.load()
    dev = torch.device("cuda:0")
    stream = torch.cuda.current_stream().cuda_stream
    rng = np.random.default_rng(11)
    # two calls in a row with different sizes: the second sees the array as
    # the first left it
    for n_heads, n_kv, hd, max_seq, position in ((32, 8, 128, 4096, 4095),
                                                (14, 2, 64, 300, 77)):
        qh = rng.standard_normal((n_heads, hd), dtype=np.float32)
        kh = rng.standard_normal((max_seq, n_kv, hd), dtype=np.float32)
        vh = rng.standard_normal((max_seq, n_kv, hd), dtype=np.float32)
        q, keys, values = (torch.from_numpy(a).to(dev) for a in (qh, kh, vh))
        got = torch.full((n_heads, hd), float("nan"), device=dev)
        want = torch.full((n_heads, hd), float("nan"), device=dev)
        assert _noalloc(lib, q, keys, values, got, position, stream) == 0, \
            lib.mlb_last_error()
        assert _with_scratch(lib, q, keys, values, want, position, stream) == 0, \
            lib.mlb_last_error()
        torch.cuda.synchronize()
        g, w = got.cpu().numpy(), want.cpu().numpy()
        assert np.isfinite(g).all()
        mag = _magnitude(qh, kh, vh, position, n_kv)
        err = np.abs(g.astype(np.float64) - w.astype(np.float64))
        assert float((err / np.maximum(mag, 1e-30)).max()) <= 1e-5


def test_noalloc_refuses_sizes_beyond_its_array():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    lib = mlb.load()
    dev = torch.device("cuda:0")
    # 1000 kv heads x 8 query heads of 256 values: one slice each, 2.08 M
    # floats of partials
    n_heads, n_kv, hd, max_seq = 8000, 1000, 256, 100
    need = lib.mlb_attention_scratch_floats(n_heads, n_kv, hd, max_seq - 1)
    assert need > (1 << 20)
    q = torch.zeros((n_heads, hd), device=dev)
    kv = torch.zeros((max_seq, n_kv, hd), device=dev)
    out = torch.zeros((n_heads, hd), device=dev)
    rc = lib.mlb_attention_decode_noalloc_f32(
        _ptr(q), _ptr(kv), _ptr(kv), _ptr(out), max_seq - 1, max_seq, n_heads,
        n_kv, hd, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 1
    assert b"floats of scratch" in lib.mlb_last_error()
