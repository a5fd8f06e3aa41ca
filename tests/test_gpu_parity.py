"""CUDA kernels vs the reference arithmetic, through libmlb.so's C ABI.

Bars: bit-exact for the embedding gather, the residual sum h, Add/AddBias and
RoPE; max relative error <= 1e-5 (REL_TOL) for RMSNorm's y, SiLU/SwiGLU and
softmax.  Expected values come from the golden fixtures (outputs of the
reference itself) and from the CPU oracle on the same seeded inputs.
"""
import numpy as np
import pytest

from conftest import REL_TOL, assert_bitexact, assert_rel, golden

import mlb
import workloads as wl

pytestmark = pytest.mark.gpu


def dev(a, device):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


def host(t):
    import torch
    torch.cuda.synchronize()
    return t.cpu().numpy()


# ---------------------------------------------------------------- RMSNorm

@pytest.mark.parametrize("name", ["warp", "block", "block_odd", "scalar", "tiny"])
def test_rmsnorm_golden(cuda, name):
    import torch
    g = golden("rmsnorm")
    x, r, w = (dev(g[f"{name}_{s}"], cuda) for s in ("x", "r", "w"))
    eps = float(g[f"{name}_eps"])
    h = torch.empty_like(x)
    y = mlb.rms_norm(x, w, eps, residual=r, h_out=h)
    assert_bitexact(host(h), g[f"{name}_h"], "h")
    assert_rel(host(y), g[f"{name}_y"], what="y")
    assert_rel(host(mlb.rms_norm(x, w, eps)), g[f"{name}_y_plain"], what="plain")


def test_rmsnorm_kat(cuda):
    g = golden("rmsnorm")
    y = host(mlb.rms_norm(dev(g["kat_x"], cuda), dev(g["kat_w"], cuda), 1e-5))
    assert abs(y[0, 0] - 0.46291) <= 1e-4       # reference tests/test_ops.cc:41
    assert_rel(y, g["kat_y"])


@pytest.mark.parametrize("cols", [4, 32, 128, 896, 1024, 1028, 2048, 3584, 4096,
                                  8192, 14336, 16384, 32768, 32772, 40, 33, 1])
@pytest.mark.parametrize("rows", [1, 3, 37])
def test_rmsnorm_shapes_vs_oracle(cuda, oracle, rows, cols):
    import torch
    rng = np.random.default_rng(rows * 100003 + cols)
    x = rng.standard_normal((rows, cols), dtype=np.float32)
    r = rng.standard_normal((rows, cols), dtype=np.float32)
    w = (rng.standard_normal(cols, dtype=np.float32) * 0.1 + 1).astype(np.float32)
    want_y, want_h = oracle.rmsnorm(x, w, 1e-5, residual=r)
    xd, rd, wd = dev(x, cuda), dev(r, cuda), dev(w, cuda)
    h = torch.full_like(xd, float("nan"))
    y = torch.full_like(xd, float("nan"))
    mlb.rms_norm(xd, wd, 1e-5, residual=rd, h_out=h, out=y)
    assert_bitexact(host(h), want_h, "h")
    assert_rel(host(y), want_y, what="y")
    # residual without h_out, and the plain norm
    y2 = mlb.rms_norm(xd, wd, 1e-5, residual=rd)
    assert_rel(host(y2), want_y, what="y no-h")
    assert_rel(host(mlb.rms_norm(xd, wd, 1e-5)), oracle.rmsnorm(x, w, 1e-5),
               what="plain")


@pytest.mark.parametrize("rows,cols", [(2500, 896), (2400, 64), (300, 4096)])
def test_rmsnorm_large_batches_vs_oracle(cuda, oracle, rows, cols):
    """Batches that fill the SMs: eight rows per CTA for cols <= 1024 (the
    weight loaded at the store), one CTA per row above."""
    import torch
    rng = np.random.default_rng(rows + cols)
    x = rng.standard_normal((rows, cols), dtype=np.float32)
    r = rng.standard_normal((rows, cols), dtype=np.float32)
    w = (rng.standard_normal(cols, dtype=np.float32) * 0.1 + 1).astype(np.float32)
    want_y, want_h = oracle.rmsnorm(x, w, 1e-6, residual=r)
    h = torch.full((rows, cols), float("nan"), device=cuda)
    y = mlb.rms_norm(dev(x, cuda), dev(w, cuda), 1e-6, residual=dev(r, cuda), h_out=h)
    assert_bitexact(host(h), want_h, "h")
    assert_rel(host(y), want_y, what="y")


def test_rmsnorm_in_place_and_unaligned(cuda, oracle):
    """h_out may alias x; without a residual y may alias x; views that are
    not 16-byte aligned take the scalar path and still match."""
    import torch
    rng = np.random.default_rng(5)
    x = rng.standard_normal((9, 4097), dtype=np.float32)
    r = rng.standard_normal((9, 4096), dtype=np.float32)
    w = rng.standard_normal(4096, dtype=np.float32)
    want_y, want_h = oracle.rmsnorm(x[:, 1:], w, 1e-6, residual=r)
    xd = dev(x, cuda)[:, 1:]            # 4-byte aligned, not 16
    xs = xd.contiguous()
    y = mlb.rms_norm(xs, dev(w, cuda), 1e-6, residual=dev(r, cuda), h_out=xs)
    assert_bitexact(host(xs), want_h, "h in place")
    assert_rel(host(y), want_y)
    base = torch.zeros(9 * 4096 + 1, device=cuda)
    xu = base[1:].view(9, 4096)
    xu.copy_(dev(x[:, 1:], cuda))
    yu = torch.empty(9 * 4096 + 1, device=cuda)[1:].view(9, 4096)
    mlb.rms_norm(xu, dev(w, cuda), 1e-6, out=yu)
    assert_rel(host(yu), oracle.rmsnorm(x[:, 1:], w, 1e-6), what="unaligned")
    xi = dev(x[:, 1:], cuda)
    mlb.rms_norm(xi, dev(w, cuda), 1e-6, out=xi)
    assert_rel(host(xi), oracle.rmsnorm(x[:, 1:], w, 1e-6), what="y aliases x")


def test_rmsnorm_shape_mismatch_raises(cuda):
    import torch
    x = torch.zeros(2, 8, device=cuda)
    with pytest.raises(ValueError):
        mlb.rms_norm(x, torch.zeros(7, device=cuda), 1e-5)


# ---------------------------------------------------------------- SwiGLU

@pytest.mark.parametrize("name", ["vec", "scalar"])
def test_swiglu_golden(cuda, name):
    g = golden("swiglu")
    gd, ud = dev(g[f"{name}_g"], cuda), dev(g[f"{name}_u"], cuda)
    assert_rel(host(mlb.swiglu(gd, ud)), g[f"{name}_o"])
    assert_rel(host(mlb.silu(gd)), g[f"{name}_silu"], what="silu")


def test_swiglu_kat_and_extremes(cuda):
    g = golden("swiglu")
    o = host(mlb.swiglu(dev(g["kat_g"], cuda), dev(g["kat_u"], cuda)))
    assert o[0, 0] == 0.0
    assert_rel(o, g["kat_o"])
    assert_rel(host(mlb.swiglu(dev(g["edge_g"], cuda), dev(g["edge_u"], cuda))),
               g["edge_o"], what="extremes")


# 1 << 20 fits one wave of CTAs on a B200; 1.6 M to 4 M take two to four
# waves, the last one partial
@pytest.mark.parametrize("n", [1, 3, 4, 1000, 4864 * 7, 1 << 20, (1 << 20) + 3,
                               1_600_000, 2_560_000, 2_880_000, 4_000_000])
def test_swiglu_sizes_vs_oracle(cuda, oracle, n):
    rng = np.random.default_rng(n)
    g = rng.standard_normal(n, dtype=np.float32) * 3
    u = rng.standard_normal(n, dtype=np.float32)
    assert_rel(host(mlb.swiglu(dev(g, cuda), dev(u, cuda))), oracle.swiglu(g, u))


def test_elementwise_bitexact_ops(cuda, oracle):
    import torch
    rng = np.random.default_rng(3)
    a = rng.standard_normal((33, 40), dtype=np.float32)
    b = rng.standard_normal((33, 40), dtype=np.float32)
    bias = rng.standard_normal(40, dtype=np.float32)
    ad, bd = dev(a, cuda), dev(b, cuda)
    assert_bitexact(host(mlb.add(ad, bd)), oracle.add(a, b), "add")
    assert_bitexact(host(mlb.mul(ad, bd)), a * b, "mul")
    assert_bitexact(host(mlb.add_bias(ad, dev(bias, cuda))),
                    oracle.add(a, np.broadcast_to(bias, a.shape)), "add_bias")
    assert_bitexact(host(mlb.add_bias(ad, None)), a, "bias copy")
    odd = rng.standard_normal((5, 7), dtype=np.float32)
    ob = rng.standard_normal(7, dtype=np.float32)
    assert_bitexact(host(mlb.add_bias(dev(odd, cuda), dev(ob, cuda))),
                    oracle.add(odd, np.broadcast_to(ob, odd.shape)), "bias scalar")
    # in place: out aliases an input
    out = dev(a, cuda)
    mlb.swiglu(out, bd, out=out)
    assert_rel(host(out), oracle.swiglu(a, b), what="swiglu in place")


@pytest.mark.parametrize("n", [1_600_000, 2_880_000])
def test_elementwise_wave_sizes_in_place(cuda, oracle, n):
    """Arrays of several waves of CTAs: the output aliasing an input, and
    the bit-exact binary ops at the same sizes."""
    rng = np.random.default_rng(n)
    a = rng.standard_normal(n, dtype=np.float32)
    b = rng.standard_normal(n, dtype=np.float32)
    ad, bd = dev(a, cuda), dev(b, cuda)
    assert_bitexact(host(mlb.add(ad, bd)), oracle.add(a, b), "add")
    assert_bitexact(host(mlb.mul(ad, bd)), a * b, "mul")
    out = dev(a, cuda)
    mlb.swiglu(out, bd, out=out)
    assert_rel(host(out), oracle.swiglu(a, b), what="swiglu in place")


# ---------------------------------------------------------------- Softmax

@pytest.mark.parametrize("name", ["warp", "block", "scalar"])
def test_softmax_golden(cuda, name):
    import torch
    g = golden("softmax")
    vl = dev(g[f"{name}_len"], cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    y = mlb.softmax_rows(dev(g[f"{name}_x"], cuda), vl, status=status)
    assert_rel(host(y), g[f"{name}_y"])
    assert mlb.status_check(status) == 0


def test_softmax_kat(cuda):
    g = golden("softmax")
    y = host(mlb.softmax_rows(dev(g["kat_x"], cuda)))
    assert abs(float(y.sum()) - 1.0) <= 1e-5 and y[0, 2] > y[0, 1]
    assert_rel(y, g["kat_y"])


@pytest.mark.parametrize("cols", [1, 4, 37, 64, 256, 1024, 1040, 4096, 16384,
                                  32768, 40000])
def test_softmax_shapes_vs_oracle(cuda, oracle, cols):
    rng = np.random.default_rng(cols)
    rows = 19
    x = rng.standard_normal((rows, cols), dtype=np.float32) * 2
    vl = rng.integers(1, cols + 1, rows).astype(np.int32)
    vl[0], vl[-1] = 1, cols
    want, bad = oracle.softmax_rows(x, vl)
    assert bad == 0
    assert_rel(host(mlb.softmax_rows(dev(x, cuda), dev(vl, cuda))), want)
    want_full, _ = oracle.softmax_rows(x)
    assert_rel(host(mlb.softmax_rows(dev(x, cuda))), want_full, what="full rows")


@pytest.mark.parametrize("rows,cols", [(2100, 1024), (9000, 256), (3584, 256)])
def test_softmax_large_masked_batch(cuda, oracle, rows, cols):
    """Many warp-per-row rows (C1's 14 x 256 rows among them): causal
    lengths plus a few bad ones, flagged and written as zeros."""
    import torch
    rng = np.random.default_rng(rows + cols)
    x = rng.standard_normal((rows, cols), dtype=np.float32) * 2
    vl = (np.arange(rows) % cols + 1).astype(np.int32)
    bad_rows = [5, rows // 2, rows - 1]
    vl[bad_rows] = [0, cols + 1, -7]
    want, bad = oracle.softmax_rows(x, vl)
    assert bad != 0
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    got = host(mlb.softmax_rows(dev(x, cuda), dev(vl, cuda), status=status))
    assert mlb.status_check(status) == mlb.STATUS_BAD_LENGTH
    assert not got[bad_rows].any()
    good = np.ones(rows, bool)
    good[bad_rows] = False
    assert_rel(got[good], want[good])


def test_softmax_bad_lengths_flagged(cuda):
    import torch
    x = torch.randn(4, 64, device=cuda)
    vl = torch.tensor([0, 65, -3, 64], dtype=torch.int32, device=cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    y = mlb.softmax_rows(x, vl, status=status)
    assert mlb.status_check(status) == mlb.STATUS_BAD_LENGTH
    yh = host(y)
    assert not yh[:3].any()
    assert abs(yh[3].sum() - 1.0) < 1e-5


# ---------------------------------------------------------------- RoPE

def _rope_gpu(cuda, q, k, pos, theta, neox, bq=None, bk=None, table_rows=None):
    import torch
    hd = q.shape[2]
    rows = int(pos.max()) + 1 if table_rows is None else table_rows
    table = dev(mlb.rope_table(theta, hd, rows), cuda)
    qd, kd = dev(q, cuda), dev(k, cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    mlb.rope(qd, kd, dev(pos, cuda), table, bool(neox),
             None if bq is None else dev(bq, cuda),
             None if bk is None else dev(bk, cuda), status=status)
    return host(qd), host(kd), mlb.status_check(status)


@pytest.mark.parametrize("name", ["neox_bias", "normal", "normal_small", "neox_small"])
def test_rope_golden(cuda, name):
    g = golden("rope")
    bq = g[f"{name}_bq"] if f"{name}_bq" in g.files else None
    bk = g[f"{name}_bk"] if f"{name}_bk" in g.files else None
    q, k, st = _rope_gpu(cuda, g[f"{name}_q"], g[f"{name}_k"], g[f"{name}_pos"],
                         float(g[f"{name}_theta"]), int(g[f"{name}_neox"]), bq, bk)
    assert st == 0
    assert_bitexact(q, g[f"{name}_qo"], "q")
    assert_bitexact(k, g[f"{name}_ko"], "k")


def test_rope_kat(cuda):
    g = golden("rope")
    for neox in (0, 1):
        q, k, _ = _rope_gpu(cuda, g["kat_in"], g["kat_in"], np.array([1], np.int32),
                            1e4, neox)
        assert_bitexact(q, g[f"kat{neox}_q"])
        assert_bitexact(k, g[f"kat{neox}_k"])


@pytest.mark.parametrize("neox", [0, 1])
@pytest.mark.parametrize("nq,nk,hd", [(14, 2, 64), (32, 32, 128), (32, 8, 128),
                                      (28, 4, 128), (3, 1, 6), (2, 2, 12),
                                      (1, 0, 8), (5, 3, 256)])
def test_rope_shapes_vs_oracle(cuda, oracle, neox, nq, nk, hd):
    rng = np.random.default_rng(nq * 7 + hd + neox)
    t = 23
    q = rng.standard_normal((t, nq, hd), dtype=np.float32)
    k = rng.standard_normal((t, nk, hd), dtype=np.float32)
    bq = rng.standard_normal(nq * hd, dtype=np.float32) * 0.02
    bk = rng.standard_normal(nk * hd, dtype=np.float32) * 0.02 if nk else None
    pos = rng.integers(0, 70000, t).astype(np.int32)
    pos[0], pos[1] = 0, 65535
    theta = 1e6 if neox else 5e5
    wq, wk, bad = oracle.rope(q, k, pos, theta, neox, bq, bk)
    assert bad == 0
    gq, gk, st = _rope_gpu(cuda, q, k, pos, theta, neox, bq, bk)
    assert st == 0
    assert_bitexact(gq, wq, "q")
    assert_bitexact(gk, wk, "k")


def test_rope_bad_position_flagged(cuda, oracle):
    rng = np.random.default_rng(9)
    q = rng.standard_normal((3, 2, 8), dtype=np.float32)
    k = rng.standard_normal((3, 1, 8), dtype=np.float32)
    bq = rng.standard_normal(16, dtype=np.float32)
    pos = np.array([5, -1, 100], np.int32)
    gq, gk, st = _rope_gpu(cuda, q, k, pos, 1e4, 0, bq, None, table_rows=10)
    assert st == mlb.STATUS_BAD_POSITION
    wq, wk, _ = oracle.rope(q[:1], k[:1], pos[:1], 1e4, 0, bq, None)
    assert_bitexact(gq[:1], wq)
    # tokens outside the table: bias added, not rotated
    assert_bitexact(gq[1:], q[1:] + bq.reshape(2, 8))
    assert_bitexact(gk[1:], k[1:])


# ---------------------------------------------------------------- Embedding

@pytest.mark.parametrize("qtype", [wl.F32, wl.Q8_0, wl.Q4_0, wl.Q4_1])
def test_embedding_golden(cuda, qtype):
    import torch
    g = golden("embedding")
    qn = wl.QNAME[qtype]
    keys = [(f"{qn}_{c}", 12, c) for c in (96, 40, 38)]
    if qtype != wl.F32:
        keys.append((f"{qn}_bits", 40, 64))
    for key, vocab, cols in keys:
        status = torch.zeros(1, dtype=torch.int32, device=cuda)
        out = mlb.embedding_rows(dev(g[f"{key}_table"], cuda), qtype, vocab, cols,
                                 dev(g[f"{key}_tokens"], cuda), status=status)
        assert_bitexact(host(out), g[f"{key}_out"], key)
        assert mlb.status_check(status) == 0


def test_fp16_all_patterns_exhaustive(cuda, oracle):
    """All 65536 fp16 scale patterns x a spread of quant codes per format."""
    codes8 = np.array([1, -1, 127, -127, 0, 64, -64, 3] * 4, np.int8)
    fp16 = np.arange(65536, dtype=np.uint16)
    tokens = np.arange(65536, dtype=np.int32)
    # Q8_0: d = pattern, qs = codes
    t8 = np.zeros((65536, 34), np.uint8)
    t8[:, 0:2] = fp16.view(np.uint8).reshape(-1, 2)
    t8[:, 2:34] = codes8.view(np.uint8)
    out = host(mlb.embedding_rows(dev(t8.reshape(-1), cuda), wl.Q8_0, 65536, 32,
                                  dev(tokens, cuda)))
    assert_bitexact(out[:, 0], golden("fp16")["bits"].view(np.float32), "d*1")
    want, _ = oracle.embedding(t8.reshape(-1), wl.Q8_0, 65536, 32, tokens)
    assert_bitexact(out, want, "Q8_0 all scales")
    # Q4_0 / Q4_1: every nibble value 0..15 in both halves
    nib = np.arange(16, dtype=np.uint8)
    qs = (nib | (nib[::-1] << 4)).astype(np.uint8)
    for qtype, bb, off in ((wl.Q4_0, 18, 2), (wl.Q4_1, 20, 4)):
        t = np.zeros((65536, bb), np.uint8)
        t[:, 0:2] = fp16.view(np.uint8).reshape(-1, 2)
        if qtype == wl.Q4_1:
            t[:, 2:4] = fp16[::-1].copy().view(np.uint8).reshape(-1, 2)
        t[:, off:off + 16] = qs
        out = host(mlb.embedding_rows(dev(t.reshape(-1), cuda), qtype, 65536, 32,
                                      dev(tokens, cuda)))
        want, _ = oracle.embedding(t.reshape(-1), qtype, 65536, 32, tokens)
        assert_bitexact(out, want, wl.QNAME[qtype])


@pytest.mark.parametrize("qtype", [wl.F32, wl.Q8_0, wl.Q4_0, wl.Q4_1])
@pytest.mark.parametrize("cols", [896, 4096, 3584, 40, 36, 38, 1, 64])
def test_embedding_shapes_vs_oracle(cuda, oracle, qtype, cols):
    vocab = 300
    table = wl.numpy_quant_table(qtype, vocab, cols, seed=cols)
    rng = np.random.default_rng(cols + qtype)
    tokens = rng.integers(0, vocab, 77).astype(np.int32)
    tokens[:3] = [0, vocab - 1, 0]
    want, bad = oracle.embedding(table, qtype, vocab, cols, tokens)
    assert bad == 0
    got = mlb.embedding_rows(dev(table, cuda), qtype, vocab, cols, dev(tokens, cuda))
    assert_bitexact(host(got), want, f"{wl.QNAME[qtype]} cols={cols}")


def test_embedding_bad_tokens_flagged(cuda, oracle):
    import torch
    table = wl.numpy_quant_table(wl.Q8_0, 10, 64, seed=1)
    tokens = np.array([3, -1, 10, 9], np.int32)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    out = host(mlb.embedding_rows(dev(table, cuda), wl.Q8_0, 10, 64,
                                  dev(tokens, cuda), status=status))
    assert mlb.status_check(status) == mlb.STATUS_BAD_TOKEN
    assert not out[1:3].any()
    want, _ = oracle.embedding(table, wl.Q8_0, 10, 64, tokens[[0, 3]])
    assert_bitexact(out[[0, 3]], want)


@pytest.mark.parametrize("qtype,offset", [(wl.Q8_0, 2), (wl.Q8_0, 14), (wl.Q4_0, 6),
                                          (wl.Q4_1, 4), (wl.Q4_1, 12)])
@pytest.mark.parametrize("cols,T", [(896, 3000), (4096, 77), (4096, 3000), (40000, 5)])
def test_embedding_table_not_16_byte_aligned(cuda, oracle, qtype, offset, cols, T):
    """A table that is only 2-byte (Q8_0, Q4_0) or 4-byte (Q4_1) aligned, as
    the C ABI allows: staged windows then start before the table or end past
    it, and only the table's own bytes may be read.  Covers the warp-per-row,
    two-rows-per-CTA, split-row (few tokens) and long-row (split to fit
    shared memory) forms."""
    import torch
    vocab = 7
    table = wl.numpy_quant_table(qtype, vocab, cols, seed=cols + offset)
    buf = torch.zeros(table.size + 32, dtype=torch.uint8, device=cuda)
    buf[offset:offset + table.size] = dev(table, cuda)
    view = buf[offset:offset + table.size]
    rng = np.random.default_rng(T + offset)
    tokens = rng.integers(0, vocab, T).astype(np.int32)
    tokens[:2] = [0, vocab - 1]
    tokens[-1] = vocab - 1
    want, bad = oracle.embedding(table, qtype, vocab, cols, tokens)
    assert bad == 0
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    got = mlb.embedding_rows(view, qtype, vocab, cols, dev(tokens, cuda), status=status)
    assert_bitexact(host(got), want, f"{wl.QNAME[qtype]} cols={cols} offset={offset}")
    assert mlb.status_check(status) == 0


# ---------------------------------------------------------------- configs

@pytest.mark.parametrize("name", ["qwen2-0.5b-t256", "llama-7b-t64"])
def test_small_configs_full_vs_oracle(cuda, oracle, name):
    """The two single-GPU configs checked in full, every operator."""
    import torch
    cfg = wl.CONFIGS[name]
    d = wl.make_inputs(cfg, cuda)
    hn = {k: (v.cpu().numpy() if v is not None else None) for k, v in d.items()}
    # embedding
    mlb.embedding_rows(d["table"], cfg.qtype, cfg.vocab, cfg.hidden, d["tokens"],
                       out=d["emb_out"], status=d["status"])
    want, bad = oracle.embedding(hn["table"], cfg.qtype, cfg.vocab, cfg.hidden,
                                 hn["tokens"])
    assert bad == 0
    assert_bitexact(host(d["emb_out"]), want, "embedding")
    # (residual) RMSNorm
    mlb.rms_norm(d["x"], d["w"], cfg.eps, residual=d["residual"], h_out=d["h"],
                 out=d["y"])
    if cfg.residual:
        wy, wh = oracle.rmsnorm(hn["x"], hn["w"], cfg.eps, residual=hn["residual"])
        assert_bitexact(host(d["h"]), wh, "h")
    else:
        wy = oracle.rmsnorm(hn["x"], hn["w"], cfg.eps)
    assert_rel(host(d["y"]), wy, what="rmsnorm")
    # RoPE
    table = dev(mlb.rope_table(cfg.theta, cfg.head_dim, cfg.max_position() + 1), cuda)
    mlb.rope(d["q"], d["k"], d["positions"], table, cfg.neox, d["bq"], d["bk"],
             status=d["status"])
    wq, wk, bad = oracle.rope(hn["q"], hn["k"], hn["positions"], cfg.theta,
                              cfg.neox, hn["bq"], hn["bk"])
    assert bad == 0
    assert_bitexact(host(d["q"]), wq, "rope q")
    assert_bitexact(host(d["k"]), wk, "rope k")
    # SwiGLU
    mlb.swiglu(d["gate"], d["up"], out=d["ffn_out"])
    assert_rel(host(d["ffn_out"]), oracle.swiglu(hn["gate"], hn["up"]), what="swiglu")
    # causal softmax rows
    if cfg.softmax_cols:
        mlb.softmax_rows(d["scores"], d["valid_len"], out=d["probs"],
                         status=d["status"])
        want, bad = oracle.softmax_rows(hn["scores"], hn["valid_len"])
        assert bad == 0
        assert_rel(host(d["probs"]), want, what="softmax")
    assert mlb.status_check(d["status"]) == 0


# ---------------------------------------------------------------- per-token forms

def test_rope_consecutive_positions_without_array(cuda, oracle):
    """positions = NULL: token t sits at position_base + t (prefill chunk);
    rows = 1 is the reference's per-token CudaRope call."""
    import torch
    rng = np.random.default_rng(21)
    for neox, base, t in ((0, 0, 40), (1, 1000, 33), (0, 2047, 1), (1, 65535, 1)):
        q = rng.standard_normal((t, 4, 64), dtype=np.float32)
        k = rng.standard_normal((t, 2, 64), dtype=np.float32)
        pos = np.arange(base, base + t, dtype=np.int32)
        wq, wk, _ = oracle.rope(q, k, pos, 1e6, neox)
        table = dev(mlb.rope_table(1e6, 64, base + t), cuda)
        qd, kd = dev(q, cuda), dev(k, cuda)
        mlb.rope(qd, kd, None, table, bool(neox), position_base=base)
        assert_bitexact(host(qd), wq, "q")
        assert_bitexact(host(kd), wk, "k")
    with pytest.raises(IndexError):
        mlb.rope(qd, kd, None, table, True, position_base=base + 1)


@pytest.mark.parametrize("qtype", [wl.F32, wl.Q8_0, wl.Q4_0, wl.Q4_1])
def test_embedding_row_host_token(cuda, oracle, qtype):
    vocab, cols = 50, 896
    table = wl.numpy_quant_table(qtype, vocab, cols, seed=3)
    td = dev(table, cuda)
    for token in (0, 17, vocab - 1):
        want, _ = oracle.embedding(table, qtype, vocab, cols,
                                   np.array([token], np.int32))
        got = mlb.embedding_row(td, qtype, vocab, cols, token)
        assert_bitexact(host(got), want[0], f"token {token}")
    for bad in (-1, vocab):
        with pytest.raises(IndexError):
            mlb.embedding_row(td, qtype, vocab, cols, bad)


def test_large_batch_flat_grids(cuda, oracle):
    """Flat one-item-per-thread grids over many rows: sampled rows match."""
    import torch
    rng = np.random.default_rng(8)
    T, vocab, cols = 20000, 3000, 4096
    table = wl.numpy_quant_table(wl.Q8_0, vocab, cols, seed=5)
    tokens = rng.integers(0, vocab, T).astype(np.int32)
    out = host(mlb.embedding_rows(dev(table, cuda), wl.Q8_0, vocab, cols,
                                  dev(tokens, cuda)))
    rows = np.r_[0:3, T - 3:T, rng.integers(0, T, 50)]
    want, _ = oracle.embedding(table, wl.Q8_0, vocab, cols, tokens[rows])
    assert_bitexact(out[rows], want, "embedding sample")
    q = rng.standard_normal((T, 8, 128), dtype=np.float32)
    k = rng.standard_normal((T, 2, 128), dtype=np.float32)
    table_r = dev(mlb.rope_table(5e5, 128, T), cuda)
    qd, kd = dev(q, cuda), dev(k, cuda)
    mlb.rope(qd, kd, None, table_r, False)
    wq, wk, _ = oracle.rope(q[rows], k[rows], rows.astype(np.int32), 5e5, 0)
    assert_bitexact(host(qd)[rows], wq, "rope q sample")
    assert_bitexact(host(kd)[rows], wk, "rope k sample")


@pytest.mark.parametrize("qtype", [wl.Q8_0, wl.Q4_0, wl.Q4_1])
def test_embedding_last_row_at_unaligned_table_end(cuda, oracle, qtype):
    """The staged 16-byte window of the last row would run past a table
    whose size is not a multiple of 16; those bytes are never read."""
    for vocab, cols in ((3, 896), (1, 40), (5, 36)):
        table = wl.numpy_quant_table(qtype, vocab, cols, seed=vocab)
        tokens = np.array([vocab - 1, 0, vocab - 1], np.int32)
        want, _ = oracle.embedding(table, qtype, vocab, cols, tokens)
        got = mlb.embedding_rows(dev(table, cuda), qtype, vocab, cols,
                                 dev(tokens, cuda))
        assert_bitexact(host(got), want, f"{wl.QNAME[qtype]} vocab={vocab}")


@pytest.mark.parametrize("qtype,cols", [(wl.Q8_0, 2432), (wl.Q8_0, 4096), (wl.Q4_0, 8192),
                                        (wl.Q4_1, 8192)])
def test_embedding_large_batch_long_rows(cuda, oracle, qtype, cols):
    """Large batches of long rows (the staged one-row-per-CTA gather): every
    row bit-exact, out-of-range ids zeroed and flagged, and the last row of a
    table whose size is not a multiple of 16 bytes."""
    import torch
    rng = np.random.default_rng(cols + qtype)
    vocab, T = 5, 3000
    table = wl.numpy_quant_table(qtype, vocab, cols, seed=cols)
    tokens = rng.integers(0, vocab, T).astype(np.int32)
    tokens[-1] = vocab - 1
    tokens[[7, 1500]] = [-1, vocab]
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    got = host(mlb.embedding_rows(dev(table, cuda), qtype, vocab, cols, dev(tokens, cuda),
                                  status=status))
    ok = (tokens >= 0) & (tokens < vocab)
    want, _ = oracle.embedding(table, qtype, vocab, cols, tokens[ok])
    assert_bitexact(got[ok], want, f"{wl.QNAME[qtype]} cols={cols}")
    assert (got[~ok] == 0).all()
    assert int(status.item()) & mlb.STATUS_BAD_TOKEN
