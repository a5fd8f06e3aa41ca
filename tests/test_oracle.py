"""Pins the CPU oracle (oracle/mlb_oracle.c) before it is trusted.

1. Against the golden fixtures made by the reference itself
   (tests/golden/make_golden.py, outputs of mini-lla's ops.cc / quant.cc).
2. Against the reference's own unit-test constants (tests/test_ops.cc:35-82,
   tests/test_quant.cc:13-64 of the reference).
3. Against the reference library built from source (oracle/_ref), on fresh
   seeded inputs, when that library is present.
All comparisons are bit-exact: the oracle keeps the reference's evaluation
order and calls the same libm functions.
"""
import math

import numpy as np
import pytest

from conftest import assert_bitexact, golden

import workloads as wl


def test_fp16_all_patterns(oracle):
    """Fp16ToFloat (quant.cc:44-71) for all 65536 bit patterns: the oracle's
    decode equals the reference's decode (seen through d * 1.0f) and numpy's
    IEEE half conversion wherever the value is not a NaN."""
    from oracle import fp16_bits_to_f32_numpy
    ref_bits = golden("fp16")["bits"]
    mine = np.array([oracle.fp16_to_f32(i) for i in range(65536)], np.float32)
    # decode then * 1.0f exactly as the reference's Q8_0 path does
    table = np.zeros((65536, 34), np.uint8)
    table[:, 0:2] = np.arange(65536, dtype=np.uint16).view(np.uint8).reshape(-1, 2)
    table[:, 2] = 1
    out, bad = oracle.embedding(table.reshape(-1), wl.Q8_0, 65536, 32,
                                np.arange(65536, dtype=np.int32))
    assert bad == 0
    assert np.array_equal(out[:, 0].view(np.uint32), ref_bits)
    assert_bitexact(mine, ref_bits.view(np.float32), "fp16 decode")
    npy = fp16_bits_to_f32_numpy(np.arange(65536, dtype=np.uint16))
    finite = ~np.isnan(npy)
    assert np.array_equal(mine[finite].view(np.uint32), npy[finite].view(np.uint32))
    # subnormals, zero signs, infinities explicitly
    assert oracle.fp16_to_f32(0x0001) == 2.0 ** -24
    assert oracle.fp16_to_f32(0x03ff) == 1023 * 2.0 ** -24
    assert math.copysign(1.0, oracle.fp16_to_f32(0x8000)) == -1.0
    assert oracle.fp16_to_f32(0x7c00) == math.inf
    assert oracle.fp16_to_f32(0xfc00) == -math.inf


def test_rmsnorm_golden(oracle):
    g = golden("rmsnorm")
    y = oracle.rmsnorm(g["kat_x"], g["kat_w"], 1e-5)
    assert abs(y[0, 0] - 0.46291) <= 1e-4           # test_ops.cc:41
    assert_bitexact(y, g["kat_y"], "kat")
    for name in ("warp", "block", "block_odd", "scalar", "tiny"):
        eps = float(g[f"{name}_eps"])
        y, h = oracle.rmsnorm(g[f"{name}_x"], g[f"{name}_w"], eps,
                              residual=g[f"{name}_r"])
        assert_bitexact(h, g[f"{name}_h"], f"{name} h")
        assert_bitexact(y, g[f"{name}_y"], f"{name} y")
        assert_bitexact(oracle.rmsnorm(g[f"{name}_x"], g[f"{name}_w"], eps),
                        g[f"{name}_y_plain"], f"{name} plain")


def test_swiglu_golden(oracle):
    g = golden("swiglu")
    o = oracle.swiglu(g["kat_g"], g["kat_u"])
    assert o[0, 0] == 0.0
    assert abs(o[0, 1] - 2.0 / (1.0 + math.exp(-1.0))) <= 1e-5   # test_ops.cc:53
    assert_bitexact(o, g["kat_o"], "kat")
    for name in ("vec", "scalar"):
        assert_bitexact(oracle.swiglu(g[f"{name}_g"], g[f"{name}_u"]),
                        g[f"{name}_o"], name)
        assert_bitexact(oracle.silu(g[f"{name}_g"]), g[f"{name}_silu"],
                        f"{name} silu")
    assert_bitexact(oracle.swiglu(g["edge_g"], g["edge_u"]), g["edge_o"], "edge")


def test_softmax_golden(oracle):
    g = golden("softmax")
    y, bad = oracle.softmax_rows(g["kat_x"])
    assert bad == 0
    assert abs(float(y.sum()) - 1.0) <= 1e-5          # test_ops.cc:45-46
    assert y[0, 2] > y[0, 1]                          # test_ops.cc:47
    assert_bitexact(y, g["kat_y"], "kat")
    for name in ("warp", "block", "scalar"):
        y, bad = oracle.softmax_rows(g[f"{name}_x"], g[f"{name}_len"])
        assert bad == 0
        assert_bitexact(y, g[f"{name}_y"], name)


def test_softmax_rejects_empty(oracle):
    """The reference throws on an empty vector (ops.cc:84-86); the row form
    reports it and writes zeros."""
    x = np.ones((2, 4), np.float32)
    y, bad = oracle.softmax_rows(x, np.array([0, 5], np.int32))
    assert bad == 2 and not y.any()


def _rope_golden_case(g, name):
    bq = g[f"{name}_bq"] if f"{name}_bq" in g.files else None
    bk = g[f"{name}_bk"] if f"{name}_bk" in g.files else None
    return (g[f"{name}_q"], g[f"{name}_k"], g[f"{name}_pos"],
            float(g[f"{name}_theta"]), int(g[f"{name}_neox"]), bq, bk)


def test_rope_golden(oracle):
    g = golden("rope")
    for neox in (0, 1):
        q, k, bad = oracle.rope(g["kat_in"], g["kat_in"], np.array([1], np.int32),
                                1e4, neox)
        assert bad == 0
        # test_ops.cc:76-79: (cos 1, sin 1)
        assert abs(q[0, 0, 0] - math.cos(1.0)) <= 1e-5
        assert abs(q[0, 0, 1] - math.sin(1.0)) <= 1e-5
        assert_bitexact(q, g[f"kat{neox}_q"], f"kat{neox} q")
        assert_bitexact(k, g[f"kat{neox}_k"], f"kat{neox} k")
    for name in ("neox_bias", "normal", "normal_small", "neox_small"):
        q, k, pos, theta, neox, bq, bk = _rope_golden_case(g, name)
        qo, ko, bad = oracle.rope(q, k, pos, theta, neox, bq, bk)
        assert bad == 0
        assert_bitexact(qo, g[f"{name}_qo"], f"{name} q")
        assert_bitexact(ko, g[f"{name}_ko"], f"{name} k")


def test_rope_table_matches_inline_angles(oracle):
    """The host table holds exactly the cos/sin the reference evaluates
    inline: rotating a unit pair by the table equals the oracle's inline
    rotation, for both layouts and large positions."""
    hd, theta = 8, 5e5
    positions = np.array([0, 1, 2047, 16383, 65535], np.int32)
    table = oracle.rope_table(theta, hd, 0, 65536)
    for neox in (0, 1):
        q = np.zeros((positions.size, 1, hd), np.float32)
        half = hd // 2
        for j in range(half):
            a = j if neox else 2 * j
            q[:, 0, a] = 1.0
        qo, _, _ = oracle.rope(q, q.copy(), positions, theta, neox)
        for j in range(half):
            a, b = (j, j + half) if neox else (2 * j, 2 * j + 1)
            c = table[positions, 2 * j]
            s = table[positions, 2 * j + 1]
            assert np.array_equal(qo[:, 0, a].view(np.uint32), c.view(np.uint32))
            assert np.array_equal(qo[:, 0, b].view(np.uint32), s.view(np.uint32))


def test_embedding_golden(oracle):
    g = golden("embedding")
    for qtype in (wl.F32, wl.Q8_0, wl.Q4_0, wl.Q4_1):
        qn = wl.QNAME[qtype]
        for cols in (96, 40, 38):
            key = f"{qn}_{cols}"
            out, bad = oracle.embedding(g[f"{key}_table"], qtype, 12, cols,
                                        g[f"{key}_tokens"])
            assert bad == 0
            assert_bitexact(out, g[f"{key}_out"], key)
        if qtype != wl.F32:
            out, bad = oracle.embedding(g[f"{qn}_bits_table"], qtype, 40, 64,
                                        g[f"{qn}_bits_tokens"])
            assert_bitexact(out, g[f"{qn}_bits_out"], f"{qn} random bits")


def test_quant_roundtrip_bounds(oracle, reference):
    """tests/test_quant.cc:18-56: Q8_0 round trip within 0.01, Q4 within 0.08,
    tail block (cols=40) within 0.02 — through the oracle's decode of the
    reference quantiser's blocks."""
    w = np.zeros((2, 32), np.float32)
    w[0] = 0.01 * np.arange(32) - 0.25
    w[1] = 0.01 * np.arange(32)
    for qtype, tol in ((wl.Q8_0, 0.01), (wl.Q4_0, 0.08), (wl.Q4_1, 0.08)):
        table = reference.quantize(w, qtype, wl.row_bytes(qtype, 32))
        out, bad = oracle.embedding(table, qtype, 2, 32, np.array([0, 1], np.int32))
        assert np.all(np.abs(out - w) <= tol + 1e-7)
    tail = np.sin(np.arange(40, dtype=np.float32))[None, :]
    table = reference.quantize(tail, wl.Q8_0, wl.row_bytes(wl.Q8_0, 40))
    out, _ = oracle.embedding(table, wl.Q8_0, 1, 40, np.array([0], np.int32))
    assert np.all(np.abs(out - tail) <= 0.02)
    # out-of-range row (test_quant.cc:63): reported, not written
    _, bad = oracle.embedding(table, wl.Q8_0, 1, 40, np.array([5, -1], np.int32))
    assert bad == 2


@pytest.mark.parametrize("seed", [1, 2])
def test_oracle_matches_reference_library(oracle, reference, seed):
    """Fresh seeded inputs through both the restatement and the reference
    compiled from source: identical bits."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((7, 1536), dtype=np.float32)
    r = rng.standard_normal((7, 1536), dtype=np.float32)
    w = rng.standard_normal(1536, dtype=np.float32) * 0.1 + 1
    y1, h1 = oracle.rmsnorm(x, w, 1e-6, residual=r)
    y2, h2 = reference.rmsnorm(x, w, 1e-6, residual=r)
    assert_bitexact(h1, h2, "h")
    assert_bitexact(y1, y2, "y")
    g = rng.standard_normal((5, 2000), dtype=np.float32) * 3
    u = rng.standard_normal((5, 2000), dtype=np.float32)
    assert_bitexact(oracle.swiglu(g, u), reference.swiglu(g, u), "swiglu")
    s = rng.standard_normal((9, 300), dtype=np.float32) * 2
    vl = rng.integers(1, 301, 9).astype(np.int32)
    assert_bitexact(oracle.softmax_rows(s, vl)[0], reference.softmax_rows(s, vl),
                    "softmax")
    for neox in (0, 1):
        q = rng.standard_normal((6, 4, 128), dtype=np.float32)
        k = rng.standard_normal((6, 2, 128), dtype=np.float32)
        bq = rng.standard_normal(4 * 128, dtype=np.float32) * 0.02
        bk = rng.standard_normal(2 * 128, dtype=np.float32) * 0.02
        pos = rng.integers(0, 70000, 6).astype(np.int32)
        qa, ka, _ = oracle.rope(q, k, pos, 1e6, neox, bq, bk)
        qb, kb = reference.rope(q, k, pos, 1e6, neox, bq, bk)
        assert_bitexact(qa, qb, "rope q")
        assert_bitexact(ka, kb, "rope k")
    for qtype in (wl.F32, wl.Q8_0, wl.Q4_0, wl.Q4_1):
        vocab, cols = 50, 224
        table = wl.numpy_quant_table(qtype, vocab, cols, seed)
        tokens = rng.integers(0, vocab, 33).astype(np.int32)
        a, bad = oracle.embedding(table, qtype, vocab, cols, tokens)
        b, rc = reference.embedding(table, qtype, vocab, cols, tokens)
        assert bad == 0 and rc == 0
        assert_bitexact(a, b, wl.QNAME[qtype])
        # linear layer over the same table (quant.cc:171-226 / F32 Linear)
        for k in (cols, 40):
            tab = wl.numpy_quant_table(qtype, 31, k, seed)
            x = rng.standard_normal((3, k), dtype=np.float32)
            assert_bitexact(oracle.linear(tab, qtype, 31, k, x),
                            reference.linear(tab, qtype, 31, k, x),
                            f"linear {wl.QNAME[qtype]} k={k}")
