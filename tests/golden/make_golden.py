"""Generates the golden fixtures in this directory from the reference itself.

Every expected output here is produced by mini-lla's own CPU operators
(src/ops.cc, src/quant.cc), compiled from the reference sources into
oracle/_ref/libmlref.so by `make -C oracle ref`.  Inputs are seeded and small
enough to commit.  Run from the repository root:

    make -C oracle all ref && python tests/golden/make_golden.py

The fixtures pin the CPU oracle (tests/test_oracle.py) and the CUDA kernels
(tests/test_gpu_parity.py) without needing the reference at test time.
"""
from __future__ import annotations

import os
import sys

import numpy as np

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), "..", ".."))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "mini-lla_b200"))

from oracle import Reference  # noqa: E402
import workloads as wl  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))


def rmsnorm_cases(ref, rng):
    cases = {}
    # tests/test_ops.cc:41-43: RmsNorm([1,2,3], w=1, eps 1e-5)[0] ~ 0.46291
    x = np.array([[1, 2, 3]], np.float32)
    cases["kat_x"] = x
    cases["kat_w"] = np.ones(3, np.float32)
    cases["kat_y"] = ref.rmsnorm(x, cases["kat_w"], 1e-5)
    for name, rows, cols, eps in (("warp", 6, 896, 1e-6), ("block", 3, 4096, 1e-5),
                                  ("block_odd", 2, 3584, 1e-6),
                                  ("scalar", 5, 37, 1e-5), ("tiny", 3, 4, 1e-6)):
        x = rng.standard_normal((rows, cols), dtype=np.float32)
        r = rng.standard_normal((rows, cols), dtype=np.float32)
        w = (rng.standard_normal(cols, dtype=np.float32) * 0.1 + 1).astype(np.float32)
        y, h = ref.rmsnorm(x, w, eps, residual=r)
        cases[f"{name}_x"], cases[f"{name}_r"], cases[f"{name}_w"] = x, r, w
        cases[f"{name}_eps"] = np.float32(eps)
        cases[f"{name}_h"], cases[f"{name}_y"] = h, y
        cases[f"{name}_y_plain"] = ref.rmsnorm(x, w, eps)
    return cases


def swiglu_cases(ref, rng):
    cases = {}
    # tests/test_ops.cc:48-56
    cases["kat_g"] = np.array([[0.0, 1.0]], np.float32)
    cases["kat_u"] = np.array([[2.0, 2.0]], np.float32)
    cases["kat_o"] = ref.swiglu(cases["kat_g"], cases["kat_u"])
    for name, rows, cols in (("vec", 4, 1024), ("scalar", 3, 999)):
        g = rng.standard_normal((rows, cols), dtype=np.float32) * 4
        u = rng.standard_normal((rows, cols), dtype=np.float32)
        cases[f"{name}_g"], cases[f"{name}_u"] = g, u
        cases[f"{name}_o"] = ref.swiglu(g, u)
        cases[f"{name}_silu"] = ref.silu(g)
    # extremes: large |g| where exp under/overflows
    g = np.array([[-100.0, -88.0, -30.0, -1e-30, 0.0, 1e-30, 30.0, 88.0, 100.0,
                   -5.5, 5.5, 1.0]], np.float32)
    cases["edge_g"], cases["edge_u"] = g, np.ones_like(g)
    cases["edge_o"] = ref.swiglu(g, np.ones_like(g))
    return cases


def softmax_cases(ref, rng):
    cases = {}
    cases["kat_x"] = np.array([[1, 2, 3]], np.float32)   # test_ops.cc:45-47
    cases["kat_y"] = ref.softmax_rows(cases["kat_x"])
    for name, rows, cols in (("warp", 64, 64), ("block", 4, 1040),
                             ("scalar", 5, 37)):
        x = rng.standard_normal((rows, cols), dtype=np.float32) * 2
        vl = (np.arange(rows) % cols + 1).astype(np.int32)
        vl[-1] = cols
        cases[f"{name}_x"], cases[f"{name}_len"] = x, vl
        cases[f"{name}_y"] = ref.softmax_rows(x, vl)
    return cases


def rope_cases(ref, rng):
    cases = {}
    # tests/test_ops.cc:65-82: pos 1, hd 2, theta 1e4 rotates by 1 rad.
    q = np.array([[[1.0, 0.0]]], np.float32)
    for neox in (0, 1):
        qo, ko = ref.rope(q, q.copy(), np.array([1], np.int32), 1e4, neox)
        cases[f"kat{neox}_q"], cases[f"kat{neox}_k"] = qo, ko
    cases["kat_in"] = q
    specs = (("neox_bias", 6, 14, 2, 64, 1e6, 1, True,
              [0, 1, 255, 2047, 16383, 65535]),
             ("normal", 5, 8, 2, 128, 5e5, 0, False, [0, 7, 2047, 16383, 100000]),
             ("normal_small", 4, 3, 1, 6, 1e4, 0, True, [0, 3, 11, 4095]),
             ("neox_small", 4, 2, 2, 12, 1e4, 1, False, [1, 2, 30, 999]))
    for name, t, nq, nk, hd, theta, neox, bias, pos in specs:
        q = rng.standard_normal((t, nq, hd), dtype=np.float32)
        k = rng.standard_normal((t, nk, hd), dtype=np.float32)
        bq = (rng.standard_normal(nq * hd, dtype=np.float32) * 0.02) if bias else None
        bk = (rng.standard_normal(nk * hd, dtype=np.float32) * 0.02) if bias else None
        pos = np.array(pos[:t] + [0] * (t - len(pos[:t])), np.int32)
        qo, ko = ref.rope(q, k, pos, theta, neox, bq, bk)
        cases.update({f"{name}_q": q, f"{name}_k": k, f"{name}_pos": pos,
                      f"{name}_theta": np.float32(theta),
                      f"{name}_neox": np.int32(neox), f"{name}_qo": qo,
                      f"{name}_ko": ko})
        if bias:
            cases[f"{name}_bq"], cases[f"{name}_bk"] = bq, bk
    return cases


def embedding_cases(ref, rng):
    cases = {}
    for qtype in (wl.F32, wl.Q8_0, wl.Q4_0, wl.Q4_1):
        qn = wl.QNAME[qtype]
        for cols in (96, 40, 38):
            vocab = 12
            values = rng.standard_normal((vocab, cols), dtype=np.float32)
            values[1] = 0.0                       # all-zero block path
            values[2] = np.abs(values[2]) + 0.5   # one-signed row
            rb = wl.row_bytes(qtype, cols)
            table = ref.quantize(values, qtype, rb)
            tokens = np.array([0, 11, 5, 1, 2, 7, 7, 3], np.int32)
            out, rc = ref.embedding(table, qtype, vocab, cols, tokens)
            assert rc == 0
            key = f"{qn}_{cols}"
            cases[f"{key}_table"], cases[f"{key}_tokens"] = table, tokens
            cases[f"{key}_out"] = out
        if qtype != wl.F32:
            # random block bits: scales cover subnormal, inf and NaN patterns
            cols, vocab = 64, 40
            rb = wl.row_bytes(qtype, cols)
            table = rng.integers(0, 256, size=vocab * rb, dtype=np.uint8)
            tokens = np.arange(vocab, dtype=np.int32)[::-1].copy()
            out, rc = ref.embedding(table, qtype, vocab, cols, tokens)
            assert rc == 0
            cases[f"{qn}_bits_table"], cases[f"{qn}_bits_tokens"] = table, tokens
            cases[f"{qn}_bits_out"] = out
    return cases


def fp16_case(ref):
    """All 65536 fp16 scale patterns through the reference's Q8_0 decode:
    row i has d = i and qs[0] = 1, so out[i, 0] == Fp16ToFloat(i)."""
    vocab, cols = 65536, 32
    blocks = np.zeros((vocab, 34), np.uint8)
    blocks[:, 0:2] = np.arange(vocab, dtype=np.uint16).view(np.uint8).reshape(vocab, 2)
    blocks[:, 2] = 1
    tokens = np.arange(vocab, dtype=np.int32)
    out, rc = ref.embedding(blocks.reshape(-1), wl.Q8_0, vocab, cols, tokens)
    assert rc == 0
    return {"bits": out[:, 0].view(np.uint32).copy()}


def main():
    ref = Reference()
    rng = np.random.default_rng(20261201)
    for name, fn in (("rmsnorm", rmsnorm_cases), ("swiglu", swiglu_cases),
                     ("softmax", softmax_cases), ("rope", rope_cases),
                     ("embedding", embedding_cases)):
        cases = fn(ref, rng)
        np.savez_compressed(os.path.join(OUT, f"{name}.npz"), **cases)
        print(name, len(cases), "arrays")
    np.savez_compressed(os.path.join(OUT, "fp16.npz"), **fp16_case(ref))
    print("fp16 65536 patterns")


if __name__ == "__main__":
    main()
