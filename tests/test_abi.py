"""The C-ABI library without a GPU: it loads, exports exactly what
include/*.h declares, rejects bad arguments before touching the device, and
its host-side RoPE table is bit-identical to the oracle's."""
import ctypes
import glob
import os
import re

import numpy as np
import pytest

from conftest import ROOT, assert_bitexact

import mlb
import workloads as wl


def declared_symbols():
    names = set()
    for header in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(header).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names.update(re.findall(r"\b(mlb_\w+)\s*\(", text))
    return names


def test_library_exports_every_declared_symbol():
    lib = mlb.load()
    names = declared_symbols()
    assert "mlb_rmsnorm_f32" in names and len(names) >= 14
    for name in sorted(names):
        assert hasattr(lib, name), f"libmlb.so does not export {name}"


def test_python_binding_covers_header():
    assert declared_symbols() <= set(mlb.SIGNATURES)


def test_version_and_row_bytes():
    lib = mlb.load()
    assert lib.mlb_version() >= 100
    for qtype in (wl.F32, wl.Q8_0, wl.Q4_0, wl.Q4_1):
        for cols in (1, 31, 32, 33, 40, 896, 4096):
            assert mlb.row_bytes(qtype, cols) == wl.row_bytes(qtype, cols)
    assert mlb.row_bytes(7, 32) == -1
    assert mlb.row_bytes(wl.Q8_0, 896) == 952       # only 8-byte aligned rows


def test_bad_arguments_rejected_on_host():
    """Every entry validates its arguments before launching: null required
    pointers, non-positive widths, odd head_dim and unknown formats return
    MLB_ERR_ARG with a message (no device is touched here)."""
    lib = mlb.load()
    bogus = ctypes.c_void_p(16)
    cases = [
        lambda: lib.mlb_rmsnorm_f32(None, None, None, bogus, bogus, 1, 8, 1e-5, None),
        lambda: lib.mlb_rmsnorm_f32(bogus, None, None, bogus, bogus, 1, 0, 1e-5, None),
        lambda: lib.mlb_rmsnorm_f32(bogus, None, None, bogus, bogus, -1, 8, 1e-5, None),
        lambda: lib.mlb_swiglu_f32(None, bogus, bogus, 1, 8, None),
        lambda: lib.mlb_swiglu_f32(bogus, bogus, bogus, -2, 8, None),
        lambda: lib.mlb_silu_f32(None, bogus, 8, None),
        lambda: lib.mlb_mul_f32(bogus, None, bogus, 8, None),
        lambda: lib.mlb_add_f32(bogus, bogus, None, 8, None),
        lambda: lib.mlb_add_bias_f32(None, None, bogus, 1, 8, None),
        lambda: lib.mlb_rope_f32(bogus, bogus, None, None, bogus, 0, bogus, 4, 1,
                                 1, 1, 7, 0, None, None),
        lambda: lib.mlb_rope_f32(bogus, bogus, None, None, bogus, 0, None, 4, 1,
                                 1, 1, 8, 0, None, None),
        lambda: lib.mlb_softmax_rows_f32(bogus, None, 1, 8, None, None, None),
        lambda: lib.mlb_softmax_rows_f32(bogus, bogus, 1, 0, None, None, None),
        lambda: lib.mlb_embedding_gather(bogus, 9, 4, 32, bogus, 1, bogus, None, None),
        lambda: lib.mlb_embedding_gather(None, 1, 4, 32, bogus, 1, bogus, None, None),
        lambda: lib.mlb_embedding_gather(ctypes.c_void_p(17), 1, 4, 32, bogus, 1,
                                         bogus, None, None),
        lambda: lib.mlb_status_check(None, None, None),
        # linear layers: unknown format, negative sizes, missing scratch for
        # a prompt-sized batch
        lambda: lib.mlb_linear_f32(bogus, 9, 4, 32, bogus, 1, bogus, None),
        lambda: lib.mlb_linear_f32(bogus, 1, -4, 32, bogus, 1, bogus, None),
        lambda: lib.mlb_linear_rows_f32(bogus, 9, 4, 32, bogus, 64, bogus, bogus, 1 << 20,
                                        None),
        lambda: lib.mlb_linear_rows_f32(ctypes.c_void_p(64), 1, 128, 256,
                                        ctypes.c_void_p(64), 64, bogus, None, 0, None),
        # attention: group not dividing, null scratch, rows < 0
        lambda: lib.mlb_attention_decode_f32(bogus, bogus, bogus, bogus, 3, 8, 6, 4, 64,
                                             bogus, 1 << 20, None),
        lambda: lib.mlb_attention_rows_f32(bogus, bogus, bogus, bogus, 0, 4, 8, 8, 2, 64,
                                           None, 0, None),
        lambda: lib.mlb_attention_rows_f32(bogus, bogus, bogus, bogus, 0, -1, 8, 8, 2, 64,
                                           bogus, 1 << 20, None),
        lambda: lib.mlb_kv_write_f32(None, bogus, bogus, bogus, 0, 1, 8, 2, 64, None),
        lambda: lib.mlb_wait_timeouts(None),
    ]
    for i, call in enumerate(cases):
        assert call() == 1, f"case {i} not rejected"
        assert lib.mlb_last_error(), f"case {i} left no message"


def test_host_side_range_checks():
    """Per-token forms check the token id / position range on the host and
    return MLB_ERR_RANGE without launching (the reference throws
    std::out_of_range, cuda_ops.cu:265-267, and invalid_argument for a
    negative position, ops.cc:132-134)."""
    lib = mlb.load()
    bogus = ctypes.c_void_p(16)
    assert lib.mlb_embedding_row(bogus, 1, 10, 32, 10, bogus, None) == 3
    assert lib.mlb_embedding_row(bogus, 1, 10, 32, -1, bogus, None) == 3
    # consecutive positions [base, base + rows) must sit inside the table
    assert lib.mlb_rope_f32(bogus, bogus, None, None, None, -1, bogus, 8, 1, 1,
                            1, 8, 0, None, None) == 3
    assert lib.mlb_rope_f32(bogus, bogus, None, None, None, 5, bogus, 8, 4, 1,
                            1, 8, 0, None, None) == 3
    assert lib.mlb_last_error()


def test_empty_inputs_are_noops():
    """rows == 0 launches nothing and succeeds (the reference's size-0
    early returns, cuda_ops.cu:225, 235, 246, 303)."""
    lib = mlb.load()
    bogus = ctypes.c_void_p(16)
    assert lib.mlb_rmsnorm_f32(bogus, None, None, bogus, bogus, 0, 8, 1e-5, None) == 0
    assert lib.mlb_swiglu_f32(bogus, bogus, bogus, 0, 8, None) == 0
    assert lib.mlb_silu_f32(bogus, bogus, 0, None) == 0
    assert lib.mlb_softmax_rows_f32(bogus, bogus, 0, 8, None, None, None) == 0
    assert lib.mlb_embedding_gather(bogus, 1, 4, 32, bogus, 0, bogus, None, None) == 0
    assert lib.mlb_rope_f32(bogus, bogus, None, None, bogus, 0, bogus, 4, 0, 1,
                            1, 8, 1, None, None) == 0


@pytest.mark.parametrize("hd,theta,begin,end", [
    (64, 1e6, 0, 512), (128, 5e5, 0, 2048), (128, 1e4, 16000, 16400),
    (128, 1e6, 65400, 65536), (6, 1e4, 0, 300), (2, 1e4, 0, 4)])
def test_rope_table_host_bitexact(oracle, hd, theta, begin, end):
    mine = mlb.rope_table(theta, hd, end - begin, begin)
    want = oracle.rope_table(theta, hd, begin, end)
    assert_bitexact(mine, want, f"hd={hd} theta={theta}")


def test_rope_table_rejects_bad_args():
    with pytest.raises(ValueError):
        mlb.rope_table(1e4, 7, 4)
    with pytest.raises(ValueError):
        mlb.rope_table(-1.0, 8, 4)


def test_shard_ranges_cover_rows_contiguously():
    for total in (0, 1, 7, 64, 16384, 65537):
        for world in (1, 2, 3, 4, 8):
            prev = 0
            sizes = []
            for rank in range(world):
                b, e = wl.shard_range(total, world, rank)
                assert b == prev and e >= b
                prev = e
                sizes.append(e - b)
            assert prev == total
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        wl.shard_range(10, 2, 2)


def test_algorithmic_bytes_match_formulas():
    c3 = wl.CONFIGS["llama3-8b-t16384"]
    assert c3.bytes_rmsnorm() == 16 * 16384 * 4096 + 4 * 4096
    assert c3.bytes_swiglu() == 12 * 16384 * 14336
    assert c3.bytes_rope() == 8 * 16384 * 40 * 128 + 4 * 16384
    assert c3.bytes_embedding() == 16384 * (128 * 34 + 4 * 4096 + 4)
    c1 = wl.CONFIGS["qwen2-0.5b-t256"]
    assert c1.bytes_softmax() == 4 * 14 * 256 * 257 // 2 + 4 * 14 * 256 * 256


def test_gemv_path_switch():
    """The decode-linear kernel choice (no GPU work): 0 / 1 / 2 are taken and
    read back, anything else is refused and leaves the setting alone."""
    lib = mlb.load()
    previous = lib.mlb_gemv_path()
    try:
        for path in (1, 2, 0):
            assert lib.mlb_set_gemv_path(path) == 0
            assert lib.mlb_gemv_path() == path
        for bad in (-1, 3):
            assert lib.mlb_set_gemv_path(bad) == 1  # MLB_ERR_ARG
            assert lib.mlb_gemv_path() == 0
        assert mlb.set_gemv_path(2) == 0 and mlb.set_gemv_path(0) == 2
    finally:
        lib.mlb_set_gemv_path(previous)


def test_launch_overlap_switch():
    """Programmatic dependent launch on / off (no GPU work): on by default,
    0 / 1 taken and read back, anything else refused and the setting kept."""
    lib = mlb.load()
    previous = lib.mlb_launch_overlap()
    try:
        assert previous == 1
        for on in (0, 1):
            assert lib.mlb_set_launch_overlap(on) == 0
            assert lib.mlb_launch_overlap() == on
        for bad in (-1, 2):
            assert lib.mlb_set_launch_overlap(bad) == 1  # MLB_ERR_ARG
            assert lib.mlb_launch_overlap() == 1
        assert mlb.set_launch_overlap(0) == 1 and mlb.set_launch_overlap(1) == 0
    finally:
        lib.mlb_set_launch_overlap(previous)
