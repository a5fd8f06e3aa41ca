"""numpy binding of the CPU checkers — TEST INFRASTRUCTURE ONLY.

`Oracle` wraps liboracle.so (mlb_oracle.c, the plain-C restatement of the
reference arithmetic).  `Reference` wraps _ref/libmlref.so (the reference's
own ops.cc / quant.cc compiled from source plus ref_shim.cc) and is present
only where that library was built.  Only tests, the smoke check and the CPU
baseline of bench.py use this module; the product library never does.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from ctypes import c_float, c_int, c_int64, c_void_p, c_double

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libmlref.so")


def _p(a):
    return None if a is None else a.ctypes.data_as(c_void_p)


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def build_oracle():
    """Compiles liboracle.so (and _ref/libmlref.so when the reference
    sources are reachable)."""
    subprocess.run(["make", "-s", "-C", HERE, "all"], check=True)
    # the reference checkout: MLB_REFERENCE_DIR, else `reference` beside
    # this repository
    ref_dir = os.environ.get("MLB_REFERENCE_DIR") or os.path.join(
        os.path.dirname(os.path.dirname(HERE)), "reference")
    if os.path.isdir(os.path.join(ref_dir, "src")):
        subprocess.run(["make", "-s", "-C", HERE, "ref",
                        f"MLB_REFERENCE_DIR={ref_dir}"], check=True)


class Oracle:
    """The plain-C restatement (mlb_oracle.c)."""

    def __init__(self, path: str = ORACLE_SO):
        if not os.path.exists(path):
            build_oracle()
        lib = ctypes.CDLL(path)
        sig = {
            "mlbo_fp16_to_f32": (c_float, [ctypes.c_uint16]),
            "mlbo_row_bytes": (c_int64, [c_int, c_int64]),
            "mlbo_embedding_rows": (c_int64, [c_void_p, c_int, c_int64, c_int64,
                                              c_void_p, c_int64, c_void_p]),
            "mlbo_add": (None, [c_void_p, c_void_p, c_void_p, c_int64]),
            "mlbo_rmsnorm_rows": (None, [c_void_p, c_void_p, c_void_p, c_void_p,
                                         c_void_p, c_int64, c_int64, c_float]),
            "mlbo_swiglu": (None, [c_void_p, c_void_p, c_void_p, c_int64]),
            "mlbo_silu": (None, [c_void_p, c_void_p, c_int64]),
            "mlbo_softmax_rows": (c_int64, [c_void_p, c_void_p, c_int64, c_int64,
                                            c_void_p]),
            "mlbo_rope_table": (None, [c_float, c_int, c_int64, c_int64, c_void_p]),
            "mlbo_linear_rows": (None, [c_void_p, c_int, c_int64, c_int64, c_void_p,
                                        c_int64, c_void_p]),
            "mlbo_attention_decode": (None, [c_void_p, c_void_p, c_void_p, c_void_p,
                                             c_int64, c_int, c_int, c_int,
                                             c_void_p]),
            "mlbo_rope_rows": (c_int64, [c_void_p, c_void_p, c_void_p, c_void_p,
                                         c_void_p, c_int64, c_int, c_int, c_int,
                                         c_float, c_int]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        self.lib = lib

    def fp16_to_f32(self, bits: int) -> float:
        return self.lib.mlbo_fp16_to_f32(bits)

    def row_bytes(self, qtype, cols):
        return self.lib.mlbo_row_bytes(qtype, cols)

    def embedding(self, table: np.ndarray, qtype: int, vocab: int, cols: int,
                  tokens: np.ndarray):
        tokens = np.ascontiguousarray(tokens, dtype=np.int32)
        table = np.ascontiguousarray(table)
        out = np.zeros((tokens.size, cols), dtype=np.float32)
        bad = self.lib.mlbo_embedding_rows(_p(table), qtype, vocab, cols,
                                           _p(tokens), tokens.size, _p(out))
        return out, bad

    def rmsnorm(self, x, w, eps, residual=None):
        x = _f32(x)
        cols = x.shape[-1]
        rows = x.size // cols
        y = np.empty_like(x)
        h = np.empty_like(x) if residual is not None else None
        r = _f32(residual) if residual is not None else None
        self.lib.mlbo_rmsnorm_rows(_p(x), _p(r), _p(h), _p(y), _p(_f32(w)),
                                   rows, cols, eps)
        return (y, h) if residual is not None else y

    def add(self, a, b):
        a, b = _f32(a), _f32(b)
        out = np.empty_like(a)
        self.lib.mlbo_add(_p(a), _p(b), _p(out), a.size)
        return out

    def swiglu(self, g, u):
        g, u = _f32(g), _f32(u)
        out = np.empty_like(g)
        self.lib.mlbo_swiglu(_p(g), _p(u), _p(out), g.size)
        return out

    def silu(self, x):
        x = _f32(x)
        out = np.empty_like(x)
        self.lib.mlbo_silu(_p(x), _p(out), x.size)
        return out

    def softmax_rows(self, x, valid_len=None):
        x = _f32(x)
        cols = x.shape[-1]
        rows = x.size // cols
        y = np.empty_like(x)
        vl = None if valid_len is None else np.ascontiguousarray(valid_len, np.int32)
        bad = self.lib.mlbo_softmax_rows(_p(x), _p(y), rows, cols, _p(vl))
        return y, bad

    def linear(self, table, qtype, n, k, x):
        """y = x · dequant(W)^T with the reference's sequential sums."""
        x = _f32(x)
        t_rows = x.size // k
        y = np.empty((t_rows, n), dtype=np.float32)
        self.lib.mlbo_linear_rows(_p(np.ascontiguousarray(table)), qtype, n, k,
                                  _p(x), t_rows, _p(y))
        return y

    def attention_decode(self, q, keys, values, position, n_heads, n_kv_heads):
        """q [n_heads, hd]; keys/values [>= position+1, n_kv_heads, hd]."""
        q = _f32(q)
        hd = q.size // n_heads
        keys, values = _f32(keys), _f32(values)
        out = np.empty((n_heads, hd), np.float32)
        scores = np.empty(position + 1, np.float32)
        self.lib.mlbo_attention_decode(_p(q), _p(keys), _p(values), _p(out),
                                       position, n_heads, n_kv_heads, hd,
                                       _p(scores))
        return out

    def rope_table(self, theta, hd, pos_begin, pos_end):
        out = np.empty((pos_end - pos_begin, hd), dtype=np.float32)
        self.lib.mlbo_rope_table(theta, hd, pos_begin, pos_end, _p(out))
        return out

    def rope(self, q, k, positions, theta, neox, bq=None, bk=None):
        """Returns rotated copies of q [T, nq, hd] and k [T, nk, hd]."""
        q = _f32(q).copy()
        k = _f32(k).copy()
        rows, nq, hd = q.shape
        nk = k.shape[1]
        pos = np.ascontiguousarray(positions, dtype=np.int32)
        bad = self.lib.mlbo_rope_rows(_p(q), _p(k), _p(_f32(bq) if bq is not None else None),
                                      _p(_f32(bk) if bk is not None else None),
                                      _p(pos), rows, nq, nk, hd, theta,
                                      1 if neox else 0)
        return q, k, bad


class Reference:
    """The reference's own CPU operators (oracle/_ref/libmlref.so)."""

    def __init__(self, path: str = REF_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        lib = ctypes.CDLL(path)
        V = c_void_p
        sig = {
            "mlref_thread_count": (c_int, []),
            "mlref_set_thread_count": (None, [c_int]),
            "mlref_rmsnorm_rows": (c_int, [V, V, V, V, V, c_int64, c_int64, c_float]),
            "mlref_swiglu_rows": (c_int, [V, V, V, c_int64, c_int64]),
            "mlref_silu": (c_int, [V, V, c_int64]),
            "mlref_softmax_rows": (c_int, [V, V, c_int64, c_int64, V]),
            "mlref_rope_rows": (c_int, [V, V, V, V, V, c_int64, c_int, c_int,
                                        c_int, c_float, c_int]),
            "mlref_embedding_rows": (c_int, [V, c_int, c_int64, c_int64, V,
                                             c_int64, V]),
            "mlref_quantize": (c_int, [V, c_int64, c_int64, c_int, V]),
            "mlref_linear": (c_int, [V, c_int, c_int64, c_int64, V, c_int64, V]),
            "mlref_attention_decode": (c_int, [V, V, V, V, c_int64, c_int, c_int,
                                               c_int]),
            "mlref_rows_new": (V, [V, c_int64, c_int64]),
            "mlref_heads_new": (V, [V, c_int64, c_int, c_int]),
            "mlref_rows_free": (None, [V]),
            "mlref_table_new": (V, [V, c_int, c_int64, c_int64]),
            "mlref_table_free": (None, [V]),
            "mlref_bench_rmsnorm": (c_double, [V, V, V, c_float]),
            "mlref_bench_swiglu": (c_double, [V, V]),
            "mlref_bench_rope": (c_double, [V, V, V, V, V, c_float, c_int]),
            "mlref_bench_softmax": (c_double, [V, V]),
            "mlref_bench_embedding": (c_double, [V, V, c_int64, V]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        self.lib = lib

    def rmsnorm(self, x, w, eps, residual=None):
        x = _f32(x)
        cols = x.shape[-1]
        rows = x.size // cols
        y = np.empty_like(x)
        h = np.empty_like(x) if residual is not None else None
        r = _f32(residual) if residual is not None else None
        rc = self.lib.mlref_rmsnorm_rows(_p(x), _p(r), _p(h), _p(y), _p(_f32(w)),
                                         rows, cols, eps)
        assert rc == 0, rc
        return (y, h) if residual is not None else y

    def swiglu(self, g, u):
        g, u = _f32(g), _f32(u)
        cols = g.shape[-1]
        out = np.empty_like(g)
        assert self.lib.mlref_swiglu_rows(_p(g), _p(u), _p(out), g.size // cols,
                                          cols) == 0
        return out

    def silu(self, x):
        x = _f32(x)
        out = np.empty_like(x)
        assert self.lib.mlref_silu(_p(x), _p(out), x.size) == 0
        return out

    def softmax_rows(self, x, valid_len=None):
        x = _f32(x)
        cols = x.shape[-1]
        y = np.empty_like(x)
        vl = None if valid_len is None else np.ascontiguousarray(valid_len, np.int32)
        rc = self.lib.mlref_softmax_rows(_p(x), _p(y), x.size // cols, cols, _p(vl))
        assert rc == 0, rc
        return y

    def rope(self, q, k, positions, theta, neox, bq=None, bk=None):
        q = _f32(q).copy()
        k = _f32(k).copy()
        rows, nq, hd = q.shape
        pos = np.ascontiguousarray(positions, dtype=np.int32)
        rc = self.lib.mlref_rope_rows(_p(q), _p(k),
                                      _p(_f32(bq) if bq is not None else None),
                                      _p(_f32(bk) if bk is not None else None),
                                      _p(pos), rows, nq, k.shape[1], hd, theta,
                                      1 if neox else 0)
        assert rc == 0, rc
        return q, k

    def embedding(self, table, qtype, vocab, cols, tokens):
        tokens = np.ascontiguousarray(tokens, dtype=np.int32)
        table = np.ascontiguousarray(table)
        out = np.zeros((tokens.size, cols), dtype=np.float32)
        rc = self.lib.mlref_embedding_rows(_p(table), qtype, vocab, cols,
                                           _p(tokens), tokens.size, _p(out))
        return out, rc

    def linear(self, table, qtype, n, k, x):
        x = _f32(x)
        t_rows = x.size // k
        y = np.empty((t_rows, n), dtype=np.float32)
        rc = self.lib.mlref_linear(_p(np.ascontiguousarray(table)), qtype, n, k,
                                   _p(x), t_rows, _p(y))
        assert rc == 0, rc
        return y

    def attention_decode(self, q, keys, values, position, n_heads, n_kv_heads):
        q = _f32(q)
        hd = q.size // n_heads
        out = np.empty((n_heads, hd), np.float32)
        rc = self.lib.mlref_attention_decode(_p(q), _p(_f32(keys)), _p(_f32(values)),
                                             _p(out), position, n_heads,
                                             n_kv_heads, hd)
        assert rc == 0, rc
        return out

    def quantize(self, values, qtype, row_bytes):
        values = _f32(values)
        rows, cols = values.shape
        out = np.zeros(rows * row_bytes, dtype=np.uint8)
        assert self.lib.mlref_quantize(_p(values), rows, cols, qtype, _p(out)) == 0
        return out


def fp16_bits_to_f32_numpy(bits: np.ndarray) -> np.ndarray:
    """Independent decode through numpy's IEEE half type (for pinning)."""
    return np.asarray(bits, dtype=np.uint16).view(np.float16).astype(np.float32)
