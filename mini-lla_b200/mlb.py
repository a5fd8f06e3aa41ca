"""ctypes binding of libmlb.so (include/mlb_ops.h) for Python callers.

Tensors are torch CUDA tensors (torch supplies device memory and streams);
every call goes straight to the C ABI and from there to the sm_100a kernels.
There is no CPU fallback: loading fails loudly when libmlb.so is missing.

Error behaviour follows the reference's C++ operator layer
(src/cuda_ops.cu): a shape mismatch raises ValueError (std::invalid_argument
there), an out-of-range token or position reported by the device raises
IndexError (std::out_of_range), a CUDA failure raises RuntimeError
(std::runtime_error from CudaCheckLastError).
"""
from __future__ import annotations

import ctypes
import os
from ctypes import c_float, c_int, c_int64, c_void_p

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libmlb.so")

F32, Q8_0, Q4_0, Q4_1 = 0, 1, 2, 3
QTYPE_NAMES = {"F32": F32, "Q8_0": Q8_0, "Q4_0": Q4_0, "Q4_1": Q4_1}
STATUS_BAD_TOKEN, STATUS_BAD_POSITION, STATUS_BAD_LENGTH = 1, 2, 4

# Every symbol include/mlb_ops.h declares, with (restype, argtypes).
SIGNATURES = {
    "mlb_version": (c_int, []),
    "mlb_last_error": (ctypes.c_char_p, []),
    "mlb_row_bytes": (c_int64, [c_int, c_int64]),
    "mlb_rmsnorm_f32": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p,
                                c_void_p, c_int64, c_int64, c_float, c_void_p]),
    "mlb_swiglu_f32": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64,
                               c_void_p]),
    "mlb_silu_f32": (c_int, [c_void_p, c_void_p, c_int64, c_void_p]),
    "mlb_mul_f32": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_void_p]),
    "mlb_add_f32": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_void_p]),
    "mlb_add_bias_f32": (c_int, [c_void_p, c_void_p, c_void_p, c_int64,
                                 c_int64, c_void_p]),
    "mlb_rope_table_build_host": (c_int, [c_float, c_int, c_int64, c_int64,
                                          c_void_p]),
    "mlb_rope_f32": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                             c_int64, c_void_p, c_int64, c_int64, c_int, c_int,
                             c_int, c_int, c_void_p, c_void_p]),
    "mlb_embedding_row": (c_int, [c_void_p, c_int, c_int64, c_int64, ctypes.c_int32,
                                  c_void_p, c_void_p]),
    "mlb_softmax_rows_f32": (c_int, [c_void_p, c_void_p, c_int64, c_int64,
                                     c_void_p, c_void_p, c_void_p]),
    "mlb_embedding_gather": (c_int, [c_void_p, c_int, c_int64, c_int64,
                                     c_void_p, c_int64, c_void_p, c_void_p,
                                     c_void_p]),
    "mlb_status_check": (c_int, [c_void_p, c_void_p, c_void_p]),
    "mlb_wait_timeouts": (c_int, [c_void_p]),
    "mlb_set_gemv_path": (c_int, [c_int]),
    "mlb_set_attention_path": (c_int, [c_int]),
    "mlb_attention_path": (c_int, []),
    "mlb_gemv_path": (c_int, []),
    "mlb_set_launch_overlap": (c_int, [c_int]),
    "mlb_launch_overlap": (c_int, []),
    "mlb_linear_rows_scratch_floats": (c_int64, [c_int64, c_int64]),
    "mlb_linear_rows_f32": (c_int, [c_void_p, c_int, c_int64, c_int64, c_void_p,
                                    c_int64, c_void_p, c_void_p, c_int64, c_void_p]),
    "mlb_linear_rows_group_f32": (c_int, [c_int, c_void_p, c_int, c_void_p, c_int64,
                                          c_void_p, c_int64, c_void_p, c_void_p, c_int64,
                                          c_void_p]),
    "mlb_attention_rows_scratch_floats": (c_int64, [c_int, c_int, c_int, c_int64,
                                                    c_int64]),
    "mlb_attention_rows_f32": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p,
                                       c_int64, c_int64, c_int64, c_int, c_int,
                                       c_int, c_void_p, c_int64, c_void_p]),
    "mlb_linear_f32": (c_int, [c_void_p, c_int, c_int64, c_int64, c_void_p,
                               c_int64, c_void_p, c_void_p]),
    "mlb_kv_write_f32": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64,
                                 c_int64, c_int64, c_int, c_int, c_void_p]),
    "mlb_attention_scratch_floats": (c_int64, [c_int, c_int, c_int, c_int64]),
    "mlb_attention_decode_f32": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p,
                                         c_int64, c_int64, c_int, c_int, c_int,
                                         c_void_p, c_int64, c_void_p]),
    "mlb_attention_decode_noalloc_f32": (c_int, [c_void_p, c_void_p, c_void_p,
                                                 c_void_p, c_int64, c_int64, c_int,
                                                 c_int, c_int, c_void_p]),
}

_lib = None


def load(path: str = LIB_PATH) -> ctypes.CDLL:
    """Loads libmlb.so once and binds every declared symbol."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise RuntimeError(
            f"libmlb.so not found at {path}: build it with "
            "`make -C mini-lla_b200` (there is no CPU fallback)")
    lib = ctypes.CDLL(path)
    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    _lib = lib
    return lib


def _ptr(t):
    return None if t is None else c_void_p(t.data_ptr())


def _stream(stream):
    import torch
    if stream is None:
        stream = torch.cuda.current_stream()
    return c_void_p(stream.cuda_stream)


def _check(rc: int, op: str):
    if rc == 0:
        return
    msg = load().mlb_last_error().decode()
    if rc == 1:
        raise ValueError(f"{op}: {msg}")
    if rc == 3:
        raise IndexError(f"{op}: {msg}")
    raise RuntimeError(f"{op}: {msg}")


def _require(cond: bool, op: str, what: str):
    if not cond:
        raise ValueError(f"{op}: {what}")


def _f32_cuda(t, op, name):
    import torch
    _require(t.is_cuda and t.dtype == torch.float32 and t.is_contiguous(), op,
             f"{name} must be a contiguous float32 CUDA tensor")


def row_bytes(qtype: int, cols: int) -> int:
    return int(load().mlb_row_bytes(qtype, cols))


def rms_norm(x, weight, eps: float, residual=None, h_out=None, out=None,
             stream=None):
    """y = RmsNorm(x [+ residual]) row-wise over the last dim; returns y.

    With `residual`, the sum h = x + residual is also written to `h_out`
    when given (the new residual stream)."""
    op = "rms_norm"
    _f32_cuda(x, op, "x")
    _f32_cuda(weight, op, "weight")
    cols = x.shape[-1]
    _require(weight.numel() == cols, op, "weight size mismatch")
    if residual is not None:
        _f32_cuda(residual, op, "residual")
        _require(residual.shape == x.shape, op, "residual shape mismatch")
    if h_out is not None:
        _f32_cuda(h_out, op, "h_out")
        _require(h_out.shape == x.shape, op, "h_out shape mismatch")
    if out is None:
        import torch
        out = torch.empty_like(x)
    rows = x.numel() // cols if cols else 0
    _check(load().mlb_rmsnorm_f32(_ptr(x), _ptr(residual), _ptr(h_out),
                                  _ptr(out), _ptr(weight), rows, cols,
                                  float(eps), _stream(stream)), op)
    return out


def swiglu(gate, up, out=None, stream=None):
    op = "swiglu"
    _f32_cuda(gate, op, "gate")
    _f32_cuda(up, op, "up")
    _require(gate.shape == up.shape, op, "shape mismatch")
    if out is None:
        import torch
        out = torch.empty_like(gate)
    cols = gate.shape[-1] if gate.dim() else 1
    rows = gate.numel() // cols if cols else 0
    _check(load().mlb_swiglu_f32(_ptr(gate), _ptr(up), _ptr(out), rows, cols,
                                 _stream(stream)), op)
    return out


def silu(x, out=None, stream=None):
    _f32_cuda(x, "silu", "x")
    if out is None:
        import torch
        out = torch.empty_like(x)
    _check(load().mlb_silu_f32(_ptr(x), _ptr(out), x.numel(), _stream(stream)),
           "silu")
    return out


def mul(a, b, out=None, stream=None):
    _f32_cuda(a, "mul", "a")
    _f32_cuda(b, "mul", "b")
    _require(a.numel() == b.numel(), "mul", "size mismatch")
    if out is None:
        import torch
        out = torch.empty_like(a)
    _check(load().mlb_mul_f32(_ptr(a), _ptr(b), _ptr(out), a.numel(),
                              _stream(stream)), "mul")
    return out


def add(a, b, out=None, stream=None):
    _f32_cuda(a, "add", "a")
    _f32_cuda(b, "add", "b")
    _require(a.numel() == b.numel(), "add", "size mismatch")
    if out is None:
        import torch
        out = torch.empty_like(a)
    _check(load().mlb_add_f32(_ptr(a), _ptr(b), _ptr(out), a.numel(),
                              _stream(stream)), "add")
    return out


def add_bias(value, bias=None, out=None, stream=None):
    _f32_cuda(value, "add_bias", "value")
    cols = value.shape[-1]
    if bias is not None:
        _f32_cuda(bias, "add_bias", "bias")
        _require(bias.numel() == cols, "add_bias", "bias shape mismatch")
    if out is None:
        import torch
        out = torch.empty_like(value)
    rows = value.numel() // cols if cols else 0
    _check(load().mlb_add_bias_f32(_ptr(value), _ptr(bias), _ptr(out), rows,
                                   cols, _stream(stream)), "add_bias")
    return out


def rope_table(theta: float, head_dim: int, positions: int, pos_begin: int = 0):
    """Host-built (cos, sin) table as a numpy float32 array [P, head_dim]."""
    import numpy as np
    table = np.empty((positions, head_dim), dtype=np.float32)
    rc = load().mlb_rope_table_build_host(
        float(theta), int(head_dim), int(pos_begin), int(pos_begin + positions),
        table.ctypes.data_as(c_void_p))
    if rc != 0:
        raise ValueError("rope_table: invalid theta, head_dim or range")
    return table


def rope(q, k, positions, table, neox: bool, bq=None, bk=None, status=None,
         stream=None, position_base: int = 0):
    """In-place bias add + RoPE on q [T, nq, hd] and k [T, nk, hd].

    `positions` is an int32 [T] CUDA tensor, or None for consecutive
    positions position_base + t."""
    import torch
    op = "rope"
    _f32_cuda(q, op, "q")
    _require(q.dim() == 3, op, "q must be [tokens, heads, head_dim]")
    rows, nq, hd = q.shape
    nk = 0
    if k is not None:
        _f32_cuda(k, op, "k")
        _require(k.dim() == 3 and k.shape[0] == rows and k.shape[2] == hd, op,
                 "k must be [tokens, kv_heads, head_dim]")
        nk = k.shape[1]
    _require(hd % 2 == 0, op, "expected [heads, even_dim]")
    if positions is not None:
        _require(positions.is_cuda and positions.dtype == torch.int32 and
                 positions.numel() == rows, op, "positions must be int32 [tokens]")
    _f32_cuda(table, op, "table")
    _require(table.dim() == 2 and table.shape[1] == hd, op,
             "table must be [positions, head_dim]")
    for b, n, name in ((bq, nq, "bq"), (bk, nk, "bk")):
        if b is not None:
            _f32_cuda(b, op, name)
            _require(b.numel() == n * hd, op, f"{name} shape mismatch")
    _check(load().mlb_rope_f32(_ptr(q), _ptr(k), _ptr(bq), _ptr(bk),
                               _ptr(positions), int(position_base), _ptr(table),
                               table.shape[0], rows, nq, nk, hd,
                               1 if neox else 0, _ptr(status), _stream(stream)),
           op)


def softmax_rows(x, valid_len=None, out=None, status=None, stream=None):
    import torch
    op = "softmax_rows"
    _f32_cuda(x, op, "x")
    cols = x.shape[-1]
    _require(x.numel() > 0 and cols > 0, op, "expected a non-empty vector")
    rows = x.numel() // cols
    if valid_len is not None:
        _require(valid_len.is_cuda and valid_len.dtype == torch.int32 and
                 valid_len.numel() == rows, op, "valid_len must be int32 [rows]")
    if out is None:
        out = torch.empty_like(x)
    _check(load().mlb_softmax_rows_f32(_ptr(x), _ptr(out), rows, cols,
                                       _ptr(valid_len), _ptr(status),
                                       _stream(stream)), op)
    return out


def embedding_rows(table, qtype: int, vocab: int, cols: int, tokens, out=None,
                   status=None, stream=None):
    """Gathers and dequantises one table row per token id -> [T, cols] f32."""
    import torch
    op = "embedding_rows"
    _require(table.is_cuda and table.is_contiguous(), op,
             "table must be a contiguous CUDA tensor")
    _require(table.numel() * table.element_size() >= vocab * row_bytes(qtype, cols),
             op, "table smaller than vocab rows")
    _require(tokens.is_cuda and tokens.dtype == torch.int32, op,
             "tokens must be int32 CUDA")
    rows = tokens.numel()
    if out is None:
        out = torch.empty((rows, cols), dtype=torch.float32, device=tokens.device)
    _check(load().mlb_embedding_gather(_ptr(table), qtype, vocab, cols,
                                       _ptr(tokens), rows, _ptr(out),
                                       _ptr(status), _stream(stream)), op)
    return out


def embedding_row(table, qtype: int, vocab: int, cols: int, token: int,
                  out=None, stream=None):
    """One dequantised row for a host token id -> [cols] f32 (IndexError when
    the id is outside the table, like the reference's std::out_of_range)."""
    import torch
    if out is None:
        out = torch.empty((cols,), dtype=torch.float32, device=table.device)
    _check(load().mlb_embedding_row(_ptr(table), qtype, vocab, cols, int(token),
                                    _ptr(out), _stream(stream)), "embedding_row")
    return out


def linear(weight, qtype: int, n: int, k: int, x, out=None, stream=None):
    """y = x · dequant(W)^T for x [T, k] (or [k]) -> [T, n] (or [n])."""
    import torch
    op = "linear"
    _require(weight.is_cuda and weight.is_contiguous(), op,
             "weight must be a contiguous CUDA tensor")
    _require(weight.numel() * weight.element_size() >= n * row_bytes(qtype, k), op,
             "weight smaller than n rows")
    _f32_cuda(x, op, "x")
    _require(x.shape[-1] == k, op, "input size mismatch")
    t_rows = x.numel() // k
    if out is None:
        shape = (n,) if x.dim() == 1 else (t_rows, n)
        out = torch.empty(shape, dtype=torch.float32, device=x.device)
    _check(load().mlb_linear_f32(_ptr(weight), qtype, n, k, _ptr(x), t_rows,
                                 _ptr(out), _stream(stream)), op)
    return out


def kv_write(keys, values, k, v, position: int, stream=None):
    """Writes k, v [rows, kv_heads, hd] at positions [position, +rows) of one
    layer's cache keys/values [max_seq, kv_heads, hd]."""
    op = "kv_write"
    for t, name in ((keys, "keys"), (values, "values"), (k, "k"), (v, "v")):
        _f32_cuda(t, op, name)
    _require(keys.shape == values.shape and keys.dim() == 3, op,
             "cache must be [max_seq, kv_heads, head_dim]")
    max_seq, kvh, hd = keys.shape
    _require(k.numel() == v.numel() and k.numel() % (kvh * hd) == 0, op,
             "k/v shape mismatch")
    rows = k.numel() // (kvh * hd)
    _check(load().mlb_kv_write_f32(_ptr(keys), _ptr(values), _ptr(k), _ptr(v),
                                   int(position), rows, max_seq, kvh, hd,
                                   _stream(stream)), op)


def attention_scratch_floats(n_heads: int, n_kv_heads: int, head_dim: int,
                             position: int) -> int:
    return int(load().mlb_attention_scratch_floats(n_heads, n_kv_heads,
                                                   head_dim, position))


def attention_decode(q, keys, values, position: int, out=None, scratch=None,
                     stream=None):
    """Decode attention of q [n_heads, hd] at `position` over one layer's
    cache [max_seq, kv_heads, hd] -> [n_heads, hd]."""
    import torch
    op = "attention_decode"
    for t, name in ((q, "q"), (keys, "keys"), (values, "values")):
        _f32_cuda(t, op, name)
    max_seq, kvh, hd = keys.shape
    nh = q.numel() // hd
    if out is None:
        out = torch.empty((nh, hd), dtype=torch.float32, device=q.device)
    need = attention_scratch_floats(nh, kvh, hd, position)
    if scratch is None:
        scratch = torch.empty(max(need, 1), dtype=torch.float32, device=q.device)
    _check(load().mlb_attention_decode_f32(
        _ptr(q), _ptr(keys), _ptr(values), _ptr(out), int(position), max_seq,
        nh, kvh, hd, _ptr(scratch), scratch.numel(), _stream(stream)), op)
    return out


def attention_rows(q, keys, values, position: int, out=None, scratch=None,
                   stream=None):
    """Causal attention of q [rows, n_heads, hd] (row r at position + r) over
    one layer's cache [max_seq, kv_heads, hd] -> [rows, n_heads, hd]."""
    import torch
    op = "attention_rows"
    for t, name in ((q, "q"), (keys, "keys"), (values, "values")):
        _f32_cuda(t, op, name)
    max_seq, kvh, hd = keys.shape
    rows, nh = q.shape[0], q.shape[1]
    if out is None:
        out = torch.empty((rows, nh, hd), dtype=torch.float32, device=q.device)
    if rows == 0:
        return out
    need = load().mlb_attention_rows_scratch_floats(nh, kvh, hd, int(position), rows)
    if scratch is None:
        scratch = torch.empty(max(need, 1), dtype=torch.float32, device=q.device)
    _check(load().mlb_attention_rows_f32(
        _ptr(q), _ptr(keys), _ptr(values), _ptr(out), int(position), rows, max_seq,
        nh, kvh, hd, _ptr(scratch), scratch.numel(), _stream(stream)), op)
    return out


def linear_rows(weight, qtype: int, n: int, k: int, x, out=None, scratch=None,
                stream=None):
    """y = x . dequant(W)^T for x [T, k] -> [T, n]; tensor cores from 48
    tokens on (mlb_linear_rows_f32)."""
    import torch
    op = "linear_rows"
    _require(weight.is_cuda and weight.is_contiguous(), op,
             "weight must be a contiguous CUDA tensor")
    _require(weight.numel() * weight.element_size() >= n * row_bytes(qtype, k), op,
             "weight smaller than n rows")
    _f32_cuda(x, op, "x")
    _require(x.shape[-1] == k, op, "input size mismatch")
    t_rows = x.numel() // k
    if out is None:
        out = torch.empty((t_rows, n), dtype=torch.float32, device=x.device)
    need = load().mlb_linear_rows_scratch_floats(k, t_rows)
    if scratch is None:
        scratch = torch.empty(max(need, 1), dtype=torch.float32, device=x.device)
    _check(load().mlb_linear_rows_f32(_ptr(weight), qtype, n, k, _ptr(x), t_rows,
                                      _ptr(out), _ptr(scratch), scratch.numel(),
                                      _stream(stream)), op)
    return out


def linear_rows_group(weights, qtype: int, ns, k: int, x, scratch=None, stream=None):
    """[x . dequant(W_m)^T for each W_m] in one launch (up to 3 matrices of
    the same format and width k)."""
    import torch
    op = "linear_rows_group"
    _f32_cuda(x, op, "x")
    _require(x.shape[-1] == k, op, "input size mismatch")
    _require(1 <= len(weights) == len(ns) <= 3, op, "1 to 3 matrices")
    t_rows = x.numel() // k
    outs = [torch.empty((t_rows, n), dtype=torch.float32, device=x.device) for n in ns]
    for w, n in zip(weights, ns):
        _require(w.is_cuda and w.is_contiguous(), op, "weights must be contiguous CUDA tensors")
        _require(w.numel() * w.element_size() >= n * row_bytes(qtype, k), op,
                 "weight smaller than n rows")
    need = load().mlb_linear_rows_scratch_floats(k, t_rows)
    if scratch is None:
        scratch = torch.empty(max(need, 1), dtype=torch.float32, device=x.device)
    count = len(weights)
    wp = (ctypes.c_void_p * count)(*[w.data_ptr() for w in weights])
    na = (ctypes.c_int64 * count)(*ns)
    yp = (ctypes.c_void_p * count)(*[o.data_ptr() for o in outs])
    _check(load().mlb_linear_rows_group_f32(count, wp, qtype, na, k, _ptr(x), t_rows, yp,
                                            _ptr(scratch), scratch.numel(), _stream(stream)),
           op)
    return outs


def status_check(status, stream=None) -> int:
    """Synchronises and returns the device status bits (0 = clean)."""
    bits = ctypes.c_int32(0)
    rc = load().mlb_status_check(_ptr(status), ctypes.byref(bits),
                                 _stream(stream))
    if rc not in (0, 3):
        _check(rc, "status_check")
    return bits.value


def set_gemv_path(path: int) -> int:
    """Kernel choice of linear() for ggml formats: 0 automatic, 1 CUDA-core
    GEMV, 2 int8 tensor-core GEMV wherever its shape rules allow.  Returns
    the previous setting."""
    previous = load().mlb_gemv_path()
    _check(load().mlb_set_gemv_path(int(path)), "set_gemv_path")
    return previous


def set_attention_path(path: int) -> int:
    """Kernel choice of attention_rows() for prompt chunks: 0 automatic, 1
    CUDA-core kernels, 2 tensor cores wherever the shape allows.  Returns the
    previous setting."""
    previous = load().mlb_attention_path()
    _check(load().mlb_set_attention_path(int(path)), "set_attention_path")
    return previous


def set_launch_overlap(on: int) -> int:
    """1: kernels launch with programmatic dependent launch (each overlaps
    the tail of the stream's previous kernel; the default), 0: one after
    another.  Returns the previous setting."""
    previous = load().mlb_launch_overlap()
    _check(load().mlb_set_launch_overlap(int(on)), "set_launch_overlap")
    return previous


def wait_timeouts() -> int:
    """Bounded device waits that gave up on the current device (0 when every
    bulk copy landed in time)."""
    count = ctypes.c_uint(0)
    _check(load().mlb_wait_timeouts(ctypes.byref(count)), "wait_timeouts")
    return count.value
