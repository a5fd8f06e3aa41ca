"""Layer-operator workloads: shapes, synthetic inputs, sharding, byte counts.

The named shapes are stand-ins for the models' per-layer operator sizes
(no model weights are involved): activations ~N(0,1), RMSNorm weight
~N(1, 0.1), softmax scores ~N(0, 4) (sigma 2), attention bias ~N(0, 0.02)
(sigma 0.02), fp16 block scales d ~U(0.001, 0.05), Q4_1 minima m ~U(-0.1, 0),
Q8_0 quants ~U[-127, 127], 4-bit quants ~U{0..15}, token ids ~U[0, vocab).

Inputs are generated on the device from a seeded torch generator; the
checkers copy the rows they need back to the host.
"""
from __future__ import annotations

import dataclasses
from typing import Optional

F32, Q8_0, Q4_0, Q4_1 = 0, 1, 2, 3
QNAME = {F32: "F32", Q8_0: "Q8_0", Q4_0: "Q4_0", Q4_1: "Q4_1"}
QTYPE_BY_NAME = {v: k for k, v in QNAME.items()}
BLOCK_BYTES = {F32: 128, Q8_0: 34, Q4_0: 18, Q4_1: 20}


def row_bytes(qtype: int, cols: int) -> int:
    if qtype == F32:
        return 4 * cols
    return (cols + 31) // 32 * BLOCK_BYTES[qtype]


@dataclasses.dataclass(frozen=True)
class LayerConfig:
    name: str
    tokens: int             # T, token rows
    hidden: int             # H
    eps: float
    residual: bool          # fused residual add before RMSNorm
    ffn: int                # F, SwiGLU width
    neox: bool
    theta: float
    n_heads: int
    n_kv_heads: int
    head_dim: int
    positions: str          # "arange" (0..T-1) or "random:<max>"
    qtype: int              # embedding table format
    vocab: int
    bias: bool = False      # q/k attention bias before RoPE
    softmax_cols: int = 0   # causal softmax rows [n_heads*T, softmax_cols]
    seed: int = 0

    def max_position(self) -> int:
        if self.positions == "arange":
            return self.tokens - 1
        return int(self.positions.split(":")[1])

    # Algorithmic HBM bytes per launch (sin/cos table excluded: derived
    # data that stays resident in L2).
    def bytes_rmsnorm(self, t: Optional[int] = None) -> int:
        t = self.tokens if t is None else t
        per = 16 if self.residual else 8
        return per * t * self.hidden + 4 * self.hidden

    def bytes_swiglu(self, t: Optional[int] = None) -> int:
        t = self.tokens if t is None else t
        return 12 * t * self.ffn

    def bytes_rope(self, t: Optional[int] = None) -> int:
        t = self.tokens if t is None else t
        heads = self.n_heads + self.n_kv_heads
        b = 8 * t * heads * self.head_dim + 4 * t
        if self.bias:
            b += 4 * heads * self.head_dim
        return b

    def bytes_embedding(self, t: Optional[int] = None) -> int:
        t = self.tokens if t is None else t
        return t * (row_bytes(self.qtype, self.hidden) + 4 * self.hidden + 4)

    def bytes_softmax(self, t: Optional[int] = None) -> int:
        if not self.softmax_cols:
            return 0
        t = self.tokens if t is None else t
        rows = self.n_heads * t
        # causal: row (h, p) reads p+1 visible scores; p = 0..t-1 per head
        visible = self.n_heads * t * (t + 1) // 2
        return 4 * visible + 4 * rows * self.softmax_cols


CONFIGS = {
    # Qwen2-0.5B layer ops, T=256 (the reference's CPU-runnable case).
    "qwen2-0.5b-t256": LayerConfig(
        "qwen2-0.5b-t256", tokens=256, hidden=896, eps=1e-6, residual=True,
        ffn=4864, neox=True, theta=1e6, n_heads=14, n_kv_heads=2, head_dim=64,
        positions="arange", qtype=Q8_0, vocab=151936, softmax_cols=256),
    # LLaMA-7B decode-style batch, T=64 at random positions.
    "llama-7b-t64": LayerConfig(
        "llama-7b-t64", tokens=64, hidden=4096, eps=1e-5, residual=False,
        ffn=11008, neox=False, theta=1e4, n_heads=32, n_kv_heads=32,
        head_dim=128, positions="random:2047", qtype=Q4_0, vocab=32000),
    # LLaMA-3-8B prefill, T=16384.
    "llama3-8b-t16384": LayerConfig(
        "llama3-8b-t16384", tokens=16384, hidden=4096, eps=1e-5, residual=True,
        ffn=14336, neox=False, theta=5e5, n_heads=32, n_kv_heads=8,
        head_dim=128, positions="arange", qtype=Q8_0, vocab=128256),
    # Qwen2-7B long prefill, T=65536, q/k bias.
    "qwen2-7b-t65536": LayerConfig(
        "qwen2-7b-t65536", tokens=65536, hidden=3584, eps=1e-6, residual=False,
        ffn=18944, neox=True, theta=1e6, n_heads=28, n_kv_heads=4,
        head_dim=128, positions="arange", qtype=Q4_1, vocab=152064, bias=True),
}

SWEEP_HIDDEN = (512, 896, 2048, 4096, 8192, 16384)
SWEEP_TOKENS = (1, 64, 1024, 16384, 262144)
SWEEP_VOCAB = 32000


def shard_range(total: int, world: int, rank: int):
    """Contiguous token range [begin, end) of `rank`; the first
    total % world shards get one extra row."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad world/rank")
    base, extra = divmod(total, world)
    begin = rank * base + min(rank, extra)
    end = begin + base + (1 if rank < extra else 0)
    return begin, end


# ---------------------------------------------------------------------------
# Device-side synthetic inputs (torch is plumbing: memory + RNG).

def _gen(device, seed: int, stream_id: int):
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(seed * 1000003 + stream_id)
    return g


def quant_table(qtype: int, vocab: int, cols: int, device, seed: int = 0):
    """A [vocab] x row_bytes table of ggml blocks as a flat uint8 tensor."""
    import torch
    g = _gen(device, seed, 11)
    if qtype == F32:
        t = torch.randn(vocab * cols, generator=g, device=device,
                        dtype=torch.float32)
        return t.view(torch.uint8)
    bb = BLOCK_BYTES[qtype]
    nb = vocab * ((cols + 31) // 32)
    blocks = torch.randint(0, 256, (nb, bb), generator=g, device=device,
                           dtype=torch.uint8)
    if qtype == Q8_0:
        qs = torch.randint(-127, 128, (nb, 32), generator=g, device=device,
                           dtype=torch.int8)
        blocks[:, 2:34] = qs.view(torch.uint8)
    d = (torch.rand(nb, generator=g, device=device) * 0.049 + 0.001)
    blocks[:, 0:2] = d.to(torch.float16).view(torch.uint8).view(nb, 2)
    if qtype == Q4_1:
        m = torch.rand(nb, generator=g, device=device) * -0.1
        blocks[:, 2:4] = m.to(torch.float16).view(torch.uint8).view(nb, 2)
    return blocks.view(-1)


def positions_for(cfg: LayerConfig, device, tokens: Optional[int] = None,
                  offset: int = 0):
    import torch
    t = cfg.tokens if tokens is None else tokens
    if cfg.positions == "arange":
        return torch.arange(offset, offset + t, device=device, dtype=torch.int32)
    hi = cfg.max_position()
    g = _gen(device, cfg.seed, 7)
    return torch.randint(0, hi + 1, (t,), generator=g, device=device,
                         dtype=torch.int32)


ALL_OPS = ("embedding", "rmsnorm", "rope", "swiglu", "softmax")


def make_inputs(cfg: LayerConfig, device, tokens: Optional[int] = None,
                pos_offset: int = 0, ops=ALL_OPS):
    """Allocates and fills the input and output buffers of the layer-op
    step's operators named in `ops` (embedding, residual RMSNorm,
    RoPE(+bias), SwiGLU, softmax); buffers of other operators are None."""
    import torch
    T = cfg.tokens if tokens is None else tokens
    H, F, hd = cfg.hidden, cfg.ffn, cfg.head_dim
    s = cfg.seed
    f32 = dict(device=device, dtype=torch.float32)
    d = dict.fromkeys(["table", "tokens", "emb_out", "x", "residual", "w", "h",
                       "y", "gate", "up", "ffn_out", "q", "k", "positions",
                       "bq", "bk", "scores", "valid_len", "probs"])
    if "embedding" in ops:
        d["table"] = quant_table(cfg.qtype, cfg.vocab, H, device, s)
        d["tokens"] = torch.randint(0, cfg.vocab, (T,),
                                    generator=_gen(device, s, 1),
                                    device=device, dtype=torch.int32)
        d["emb_out"] = torch.empty((T, H), **f32)
    if "rmsnorm" in ops:
        d["x"] = torch.randn((T, H), generator=_gen(device, s, 2), **f32)
        if cfg.residual:
            d["residual"] = torch.randn((T, H), generator=_gen(device, s, 3), **f32)
            d["h"] = torch.empty((T, H), **f32)
        d["w"] = torch.randn((H,), generator=_gen(device, s, 4), **f32) * 0.1 + 1.0
        d["y"] = torch.empty((T, H), **f32)
    if "swiglu" in ops:
        d["gate"] = torch.randn((T, F), generator=_gen(device, s, 5), **f32)
        d["up"] = torch.randn((T, F), generator=_gen(device, s, 6), **f32)
        d["ffn_out"] = torch.empty((T, F), **f32)
    if "rope" in ops:
        d["q"] = torch.randn((T, cfg.n_heads, hd), generator=_gen(device, s, 8),
                             **f32)
        d["k"] = torch.randn((T, cfg.n_kv_heads, hd),
                             generator=_gen(device, s, 9), **f32)
        d["positions"] = positions_for(cfg, device, T, pos_offset)
        if cfg.bias:
            d["bq"] = torch.randn((cfg.n_heads * hd,),
                                  generator=_gen(device, s, 12), **f32) * 0.02
            d["bk"] = torch.randn((cfg.n_kv_heads * hd,),
                                  generator=_gen(device, s, 13), **f32) * 0.02
    if "softmax" in ops and cfg.softmax_cols:
        rows = cfg.n_heads * T
        d["scores"] = torch.randn((rows, cfg.softmax_cols),
                                  generator=_gen(device, s, 14), **f32) * 2.0
        # row (head, p) sees p+1 scores (causal)
        p = torch.arange(T, device=device, dtype=torch.int32) % cfg.softmax_cols
        d["valid_len"] = (p + 1).repeat(cfg.n_heads)
        d["probs"] = torch.empty_like(d["scores"])
    d["status"] = torch.zeros(1, device=device, dtype=torch.int32)
    return d


# ---------------------------------------------------------------------------
# Host-side (numpy) inputs for CPU-only checks of the oracle.

def numpy_quant_table(qtype: int, vocab: int, cols: int, seed: int = 0):
    import numpy as np
    rng = np.random.default_rng(seed)
    if qtype == F32:
        return rng.standard_normal(vocab * cols, dtype=np.float32).view(np.uint8)
    bb = BLOCK_BYTES[qtype]
    nb = vocab * ((cols + 31) // 32)
    blocks = rng.integers(0, 256, size=(nb, bb), dtype=np.uint8)
    if qtype == Q8_0:
        blocks[:, 2:34] = rng.integers(-127, 128, size=(nb, 32),
                                       dtype=np.int8).view(np.uint8)
    d = rng.uniform(0.001, 0.05, nb).astype(np.float16)
    blocks[:, 0:2] = d.view(np.uint8).reshape(nb, 2)
    if qtype == Q4_1:
        m = rng.uniform(-0.1, 0.0, nb).astype(np.float16)
        blocks[:, 2:4] = m.view(np.uint8).reshape(nb, 2)
    return blocks.reshape(-1)
