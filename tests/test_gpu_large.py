"""Full-size configs on the GPU: the LLaMA-3-8B prefill (T = 16384) and the
Qwen2-7B long prefill (T = 65536, NeoX RoPE with q/k bias, Q4_1 table).

The oracle cannot run every row of these in seconds, so each operator is
checked on a row sample — the first and last row of each of 8 token-range
shards plus random rows, 4096+ in all — against the oracle (bit-exact where
the reference is exact, 1e-5 relative otherwise), and on every row through
properties that hold at any size:
  * RMSNorm: each row of (y / w) has mean square 1 / (1 + eps / mean(h^2));
  * embedding: rows of equal token ids are identical;
  * RoPE: each rotated pair keeps its length (to fp32 rounding).
"""
import numpy as np
import pytest

from conftest import assert_bitexact, assert_rel

import mlb
import workloads as wl

pytestmark = pytest.mark.gpu


def _sample_rows(T, n_random=4064, seed=0):
    rng = np.random.default_rng(seed)
    edges = []
    for g in range(8):
        b, e = wl.shard_range(T, 8, g)
        edges += [b, e - 1]
    rows = np.unique(np.r_[edges, rng.integers(0, T, n_random)])
    return rows


@pytest.mark.parametrize("name", ["llama3-8b-t16384", "qwen2-7b-t65536"])
def test_full_size_config(cuda, oracle, name):
    import torch
    cfg = wl.CONFIGS[name]
    T = cfg.tokens
    d = wl.make_inputs(cfg, cuda, ops=("embedding", "rmsnorm", "rope", "swiglu"))
    rows = _sample_rows(T)
    rows_t = torch.from_numpy(rows).to(cuda)
    pick = lambda t: t.index_select(0, rows_t).cpu().numpy()  # noqa: E731

    # inputs of the sampled rows, captured before the in-place RoPE
    x_s, q_s, k_s = pick(d["x"]), pick(d["q"]), pick(d["k"])
    r_s = pick(d["residual"]) if cfg.residual else None
    g_s, u_s = pick(d["gate"]), pick(d["up"])
    tok = d["tokens"].cpu().numpy()
    pos = d["positions"].cpu().numpy()

    # embedding
    mlb.embedding_rows(d["table"], cfg.qtype, cfg.vocab, cfg.hidden, d["tokens"],
                       out=d["emb_out"], status=d["status"])
    table = d["table"].cpu().numpy()
    want, bad = oracle.embedding(table, cfg.qtype, cfg.vocab, cfg.hidden, tok[rows])
    assert bad == 0
    emb_s = pick(d["emb_out"])
    assert_bitexact(emb_s, want, "embedding sample")
    # property: equal ids -> identical rows (every row with a repeated id)
    order = np.argsort(tok, kind="stable")
    dup = order[1:][tok[order[1:]] == tok[order[:-1]]]
    if dup.size:
        prev = order[:-1][tok[order[1:]] == tok[order[:-1]]]
        a = d["emb_out"].index_select(0, torch.from_numpy(dup).to(cuda))
        b = d["emb_out"].index_select(0, torch.from_numpy(prev).to(cuda))
        assert torch.equal(a.view(torch.int32), b.view(torch.int32))
    del table

    # (residual) RMSNorm
    mlb.rms_norm(d["x"], d["w"], cfg.eps, residual=d["residual"], h_out=d["h"],
                 out=d["y"])
    w = d["w"].cpu().numpy()
    if cfg.residual:
        wy, wh = oracle.rmsnorm(x_s, w, cfg.eps, residual=r_s)
        assert_bitexact(pick(d["h"]), wh, "h sample")
        hsrc = d["h"]
    else:
        wy = oracle.rmsnorm(x_s, w, cfg.eps)
        hsrc = d["x"]
    assert_rel(pick(d["y"]), wy, what="rmsnorm sample")
    # property on every row: mean((y/w)^2) = ms / (ms + eps), ms = mean(h^2)
    ms = (hsrc.double() ** 2).mean(dim=1)
    lhs = ((d["y"].double() / d["w"].double()) ** 2).mean(dim=1)
    rhs = ms / (ms + cfg.eps)
    assert float(((lhs - rhs).abs() / rhs).max()) < 1e-5

    # RoPE (+bias)
    pre_norm = torch.linalg.vector_norm(d["q"].view(T, cfg.n_heads, -1), dim=2)
    table_r = torch.from_numpy(mlb.rope_table(cfg.theta, cfg.head_dim,
                                              cfg.max_position() + 1)).to(cuda)
    mlb.rope(d["q"], d["k"], d["positions"], table_r, cfg.neox, d["bq"], d["bk"],
             status=d["status"])
    bq = d["bq"].cpu().numpy() if d["bq"] is not None else None
    bk = d["bk"].cpu().numpy() if d["bk"] is not None else None
    wq, wk, bad = oracle.rope(q_s, k_s, pos[rows], cfg.theta, cfg.neox, bq, bk)
    assert bad == 0
    assert_bitexact(pick(d["q"]), wq, "rope q sample")
    assert_bitexact(pick(d["k"]), wk, "rope k sample")
    if d["bq"] is None:
        post_norm = torch.linalg.vector_norm(d["q"].view(T, cfg.n_heads, -1), dim=2)
        assert float(((post_norm - pre_norm).abs() / pre_norm).max()) < 1e-5

    # SwiGLU
    mlb.swiglu(d["gate"], d["up"], out=d["ffn_out"])
    assert_rel(pick(d["ffn_out"]), oracle.swiglu(g_s, u_s), what="swiglu sample")
    assert mlb.status_check(d["status"]) == 0
