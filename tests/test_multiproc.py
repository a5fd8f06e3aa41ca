"""Token-range sharding across ranks, as two gloo processes on the CPU.

Each rank takes its contiguous shard of a batch (workloads.shard_range),
runs the layer operators on its rows alone (the CPU oracle stands in for one
GPU's kernels), and the rows are gathered only to check the result: the
shards' outputs concatenate to the unsharded batch bit for bit, with no
exchange needed between ranks on the data path.  A second test makes one
rank fail before the check and verifies that the other rank learns of it
through the store instead of waiting forever.
"""
import os
import socket

import numpy as np
import pytest


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _batch(seed=3):
    rng = np.random.default_rng(seed)
    T, H, nq, nk, hd = 37, 96, 3, 1, 16
    return {
        "x": rng.standard_normal((T, H), dtype=np.float32),
        "r": rng.standard_normal((T, H), dtype=np.float32),
        "w": rng.standard_normal(H, dtype=np.float32),
        "q": rng.standard_normal((T, nq, hd), dtype=np.float32),
        "k": rng.standard_normal((T, nk, hd), dtype=np.float32),
        "pos": np.arange(T, dtype=np.int32) * 5,
        "g": rng.standard_normal((T, 64), dtype=np.float32),
        "u": rng.standard_normal((T, 64), dtype=np.float32),
    }


def _layer(orc, b, lo, hi):
    y, h = orc.rmsnorm(b["x"][lo:hi], b["w"], 1e-5, residual=b["r"][lo:hi])
    q, k, _ = orc.rope(b["q"][lo:hi], b["k"][lo:hi], b["pos"][lo:hi], 1e4, 1)
    o = orc.swiglu(b["g"][lo:hi], b["u"][lo:hi])
    return np.concatenate([y.ravel(), h.ravel(), q.ravel(), k.ravel(), o.ravel()])


def _worker(rank, world, port, mode, result_path):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, here)
    import conftest  # noqa: F401  (sets sys.path for the package and oracle)
    import datetime
    import torch
    import torch.distributed as dist
    import workloads as wl
    from oracle import Oracle

    store = dist.TCPStore("127.0.0.1", port, world, rank == 0,
                          timeout=datetime.timedelta(seconds=20))
    dist.init_process_group("gloo", store=store, rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=20))
    b = _batch()
    T = b["x"].shape[0]
    lo, hi = wl.shard_range(T, world, rank)
    if mode == "fail" and rank == 1:
        store.set("failed/1", "injected host failure")
        dist.destroy_process_group()
        return
    out = _layer(Oracle(), b, lo, hi)
    if mode == "fail":
        # Between steps, before any collective, rank 0 waits (bounded) for
        # rank 1's status on the store: a heartbeat or a failure record.
        import time
        deadline = time.monotonic() + 15.0
        seen = "timeout"
        while time.monotonic() < deadline:
            if store.check(["failed/1"]):
                seen = "saw-failure"
                break
            if store.check(["alive/1"]):
                seen = "no-failure"
                break
            time.sleep(0.01)
        with open(result_path, "w") as f:
            f.write(seen)
        dist.destroy_process_group()
        return
    sizes = [None] * world
    dist.all_gather_object(sizes, (lo, hi, out.tobytes()))
    if rank == 0:
        full = _layer(Oracle(), b, 0, T)
        parts = [np.frombuffer(p[2], np.float32) for p in sizes]
        # re-interleave per-op sections: compare op by op via a shard-wise run
        ok = all(sizes[i][1] == sizes[i + 1][0] for i in range(world - 1))
        ok = ok and sizes[0][0] == 0 and sizes[-1][1] == T
        stitched = []
        for lo_, hi_ in [(p[0], p[1]) for p in sizes]:
            stitched.append(_layer(Oracle(), b, lo_, hi_))
        ok = ok and all(np.array_equal(a.view(np.uint32), p.view(np.uint32))
                        for a, p in zip(stitched, parts))
        # the union of shard outputs equals the unsharded batch
        per_op = []
        for name in range(5):
            chunks = []
            for p, (lo_, hi_) in zip(parts, [(s[0], s[1]) for s in sizes]):
                n = hi_ - lo_
                lens = [n * 96, n * 96, n * 3 * 16, n * 16, n * 64]
                off = sum(lens[:name])
                chunks.append(p[off:off + lens[name]])
            per_op.append(np.concatenate(chunks))
        ok = ok and np.array_equal(np.concatenate(per_op).view(np.uint32),
                                   full.view(np.uint32))
        with open(result_path, "w") as f:
            f.write("ok" if ok else "mismatch")
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_sharded_rows_match_unsharded(tmp_path, world):
    import torch.multiprocessing as mp
    result = str(tmp_path / "result.txt")
    mp.spawn(_worker, args=(world, _free_port(), "ok", result), nprocs=world,
             join=True)
    assert open(result).read() == "ok"


def test_failed_rank_is_seen_through_the_store(tmp_path):
    import torch.multiprocessing as mp
    result = str(tmp_path / "result.txt")
    mp.spawn(_worker, args=(2, _free_port(), "fail", result), nprocs=2, join=True)
    assert open(result).read() == "saw-failure"
