"""Layer-operator benchmark: tokens/s and HBM GB/s of one fused layer-op step.

A step is one pass of the hot path over one batch of token rows, on inputs
already resident in HBM: token-embedding gather (dequantising the table's
blocks) -> residual-add + RMSNorm -> q/k bias + RoPE -> SwiGLU (-> causal
softmax rows where the workload defines them).  The default workload is the
LLaMA-3-8B-shaped prefill (T = 16384 token rows per GPU, hidden 4096, FFN
14336, 32/8 heads x 128, Q8_0 table [128256, 4096]).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME]
    python bench.py --impl reference ...   # the reference's CPU operators

For N > 1 launch one process per GPU with torch.distributed.run; the
workload's T token rows are split into N contiguous ranges, one per rank
(strong scaling: the split the sharded prefill workloads name; `--weak` gives
every rank its own T rows instead), and the data path has no collective.  Timing: W untimed steps, then K steps
between a barrier + synchronize on both sides, CUDA events on the launching
stream, max over ranks.  Inputs are far larger than the 126 MB L2, so no
flush is needed between steps.  Rank 0 prints one JSON line.
"""
from __future__ import annotations

import argparse
import dataclasses
import glob
import json
import subprocess
import math
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "mini-lla_b200")
ORACLE_DIR = os.path.join(ROOT, "oracle")
sys.path.insert(0, PKG)

import workloads as wl  # noqa: E402

METRIC = "fused layer-op tokens/s and HBM GB/s vs ~8 TB/s peak at 1/2/4/8 B200"
SPEC_HBM_GBS = 8000.0
FALLBACK_HBM_GBS = 6650.0


def measured_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def profile_traffic(kernel: str, workload: str):
    """dram bytes per launch of `kernel` recorded from an ncu capture in
    profiles/<kernel>_<workload>.md (line `traffic_bytes_per_launch: N`)."""
    path = os.path.join(ROOT, "profiles", f"{kernel}_{workload}.md")
    try:
        for line in open(path):
            if line.strip().startswith("traffic_bytes_per_launch:"):
                return int(line.split(":", 1)[1].strip())
    except OSError:
        pass
    return None


# ---------------------------------------------------------------- clocks

REASON_BITS = {
    0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
    0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
    0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
    0x100: "display_clock_setting",
}


class ClockSampler:
    """Polls SM clock and clock-event reasons through NVML (read-only)
    while the timed region runs."""

    def __init__(self, device_index: int, interval: float = 0.01):
        self.samples = []
        self.reasons = 0
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nvml = pynvml
            self._h = self._handle(pynvml, device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(
                self._h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._nvml = None
        self.interval = interval

    @staticmethod
    def _handle(nv, cuda_index):
        """NVML handle of the CUDA device (matched by PCI bus id, since
        CUDA_VISIBLE_DEVICES renumbers devices)."""
        try:
            import torch
            p = torch.cuda.get_device_properties(cuda_index)
            bus = "%08x:%02x:%02x.0" % (p.pci_domain_id, p.pci_bus_id,
                                        p.pci_device_id)
            return nv.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            return nv.nvmlDeviceGetHandleByIndex(cuda_index)

    def _run(self):
        nv = self._nvml
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                fn = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                    nv.nvmlDeviceGetCurrentClocksThrottleReasons
                self.reasons |= int(fn(self._h)) & ~0x1
            except Exception:
                pass
            time.sleep(self.interval)

    def __enter__(self):
        if self._nvml is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [],
                    "samples": 0}
        reasons = [n for b, n in REASON_BITS.items() if self.reasons & b]
        return {"sm_mhz": statistics.median(self.samples),
                "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(self.samples)}


# ---------------------------------------------------------------- GPU arm

class LayerStep:
    """Device buffers and launches of one layer-op step for `tokens` rows."""

    def __init__(self, cfg, device, tokens: int, pos_offset: int, ops=None):
        import torch
        import mlb
        self.mlb = mlb
        self.cfg = cfg
        self.T = tokens
        self.dev = device
        all_ops = ["embedding", "rmsnorm", "rope", "swiglu"]
        if cfg.softmax_cols:
            all_ops.append("softmax")
        self.ops = [o for o in all_ops if ops is None or o in ops]
        if not self.ops:
            raise ValueError(f"no operator of {ops} in workload {cfg.name}")
        self.d = wl.make_inputs(cfg, device, tokens=tokens, pos_offset=pos_offset,
                                ops=self.ops)
        max_pos = (pos_offset + tokens - 1) if cfg.positions == "arange" \
            else cfg.max_position()
        self.rope_table = torch.from_numpy(
            mlb.rope_table(cfg.theta, cfg.head_dim, max_pos + 1)).to(device)

    def bytes(self):
        c, t = self.cfg, self.T
        b = {"embedding": c.bytes_embedding(t), "rmsnorm": c.bytes_rmsnorm(t),
             "rope": c.bytes_rope(t), "swiglu": c.bytes_swiglu(t),
             "softmax": c.bytes_softmax(t)}
        return {o: b[o] for o in self.ops}

    def launch(self, op, stream=None, rows=None):
        """Launches one operator over rows [r0, r1) (all rows by default)."""
        c, d, m = self.cfg, self.d, self.mlb
        r0, r1 = (0, self.T) if rows is None else rows
        if r1 <= r0:
            return
        sl = slice(r0, r1)
        if op == "embedding":
            m.embedding_rows(d["table"], c.qtype, c.vocab, c.hidden,
                             d["tokens"][sl], out=d["emb_out"][sl],
                             status=d["status"], stream=stream)
        elif op == "rmsnorm":
            m.rms_norm(d["x"][sl], d["w"], c.eps,
                       residual=None if d["residual"] is None else d["residual"][sl],
                       h_out=None if d["h"] is None else d["h"][sl],
                       out=d["y"][sl], stream=stream)
        elif op == "rope":
            m.rope(d["q"][sl], d["k"][sl], d["positions"][sl], self.rope_table,
                   c.neox, d["bq"], d["bk"], status=d["status"], stream=stream)
        elif op == "swiglu":
            m.swiglu(d["gate"][sl], d["up"][sl], out=d["ffn_out"][sl],
                     stream=stream)
        elif op == "softmax":
            h = c.n_heads
            if (r0, r1) == (0, self.T):  # every row: one launch
                m.softmax_rows(d["scores"], d["valid_len"], out=d["probs"],
                               status=d["status"], stream=stream)
                return
            # rows of head-major scores belonging to tokens [r0, r1)
            for head in range(h):
                a, b = head * self.T + r0, head * self.T + r1
                m.softmax_rows(d["scores"][a:b], d["valid_len"][a:b],
                               out=d["probs"][a:b], status=d["status"],
                               stream=stream)

    def step(self, events=None):
        import torch
        for i, op in enumerate(self.ops):
            if events is not None:
                events[i].record()
            self.launch(op)
        if events is not None:
            events[len(self.ops)].record()


def gpu_numa_cpus(device_index: int):
    """CPUs of the NUMA node the GPU hangs off (from sysfs), or None when the
    node is unknown or the host has a single node."""
    import torch
    try:
        p = torch.cuda.get_device_properties(device_index)
        bdf = f"{p.pci_domain_id:04x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
        node = int(open(f"/sys/bus/pci/devices/{bdf}/numa_node").read().strip())
        if node < 0 or len(glob.glob("/sys/devices/system/node/node[0-9]*")) < 2:
            return None
        cpus = parse_cpulist(open(f"/sys/devices/system/node/node{node}/cpulist").read())
        return node, cpus & os.sched_getaffinity(0)
    except (OSError, ValueError, AttributeError, RuntimeError, AssertionError):
        return None


def parse_cpulist(text: str) -> set:
    """sysfs cpulist ("0-15,32-47") -> set of CPU ids."""
    cpus = set()
    for part in text.strip().split(","):
        if part:
            lo, _, hi = part.partition("-")
            cpus.update(range(int(lo), int(hi or lo) + 1))
    return cpus


def pinned_near_gpu(device_index: int, numa: bool):
    """A context for allocating pinned host buffers: pages land on the node
    of the allocating CPU, so the thread runs on the GPU's own NUMA node while
    inside (its affinity is restored on exit).  Yields that node or None."""
    import contextlib

    @contextlib.contextmanager
    def ctx():
        found = gpu_numa_cpus(device_index) if numa else None
        if not found or not found[1]:
            yield None
            return
        before = os.sched_getaffinity(0)
        os.sched_setaffinity(0, found[1])
        try:
            yield found[0]
        finally:
            os.sched_setaffinity(0, before)
    return ctx()


def e2e_run(step: LayerStep, steps: int, chunks: int = 8, numa: bool = True):
    """The same step end to end through the public API with host buffers:
    every step copies its inputs from pinned host memory, runs the
    operators, and reads every result back, pipelined over token chunks on
    three streams (copy-in, compute, copy-out)."""
    import torch
    d, cfg, T = step.d, step.cfg, step.T
    in_keys = ["tokens", "x", "residual", "q", "k", "positions", "gate", "up"]
    out_keys = ["emb_out", "h", "y", "q", "k", "ffn_out"]
    if cfg.softmax_cols:
        in_keys += ["scores", "valid_len"]
        out_keys += ["probs"]
    in_keys = [k for k in in_keys if d.get(k) is not None]
    out_keys = [k for k in out_keys if d.get(k) is not None]
    with pinned_near_gpu(step.dev.index or 0, numa) as node:
        host_in = {k: torch.empty(d[k].shape, dtype=d[k].dtype, pin_memory=True)
                   for k in in_keys}
        host_out = {k: torch.empty(d[k].shape, dtype=d[k].dtype, pin_memory=True)
                    for k in out_keys}
        for k in in_keys:
            host_in[k].copy_(d[k])
    step.e2e_numa_node = node
    h2d = sum(t.numel() * t.element_size() for t in host_in.values())
    d2h = sum(t.numel() * t.element_size() for t in host_out.values())
    s_in, s_cmp, s_out = (torch.cuda.Stream() for _ in range(3))
    bounds = [wl.shard_range(T, chunks, c) for c in range(chunks)]

    def rows_of(key, r0, r1):
        if key in ("scores", "valid_len", "probs"):
            return None  # head-major rows: copied whole with the last chunk
        return slice(r0, r1)

    # a chunk's inputs of the next step overwrite its buffers (q / k in
    # place) only once the previous step has read that chunk back: per-chunk
    # events, so the next step's uploads overlap this step's readback
    prev_out = [None] * chunks
    whole = any(rows_of(k, 0, 1) is None for k in in_keys + out_keys)

    def one_step():
        done_in = []
        for c, (r0, r1) in enumerate(bounds):
            if prev_out[c] is not None:
                s_in.wait_event(prev_out[-1] if whole and c == 0 else prev_out[c])
            with torch.cuda.stream(s_in):
                for k in in_keys:
                    sl = rows_of(k, r0, r1)
                    if sl is None:
                        if c == 0:
                            d[k].copy_(host_in[k], non_blocking=True)
                        continue
                    d[k][sl].copy_(host_in[k][sl], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(s_in)
                done_in.append(ev)
        done_cmp = []
        for c, (r0, r1) in enumerate(bounds):
            s_cmp.wait_event(done_in[c])
            for op in step.ops:
                step.launch(op, stream=s_cmp, rows=(r0, r1))
            ev = torch.cuda.Event()
            ev.record(s_cmp)
            done_cmp.append(ev)
        for c, (r0, r1) in enumerate(bounds):
            s_out.wait_event(done_cmp[c])
            with torch.cuda.stream(s_out):
                for k in out_keys:
                    sl = rows_of(k, r0, r1)
                    if sl is None:
                        if c == chunks - 1:
                            host_out[k].copy_(d[k], non_blocking=True)
                        continue
                    host_out[k][sl].copy_(d[k][sl], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(s_out)
                prev_out[c] = ev
        # (the next step's compute of a chunk waits for its uploads, which
        # wait for this step's readback of the chunk)

    for _ in range(2):
        one_step()
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record(s_in)
    for _ in range(steps):
        one_step()
    s_out.wait_stream(s_in)
    end.record(s_out)
    torch.cuda.synchronize()
    ms = start.elapsed_time(end) / steps
    return ms, h2d, d2h


GRAPH_REPEAT = 10


def rotation_timing(steps, args, world):
    """Steps whose working set is under 2 x L2: `steps` holds independent
    copies of the step's inputs (3 x L2 in all), and one CUDA graph runs one
    step on each copy in turn, so every step reads data that the steps
    since its last turn have evicted from L2, while the launches pipeline as
    they do in a model.  The graph is replayed back to back; per-operator
    times come from graphs of that operator over every copy.  Returns total
    ms over args.steps steps, per-op ms, and the clock sampler."""
    import torch
    import torch.distributed as dist
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())

    def capture(fn):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            fn()  # warm the capture stream once outside the graph
            torch.cuda.synchronize()
            with torch.cuda.graph(g, stream=stream):
                fn()
        return g

    def all_steps():
        for st in steps:
            st.step()

    copies = len(steps)
    step_graph = capture(all_steps)
    op_graphs = [capture(lambda op=op: [st.launch(op) for st in steps]) for op in steps[0].ops]
    replays = max(1, (args.steps + copies - 1) // copies)
    for g in [step_graph] + op_graphs:
        g.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(torch.cuda.current_device())
    with sampler:
        start.record()
        for _ in range(replays):
            step_graph.replay()
        end.record()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
    total_ms = start.elapsed_time(end) * args.steps / (replays * copies)
    op_ms = []
    for g in op_graphs:
        s0 = torch.cuda.Event(enable_timing=True)
        s1 = torch.cuda.Event(enable_timing=True)
        s0.record()
        for _ in range(replays):
            g.replay()
        s1.record()
        torch.cuda.synchronize()
        op_ms.append(s0.elapsed_time(s1) / (replays * copies))
    del step_graph, op_graphs
    return total_ms, op_ms, sampler


def graph_timing(step: LayerStep, args, world):
    """Steps whose launches the host could not enqueue as fast as the GPU runs
    them: GRAPH_REPEAT steps are captured in one CUDA graph and replayed back
    to back (the step's working set is at least 2 x L2, so no step reads the
    previous one's data from L2).  Per-operator times come from a graph of
    GRAPH_REPEAT launches of that operator alone, replayed back to back (an
    operator whose own bytes are under 2 x L2 then reads them from L2: the
    JSON line marks those).  Returns total ms over args.steps steps, per-op
    ms, and the clock sampler."""
    import torch
    import torch.distributed as dist
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())

    def capture(fn):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            fn()  # warm the capture stream once outside the graph
            torch.cuda.synchronize()
            with torch.cuda.graph(g, stream=stream):
                for _ in range(GRAPH_REPEAT):
                    fn()
        return g

    step_graph = capture(step.step)
    op_graphs = {op: capture(lambda op=op: step.launch(op)) for op in step.ops}
    replays = max(1, args.steps // GRAPH_REPEAT)
    for g in [step_graph] + list(op_graphs.values()):
        g.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(torch.cuda.current_device())
    with sampler:
        start.record()
        for _ in range(replays):
            step_graph.replay()
        end.record()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
    total_ms = start.elapsed_time(end) * args.steps / (replays * GRAPH_REPEAT)
    op_ms = []
    for op in step.ops:
        s0 = torch.cuda.Event(enable_timing=True)
        s1 = torch.cuda.Event(enable_timing=True)
        s0.record()
        for _ in range(replays):
            op_graphs[op].replay()
        s1.record()
        torch.cuda.synchronize()
        op_ms.append(s0.elapsed_time(s1) / (replays * GRAPH_REPEAT))
    del step_graph, op_graphs
    return total_ms, op_ms, sampler


# ---------------------------------------------------------------- CPU legs

class CpuLayerSample:
    """A bounded sample of the workload's token rows on the host, run through
    the reference's own CPU operators (oracle/_ref, kind "reference") or, if
    that library is absent, through the C restatement over a thread pool
    (kind "port")."""

    def __init__(self, cfg, rows: int, seed: int = 0):
        import numpy as np
        sys.path.insert(0, ORACLE_DIR)
        from oracle import REF_SO, Oracle, Reference
        self.np = np
        self.cfg = cfg
        self.rows = rows
        rng = np.random.default_rng(seed)
        H, F, hd = cfg.hidden, cfg.ffn, cfg.head_dim
        self.table = wl.numpy_quant_table(cfg.qtype, cfg.vocab, H, seed)
        self.tokens = rng.integers(0, cfg.vocab, rows).astype(np.int32)
        self.x = rng.standard_normal((rows, H), dtype=np.float32)
        self.r = rng.standard_normal((rows, H), dtype=np.float32)
        self.w = (rng.standard_normal(H, dtype=np.float32) * 0.1 + 1).astype(np.float32)
        self.q = rng.standard_normal((rows, cfg.n_heads, hd), dtype=np.float32)
        self.k = rng.standard_normal((rows, cfg.n_kv_heads, hd), dtype=np.float32)
        self.pos = np.linspace(0, cfg.max_position(), rows).astype(np.int32)
        self.g = rng.standard_normal((rows, F), dtype=np.float32)
        self.u = rng.standard_normal((rows, F), dtype=np.float32)
        self.bq = (rng.standard_normal(cfg.n_heads * hd, dtype=np.float32) * 0.02
                   if cfg.bias else None)
        self.bk = (rng.standard_normal(cfg.n_kv_heads * hd, dtype=np.float32) * 0.02
                   if cfg.bias else None)
        self.emb_out = np.empty((rows, H), np.float32)
        if os.path.exists(REF_SO):
            self.kind = "reference"
            self.ref = Reference()
            lib = self.ref.lib
            lib.mlref_set_thread_count(0)
            self.cores = lib.mlref_thread_count()
            P = lambda a: None if a is None else a.ctypes.data_as(__import__("ctypes").c_void_p)
            self._P = P
            self.h_table = lib.mlref_table_new(P(self.table), cfg.qtype, cfg.vocab, H)
            self.h_x = lib.mlref_rows_new(P(self.x), rows, H)
            self.h_r = lib.mlref_rows_new(P(self.r), rows, H)
            self.h_w = lib.mlref_rows_new(P(self.w), 1, H)
            self.h_q = lib.mlref_heads_new(P(self.q), rows, cfg.n_heads, hd)
            self.h_k = lib.mlref_heads_new(P(self.k), rows, cfg.n_kv_heads, hd)
            self.h_g = lib.mlref_rows_new(P(self.g), rows, F)
            self.h_u = lib.mlref_rows_new(P(self.u), rows, F)
        else:
            from concurrent.futures import ThreadPoolExecutor
            self.kind = "port"
            self.orc = Oracle()
            self.cores = os.cpu_count() or 1
            self.pool = ThreadPoolExecutor(self.cores)

    def step(self):
        cfg = self.cfg
        if self.kind == "reference":
            lib, P = self.ref.lib, self._P
            lib.mlref_bench_embedding(self.h_table, P(self.tokens), self.rows,
                                      P(self.emb_out))
            lib.mlref_bench_rmsnorm(self.h_x, self.h_r if cfg.residual else None,
                                    self.h_w, cfg.eps)
            lib.mlref_bench_rope(self.h_q, self.h_k, P(self.bq), P(self.bk),
                                 P(self.pos), cfg.theta, int(cfg.neox))
            lib.mlref_bench_swiglu(self.h_g, self.h_u)
            return
        n = self.cores
        parts = [wl.shard_range(self.rows, n, i) for i in range(n)]
        orc = self.orc

        def work(a, b):
            if b <= a:
                return
            orc.embedding(self.table, cfg.qtype, cfg.vocab, cfg.hidden,
                          self.tokens[a:b])
            orc.rmsnorm(self.x[a:b], self.w, cfg.eps,
                        residual=self.r[a:b] if cfg.residual else None)
            orc.rope(self.q[a:b], self.k[a:b], self.pos[a:b], cfg.theta,
                     int(cfg.neox), self.bq, self.bk)
            orc.swiglu(self.g[a:b], self.u[a:b])
        list(self.pool.map(lambda ab: work(*ab), parts))


def cpu_sample_rows(cfg, budget_s: float, steps: int):
    """Rows per step so that `steps` CPU steps take about `budget_s`."""
    probe = CpuLayerSample(cfg, 256)
    probe.step()
    t0 = time.perf_counter()
    probe.step()
    per_row = (time.perf_counter() - t0) / 256
    rows = int(budget_s / max(steps, 1) / max(per_row, 1e-9))
    return max(64, min(cfg.tokens, rows)), probe.kind


def run_cpu(cfg, steps: int, warmup: int, budget_s: float):
    rows, _ = cpu_sample_rows(cfg, budget_s, steps)
    sample = CpuLayerSample(cfg, rows)
    for _ in range(warmup):
        sample.step()
    per_step = []
    t0 = time.perf_counter()
    for _ in range(steps):
        t1 = time.perf_counter()
        sample.step()
        per_step.append(time.perf_counter() - t1)
    sec = (time.perf_counter() - t0) / steps
    rates = sorted(rows / s for s in per_step)
    ops_bytes = (cfg.bytes_embedding(rows) + cfg.bytes_rmsnorm(rows) +
                 cfg.bytes_rope(rows) + cfg.bytes_swiglu(rows))
    return {"tokens_per_s": rows / sec, "gbs": ops_bytes / sec / 1e9,
            "rows": rows, "sec_per_step": sec, "kind": sample.kind,
            "cores": sample.cores, "steps": steps, "warmup": warmup,
            "spread": {"min": round(rates[0], 1),
                       "median": round(statistics.median(rates), 1),
                       "max": round(rates[-1], 1)}}


def reference_arm(args, cfg):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    warm = max(1, args.warmup)
    res = run_cpu(cfg, args.steps, warm, budget_s=args.cpu_budget)
    sample = (f"{res['rows']} of {cfg.tokens} token rows of {cfg.name} per step "
              f"(embedding, {'residual ' if cfg.residual else ''}RMSNorm, RoPE, "
              f"SwiGLU), reference ops called per row inside its ParallelFor")
    line = {
        "metric": METRIC, "impl": "reference",
        "value": round(res["tokens_per_s"], 1), "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": warm,
        "ms_per_step": round(res["sec_per_step"] * 1e3, 3),
        "higher_is_better": True, "scaling": "weak" if args.weak else "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config_block(cfg, args, cfg.tokens if args.weak else
                               wl.shard_range(cfg.tokens, max(1, args.gpus), 0)[1],
                               cfg.tokens * (max(1, args.gpus) if args.weak else 1)),
        "hbm_gbs_equiv": round(res["gbs"], 2),
        "cpu_baseline": {"value": round(res["tokens_per_s"], 1), "unit": "tokens/s",
                         "cores": res["cores"], "kind": res["kind"],
                         "sample": sample, "spread_tokens_per_s": res["spread"]},
        "e2e": {"value": round(res["tokens_per_s"], 1), "unit": "tokens/s",
                "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
    }
    print(json.dumps(line), flush=True)


def config_block(cfg, args, tokens_per_gpu, global_tokens):
    return {
        "workload": cfg.name, "tokens_per_gpu": tokens_per_gpu,
        "global_tokens": global_tokens, "hidden": cfg.hidden,
        "ffn": cfg.ffn, "heads": cfg.n_heads, "kv_heads": cfg.n_kv_heads,
        "head_dim": cfg.head_dim, "rope": "neox" if cfg.neox else "normal",
        "rope_theta": cfg.theta, "qk_bias": cfg.bias,
        "residual_rmsnorm": cfg.residual, "eps": cfg.eps,
        "embedding": f"{wl.QNAME[cfg.qtype]} [{cfg.vocab}, {cfg.hidden}]",
        "parallelism": f"token-range shards x{args.gpus}, replicated weights, "
                       "no collective",
        "l2": "inputs larger than L2 (126 MB); no flush",
    }


def l2_note(step_bytes: int) -> str:
    if step_bytes < 2 * L2_BYTES:
        copies = -(-3 * L2_BYTES // step_bytes)
        return (f"inputs larger than L2: {copies} copies of the step's "
                f"{step_bytes / 1e6:.1f} MB working set ({copies * step_bytes / 1e6:.0f} MB "
                "in all), one step on each in turn; no flush")
    return "inputs larger than L2 (126 MB); no flush"


# ---------------------------------------------------------------- copy bound

def copy_bandwidth(args):
    """Pinned host <-> device copy bandwidth of the box, the bound of the
    e2e number: every rank copies `COPY_BYTES` from pinned host memory on its
    GPU's NUMA node to the device (h2d), back (d2h), and both at once on two
    streams; times are device events, max over ranks after a common barrier.
    Prints one JSON line with the aggregate GB/s over all ranks."""
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
    n = COPY_BYTES
    with pinned_near_gpu(local, True) as node:
        h_in = torch.empty(n, dtype=torch.uint8, pin_memory=True)
        h_out = torch.empty(n, dtype=torch.uint8, pin_memory=True)
        h_in.fill_(1)
    d_in = torch.empty(n, dtype=torch.uint8, device=dev)
    d_out = torch.zeros(n, dtype=torch.uint8, device=dev)
    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()

    def timed(kind):
        for _ in range(2):  # warm-up, then the timed pass
            if world > 1:
                dist.barrier()
            torch.cuda.synchronize()
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
            if kind in ("h2d", "both"):
                ev[0].record(s_in)
                with torch.cuda.stream(s_in):
                    d_in.copy_(h_in, non_blocking=True)
                ev[1].record(s_in)
            if kind in ("d2h", "both"):
                ev[2].record(s_out)
                with torch.cuda.stream(s_out):
                    h_out.copy_(d_out, non_blocking=True)
                ev[3].record(s_out)
            torch.cuda.synchronize()
        ms = []
        if kind in ("h2d", "both"):
            ms.append(ev[0].elapsed_time(ev[1]))
        if kind in ("d2h", "both"):
            ms.append(ev[2].elapsed_time(ev[3]))
        return max(ms)

    res = torch.tensor([timed(k) for k in ("h2d", "d2h", "both")],
                       dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(res, op=dist.ReduceOp.MAX)
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    h2d_ms, d2h_ms, both_ms = res.cpu().tolist()
    gb = n / 1e9
    print(json.dumps({
        "copy_bandwidth": True, "n_gpus": world, "bytes_per_gpu_per_direction": n,
        "pinned_numa_node_rank0": node,
        "h2d_gbs_aggregate": round(world * gb / (h2d_ms / 1e3), 1),
        "d2h_gbs_aggregate": round(world * gb / (d2h_ms / 1e3), 1),
        "both_directions_gbs_aggregate": round(2 * world * gb / (both_ms / 1e3), 1),
        "h2d_gbs_per_gpu": round(gb / (h2d_ms / 1e3), 1),
        "d2h_gbs_per_gpu": round(gb / (d2h_ms / 1e3), 1)}), flush=True)


COPY_BYTES = 512 << 20


# ---------------------------------------------------------------- main

def gpu_arm(args, cfg):
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        args.gpus = world
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
    # strong scaling (default): one batch of cfg.tokens rows — a sequence at
    # positions 0..T-1 — split into contiguous token ranges, one per rank;
    # --weak gives every rank its own block of cfg.tokens rows.
    total_tokens = args.tokens or cfg.tokens
    if args.weak:
        tokens, pos_offset = total_tokens, 0
    else:
        r0, r1 = wl.shard_range(total_tokens, world, rank)
        tokens, pos_offset = r1 - r0, r0
    ops = args.ops.split(",") if args.ops else None
    step = LayerStep(cfg, dev, tokens, pos_offset, ops)
    nops = len(step.ops)
    op_bytes = step.bytes()
    # CUDA-graph replay where the host could not enqueue a step's launches
    # faster than the GPU runs them (measured: 4096 rows per GPU over 4 ranks
    # spent a quarter of each step waiting on the host with direct launches)
    use_graph = args.graph == "on" or (args.graph == "auto" and (tokens <= 4096 or world > 1))
    # a working set under 2 x L2 would be read from L2 by back-to-back steps:
    # such steps rotate over independent copies of their inputs (3 x L2 in
    # all, each copy from its own seed)
    cold = sum(op_bytes.values()) < 2 * L2_BYTES
    steps = [step]
    if cold:
        copies = -(-3 * L2_BYTES // sum(op_bytes.values()))
        steps += [LayerStep(dataclasses.replace(cfg, seed=cfg.seed + 1000 * c), dev, tokens,
                            pos_offset, ops) for c in range(1, copies)]
    direct = not cold and not use_graph
    if direct:
        # NVML set-up (slow) and the events before the warm-up, so that the
        # warm-up steps lead straight into the timed ones with no idle gap
        events = [[torch.cuda.Event(enable_timing=True) for _ in range(nops + 1)]
                  for _ in range(args.steps)]
        sampler = ClockSampler(local)
        if world > 1:
            dist.barrier()
    for _ in range(args.warmup):
        for st in steps:
            st.step()
    torch.cuda.synchronize()
    if cold:
        total_ms, op_ms, sampler = rotation_timing(steps, args, world)
    elif use_graph:
        total_ms, op_ms, sampler = graph_timing(step, args, world)
    else:
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        with sampler:
            for i in range(args.steps):
                step.step(events[i])
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
        total_ms = events[0][0].elapsed_time(events[-1][nops])
        op_ms = [sum(events[i][j].elapsed_time(events[i][j + 1])
                     for i in range(args.steps)) / args.steps for j in range(nops)]
    bits = torch.zeros(1, dtype=torch.int32)
    bits.copy_(step.d["status"])
    if int(bits.item()) != 0:
        raise RuntimeError(f"device status raised: {int(bits.item())}")
    if args.no_e2e:
        e2e_ms, h2d, d2h = float("nan"), 0, 0
    else:
        e2e_ms, h2d, d2h = e2e_run(step, args.e2e_steps, chunks=args.e2e_chunks,
                                   numa=bool(args.e2e_numa))
    stats = torch.tensor([total_ms, e2e_ms] + op_ms, dtype=torch.float64,
                         device=dev)
    if world > 1:
        dist.all_reduce(stats, op=dist.ReduceOp.MAX)
    stats = stats.cpu().tolist()
    total_ms, e2e_ms, op_ms = stats[0], stats[1], stats[2:]
    clocks = sampler.summary()
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and ops is None:
        # the same steps, warm-up and time budget as the reference arm
        # (`--impl reference`), so both sample the same rows per step
        cpu = run_cpu(cfg, args.steps, max(1, args.warmup), budget_s=args.cpu_budget)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    ms_step = total_ms / args.steps
    tokens_all = tokens * world if args.weak else total_tokens
    value = tokens_all / (ms_step / 1e3)
    step_bytes = sum(op_bytes.values())
    peak, peak_kind = measured_peak()
    gbs_per_gpu = step_bytes / (ms_step / 1e3) / 1e9
    ops = {}
    for j, op in enumerate(step.ops):
        g = op_bytes[op] / (op_ms[j] / 1e3) / 1e9
        ops[op] = {"ms": round(op_ms[j], 4), "gbs": round(g, 1),
                   "frac_of_measured": round(g / peak, 4),
                   "frac_of_8tbs": round(g / SPEC_HBM_GBS, 4),
                   "bytes": op_bytes[op]}
    dom = max(step.ops, key=lambda o: op_bytes[o])
    j = step.ops.index(dom)
    achieved = op_bytes[dom] / (op_ms[j] / 1e3) / 1e9
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms_step, 4), "higher_is_better": True,
        "scaling": "weak" if args.weak else "strong", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic",
        "config": dict(config_block(cfg, args, tokens, tokens_all),
                       l2=l2_note(step_bytes)),
        "hbm_gbs": round(gbs_per_gpu * world, 1),
        "hbm_gbs_per_gpu": round(gbs_per_gpu, 1),
        "hbm_frac_of_measured": round(gbs_per_gpu / peak, 4),
        "hbm_frac_of_8tbs": round(gbs_per_gpu / SPEC_HBM_GBS, 4),
        "ops": ops,
        "roofline": {"kernel": dom, "bound": "hbm", "achieved": round(achieved, 1),
                     "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                     "frac": round(achieved / peak, 4),
                     "traffic": profile_traffic(dom, cfg.name),
                     "algorithmic_bytes": op_bytes[dom]},
        "clocks": clocks,
        "e2e": None if args.no_e2e else {
            "value": round(tokens_all / (e2e_ms / 1e3), 1), "unit": "tokens/s",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "steps": args.e2e_steps, "chunks": args.e2e_chunks,
            "ms_per_step": round(e2e_ms, 3),
            "pinned_numa_node": getattr(step, "e2e_numa_node", None)},
        "timing": ("cuda graph replay over rotating input copies" if cold
                   else "cuda graph replay" if use_graph else "direct launches"),
        "launch_overlap": args.launch_overlap,
        "gpu_launches": args.steps * len(step.ops),
    }
    if cpu is not None:
        line["cpu_baseline"] = {
            "value": round(cpu["tokens_per_s"], 1), "unit": "tokens/s",
            "cores": cpu["cores"], "kind": cpu["kind"],
            "sample": f"{cpu['rows']} of {cfg.tokens} token rows per step, "
                      f"{cpu['steps']} steps after {cpu['warmup']} warm-up",
            "spread_tokens_per_s": cpu["spread"]}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- linear

LINEAR_SHAPES = ((14336, 4096), (4096, 14336), (4864, 896), (896, 4864))


LINEAR_TC_MIN_TOKENS = 48   # mlb_linear_rows_f32 runs on the tensor cores from here
TF32_DENSE_TFLOPS = 1100.0  # B200 nominal dense TF32 (no measured figure in the pool file)


def measured_tensor_peak():
    """Measured dense bf16 TFLOP/s of this pool's B200s (burst; fp16 runs at the
    same rate), or None."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops"])
    except (OSError, KeyError, ValueError):
        return None


def linear_bench(args):
    """Decode-path linear layer (mlb_linear_f32): one JSON line per
    (format, n, k, tokens) — LLaMA-3-8B FFN gate/up [14336, 4096] and down
    [4096, 14336], Qwen2-0.5B FFN [4864, 896] / [896, 4864] — with GB/s over
    the weight bytes + activations, timed cold (L2 flushed) when the weights
    fit in L2."""
    import torch
    import mlb
    dev = torch.device("cuda", 0)
    peak, peak_kind = measured_peak()
    g = torch.Generator(device=dev)
    g.manual_seed(1)
    qts = [wl.QTYPE_BY_NAME[q] for q in args.linear_qtypes.split(",")] \
        if args.linear_qtypes else (wl.Q8_0, wl.Q4_0, wl.Q4_1, wl.F32)
    shapes = [tuple(int(v) for v in sh.split("x")) for sh in args.linear_shapes.split(",")] \
        if args.linear_shapes else LINEAR_SHAPES
    tokens = [int(t) for t in args.linear_tokens.split(",")] \
        if args.linear_tokens else (1, 4, 8)
    mlb.set_gemv_path(args.gemv_path)
    path_name = {0: "gemv", 1: "gemv cuda-core", 2: "gemv int8 tensor-core"}[args.gemv_path]
    for qt in qts:
        for n, k in shapes:
            w = wl.quant_table(qt, n, k, dev, seed=1)
            # decode-sized calls on weights under 2 x L2: one call per
            # independent weight copy (3 x L2 in all) in a CUDA graph, as the
            # linears of a decode step run (CUDA events tick in 0.512 us)
            wbytes = n * wl.row_bytes(qt, k)
            copies = max(2, -(-3 * L2_BYTES // wbytes)) if wbytes < 2 * L2_BYTES else 1
            ws = [w] + [wl.quant_table(qt, n, k, dev, seed=1 + c) for c in range(1, copies)]
            for t in tokens:
                x = torch.randn((t, k), generator=g, device=dev)
                y = torch.empty((t, n), device=dev)
                tc = t >= LINEAR_TC_MIN_TOKENS
                if tc:  # prompt-sized: the tensor-core entry, scratch preallocated
                    scratch = torch.empty(mlb.load().mlb_linear_rows_scratch_floats(k, t),
                                          device=dev)
                    fn = lambda: mlb.linear_rows(w, qt, n, k, x, out=y,  # noqa: E731
                                                 scratch=scratch)
                else:
                    fn = lambda: mlb.linear(w, qt, n, k, x, out=y)  # noqa: E731
                nbytes = n * wl.row_bytes(qt, k) + 4 * t * (k + n)
                single = None
                if not tc and copies > 1:
                    ms = rotated_call_ms([lambda wc=wc: mlb.linear(wc, qt, n, k, x, out=y)
                                          for wc in ws])
                    single = time_fn(fn, nbytes, 1)
                    timing = (f"CUDA graph of one call per weight copy ({copies} copies, "
                              "3 x L2), replayed back to back")
                else:
                    ms = time_fn(fn, nbytes, 1)
                    timing = "cold L2" if nbytes < 2 * L2_BYTES else "warm"
                gbs = nbytes / (ms / 1e3) / 1e9
                f16 = tc and qt in (wl.Q8_0, wl.Q4_0) and k % 64 == 0
                line = {
                    "linear": wl.QNAME[qt], "n": n, "k": k, "tokens": t,
                    "path": ("tcgen05 f16, d*q and x in 2 exact pieces" if f16 else
                             "tcgen05 tf32x3") if tc else path_name,
                    "us": round(ms * 1e3, 2), "gbs": round(gbs, 1),
                    "frac_of_measured": round(gbs / peak, 4),
                    "frac_of_8tbs": round(gbs / SPEC_HBM_GBS, 4),
                    "peak_kind": peak_kind, "timing": timing}
                if single is not None:
                    line["us_single_cold_launch"] = round(single * 1e3, 2)
                if f16:  # 3 fp16 products per multiply-add: against the measured bf16 peak
                    tflops = 3 * 2 * n * k * t / (ms / 1e3) / 1e12
                    peak_tf = measured_tensor_peak()
                    line.update({"f16_tflops": round(tflops, 1),
                                 "frac_of_tensor_peak": round(tflops / peak_tf, 4)
                                 if peak_tf else None,
                                 "fp32_equiv_tflops": round(tflops / 3, 1)})
                elif tc:  # 3 TF32 products per multiply-add: against the dense TF32 peak
                    tflops = 3 * 2 * n * k * t / (ms / 1e3) / 1e12
                    line.update({"tf32_tflops": round(tflops, 1),
                                 "frac_of_tf32_peak": round(tflops / TF32_DENSE_TFLOPS, 4),
                                 "fp32_equiv_tflops": round(tflops / 3, 1)})
                print(json.dumps(line), flush=True)
            del w, ws
            torch.cuda.empty_cache()


# ---------------------------------------------------------------- attention

ATTENTION_CASES = (  # (name, n_heads, n_kv_heads, head_dim, position)
    ("llama3-8b", 32, 8, 128, 2047), ("llama3-8b", 32, 8, 128, 16383),
    ("llama-7b", 32, 32, 128, 2047), ("qwen2-0.5b", 14, 2, 64, 4095),
    ("qwen2-7b", 28, 4, 128, 32767))


def attention_bench(args):
    """Decode attention (mlb_attention_decode_f32) of one token over one
    layer's cache: one JSON line per case, GB/s over K + V bytes read."""
    import torch
    import mlb
    dev = torch.device("cuda", 0)
    peak, peak_kind = measured_peak()
    g = torch.Generator(device=dev)
    g.manual_seed(1)
    for name, nh, nkv, hd, pos in ATTENTION_CASES:
        nbytes = 8 * (pos + 1) * nkv * hd + 8 * nh * hd
        # independent caches, 3 x L2 in all: each call reads what the others
        # evicted (CUDA events tick in 0.512 us steps, so single launches of
        # 15-50 us cannot show sub-microsecond changes)
        copies = max(2, -(-3 * L2_BYTES // nbytes))
        caches = [(torch.randn((pos + 1, nkv, hd), generator=g, device=dev),
                   torch.randn((pos + 1, nkv, hd), generator=g, device=dev))
                  for _ in range(copies)]
        q = torch.randn((nh, hd), generator=g, device=dev)
        out = torch.empty((nh, hd), device=dev)
        scratch = torch.empty(mlb.attention_scratch_floats(nh, nkv, hd, pos), device=dev)
        calls = [lambda kv=kv: mlb.attention_decode(q, kv[0], kv[1], pos, out=out,
                                                    scratch=scratch) for kv in caches]
        ms = rotated_call_ms(calls)
        single = time_fn(calls[0], nbytes, 1)
        gbs = nbytes / (ms / 1e3) / 1e9
        print(json.dumps({
            "attention": name, "heads": nh, "kv_heads": nkv, "head_dim": hd,
            "position": pos, "us": round(ms * 1e3, 2), "gbs": round(gbs, 1),
            "frac_of_measured": round(gbs / peak, 4), "peak_kind": peak_kind,
            "timing": f"CUDA graph of one call per cache copy ({copies} copies, "
                      "3 x L2), replayed back to back",
            "us_single_cold_launch": round(single * 1e3, 2)}), flush=True)
        del caches
        torch.cuda.empty_cache()
    attention_rows_bench(args)


def rotated_call_ms(calls, replays=8):
    """Device ms per call: `calls` (one per independent input copy) captured
    in one CUDA graph, replayed back to back after a warm-up replay."""
    import torch
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        for c in calls:
            c()  # warm the capture stream once outside the graph
        torch.cuda.synchronize()
        with torch.cuda.graph(graph, stream=stream):
            for c in calls:
                c()
    graph.replay()
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(replays):
        graph.replay()
    end.record()
    torch.cuda.synchronize()
    del graph
    return start.elapsed_time(end) / (replays * len(calls))


ATTENTION_ROWS_CASES = (  # (name, n_heads, n_kv_heads, head_dim, position, rows)
    ("llama3-8b", 32, 8, 128, 0, 512), ("llama3-8b", 32, 8, 128, 0, 2048),
    ("llama3-8b", 32, 8, 128, 2048, 2048), ("qwen2-7b", 28, 4, 128, 0, 2048),
    ("qwen2-0.5b", 14, 2, 64, 0, 2048))


def attention_rows_bench(args):
    """Causal attention of a prompt chunk (mlb_attention_rows_f32) on the
    CUDA-core kernels and on the tensor cores: one JSON line per (case,
    path), TFLOP/s over the fp32-equivalent flops of the causal products
    (2 x 2 x hd per visible (query head, key) pair)."""
    import torch
    import mlb
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev)
    g.manual_seed(2)
    cases = ATTENTION_ROWS_CASES
    if args.attention_rows:  # one Llama-3-8B case of that many rows from position 0
        cases = (("llama3-8b", 32, 8, 128, 0, args.attention_rows),)
    for name, nh, nkv, hd, pos, rows in cases:
        max_seq = pos + rows
        keys = torch.randn((max_seq, nkv, hd), generator=g, device=dev)
        values = torch.randn((max_seq, nkv, hd), generator=g, device=dev)
        q = torch.randn((rows, nh, hd), generator=g, device=dev)
        out = torch.empty((rows, nh, hd), device=dev)
        pairs = nh * (rows * pos + rows * (rows + 1) // 2)
        flops = 4.0 * hd * pairs
        for path in (1, 2):
            previous = mlb.set_attention_path(path)
            fn = lambda: mlb.attention_rows(q, keys, values, pos, out=out)  # noqa: E731
            ms = time_fn(fn, 1 << 40, 1)  # compute-bound: back-to-back launches
            mlb.set_attention_path(previous)
            print(json.dumps({
                "attention_rows": name, "heads": nh, "kv_heads": nkv, "head_dim": hd,
                "position": pos, "rows": rows,
                "path": "tensor cores (TF32 head + tail)" if path == 2 else "CUDA cores",
                "ms": round(ms, 4), "tflops_fp32_equiv": round(flops / (ms / 1e3) / 1e12, 1)}),
                flush=True)
        del keys, values, q, out
        torch.cuda.empty_cache()


# ---------------------------------------------------------------- prefill

PREFILL_EXE = os.path.join(ROOT, "mini-lla_b200", "host", "_build", "mlb_prefill_bench")


def prefill_bench(args):
    """Whole-model prefill and decode through the C++ layer's
    ForwardBatchCuda on a random-weight model of Llama-3-8B shape
    (--prefill-layers layers), beside the reference's per-token GPU driver
    and its CPU forward pass; one JSON line (the program's)."""
    if not os.path.exists(PREFILL_EXE):
        print(json.dumps({"prefill": "unavailable",
                          "why": "mlb_prefill_bench not built (needs the reference "
                                 "headers: make -C mini-lla_b200/host)"}))
        return
    cmd = [PREFILL_EXE, "--layers", str(args.prefill_layers), "--tokens",
           str(args.prefill_tokens), "--type", args.prefill_type,
           "--steps", str(max(1, min(args.steps, 10))), "--warmup", str(max(1, args.warmup)),
           "--max-rows", str(max(512, args.prefill_tokens)),
           "--overlap", str(args.launch_overlap)]
    if args.no_cpu_baseline:
        cmd += ["--cpu-tokens", "0"]
    res = subprocess.run(cmd, capture_output=True, text=True, timeout=1800)
    if res.returncode != 0:
        raise RuntimeError(f"mlb_prefill_bench failed: {res.stderr[-2000:]}")
    line = json.loads(res.stdout.strip().splitlines()[-1])
    line.update({"metric": "prefill tokens/s (ForwardBatchCuda, whole layers)",
                 "data": "synthetic random-weight model", "dtype": "f32 (ggml blocks)"})
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- sweep

SWEEP_OPS = ("rmsnorm", "res_rmsnorm", "swiglu", "emb_q8_0", "emb_q4_0", "emb_q4_1")


def sweep(args):
    """Bandwidth sweep: every operator (RMSNorm, residual RMSNorm, SwiGLU,
    Q8_0 / Q4_0 / Q4_1 gather) x hidden size {512 .. 16384} x token count
    {1 .. 262144}, seed 1, quant tables of 32000 rows; one JSON line per point with
    GB/s per GPU and the fractions of the measured and spec peaks.  Under
    torchrun a point's T rows are split into equal contiguous ranges, one per
    rank (points whose T is not a multiple of the rank count are skipped),
    and the slowest rank's time is reported; `--weak` runs the whole point on
    every rank instead."""
    import torch
    import torch.distributed as dist
    import mlb
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=dev)
    peak, peak_kind = measured_peak()
    ops = args.sweep_ops.split(",") if args.sweep_ops else SWEEP_OPS
    hiddens = [int(h) for h in args.sweep_hidden.split(",")] if args.sweep_hidden \
        else wl.SWEEP_HIDDEN
    tokens_list = [int(t) for t in args.sweep_tokens.split(",")] if args.sweep_tokens \
        else wl.SWEEP_TOKENS
    g = torch.Generator(device=dev)
    g.manual_seed(1)
    f32 = dict(device=dev, dtype=torch.float32)
    for op in ops:
        for H in hiddens:
            table = None
            if op.startswith("emb"):
                qt = {"emb_q8_0": wl.Q8_0, "emb_q4_0": wl.Q4_0,
                      "emb_q4_1": wl.Q4_1}[op]
                table = wl.quant_table(qt, wl.SWEEP_VOCAB, H, dev, seed=1)
            for T_point in tokens_list:
                if world > 1 and not args.weak and T_point % world != 0:
                    continue
                T = T_point if (world == 1 or args.weak) else T_point // world
                if op in ("rmsnorm", "res_rmsnorm"):
                    x = torch.randn((T, H), generator=g, **f32)
                    r = torch.randn((T, H), generator=g, **f32) \
                        if op == "res_rmsnorm" else None
                    w = torch.randn((H,), generator=g, **f32) * 0.1 + 1
                    h = torch.empty_like(x) if r is not None else None
                    y = torch.empty_like(x)
                    fn = lambda: mlb.rms_norm(x, w, 1e-5, residual=r, h_out=h, out=y)  # noqa: E731
                    nbytes = (16 if r is not None else 8) * T * H + 4 * H
                elif op == "swiglu":
                    a = torch.randn((T, H), generator=g, **f32)
                    b = torch.randn((T, H), generator=g, **f32)
                    o = torch.empty_like(a)
                    fn = lambda: mlb.swiglu(a, b, out=o)  # noqa: E731
                    nbytes = 12 * T * H
                else:
                    tok = torch.randint(0, wl.SWEEP_VOCAB, (T,), generator=g,
                                        device=dev, dtype=torch.int32)
                    o = torch.empty((T, H), **f32)
                    fn = lambda: mlb.embedding_rows(table, qt, wl.SWEEP_VOCAB, H, tok,  # noqa: E731
                                                    out=o)
                    nbytes = T * (wl.row_bytes(qt, H) + 4 * H + 4)
                ms = time_fn(fn, nbytes, world)
                if rank == 0:
                    gbs = nbytes / (ms / 1e3) / 1e9
                    print(json.dumps({
                        "sweep": op, "hidden": H, "tokens": T_point,
                        "tokens_per_gpu": T, "n_gpus": world,
                        "scaling": "weak" if args.weak else "strong",
                        "ms": round(ms, 5),
                        "tokens_per_s": round(T * world / (ms / 1e3), 1),
                        "gbs_per_gpu": round(gbs, 1),
                        "frac_of_measured": round(gbs / peak, 4),
                        "frac_of_8tbs": round(gbs / SPEC_HBM_GBS, 4),
                        "peak_kind": peak_kind}), flush=True)
                del fn
                torch.cuda.empty_cache()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


L2_BYTES = 126 * 1024 * 1024
_flush_buf = None


def time_fn(fn, nbytes, world):
    """Device time of one launch.  Working sets under 2 x L2 are timed cold:
    each launch sits alone between two events after a read of a 512 MiB
    buffer (evicting L2 with clean lines) and a ~0.5 ms device sleep (during
    which the host enqueues the launch, so the events bracket only the
    kernel), and the median of 21 launches is kept.  Larger
    ones are timed back to back (inputs larger than L2) over enough launches
    for ~20 ms of device time."""
    import torch
    import torch.distributed as dist
    global _flush_buf
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    if nbytes < 2 * L2_BYTES:
        if _flush_buf is None:
            _flush_buf = torch.ones(512 * 1024 * 1024 // 4, device="cuda")
        times = []
        for _ in range(21):
            # a read-only pass evicts the inputs and leaves only clean lines
            # (a write would leave dirty lines whose write-back would land in
            # the timed kernel)
            _flush_buf.sum()
            torch.cuda._sleep(1_000_000)  # the host enqueues the launch meanwhile
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize()
            times.append(e0.elapsed_time(e1))
        ms = statistics.median(times)
    else:
        reps = int(min(2000, max(5, 20.0 / (nbytes / 6.5e9))))
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / reps
    if world > 1:
        t = torch.tensor([ms], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="llama3-8b-t16384",
                    choices=sorted(wl.CONFIGS))
    ap.add_argument("--impl", default="mlb", choices=["mlb", "reference"])
    ap.add_argument("--weak", action="store_true",
                    help="every GPU runs its own T rows (default: the T rows "
                         "are split across the GPUs)")
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--e2e-chunks", type=int, default=8,
                    help="token chunks the e2e leg pipelines copies and compute over")
    ap.add_argument("--cpu-budget", type=float, default=20.0,
                    help="seconds of CPU work for the CPU legs")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--e2e-numa", type=int, default=1, choices=(0, 1),
                    help="1: allocate the pinned host buffers on the GPU's NUMA node")
    ap.add_argument("--ops", default="",
                    help="comma list: time only these operators of the step")
    ap.add_argument("--graph", default="auto", choices=["auto", "on", "off"],
                    help="replay the step from a CUDA graph (auto: T <= 4096 rows per "
                         "GPU, or several GPUs)")
    ap.add_argument("--tokens", type=int, default=0,
                    help="token rows per step instead of the workload's T")
    ap.add_argument("--sweep", action="store_true",
                    help="bandwidth sweep: one JSON line per (op, H, T) point")
    ap.add_argument("--linear", action="store_true",
                    help="decode-path linear layer: one JSON line per shape")
    ap.add_argument("--attention", action="store_true",
                    help="decode attention: one JSON line per case")
    ap.add_argument("--attention-rows", type=int, default=0,
                    help="prompt attention only: one Llama-3-8B chunk of this many "
                         "rows, CUDA cores then tensor cores")
    ap.add_argument("--prefill", action="store_true",
                    help="whole-model prefill / decode through ForwardBatchCuda")
    ap.add_argument("--prefill-layers", type=int, default=4)
    ap.add_argument("--prefill-tokens", type=int, default=512)
    ap.add_argument("--prefill-type", default="Q8_0")
    ap.add_argument("--linear-qtypes", default="", help="e.g. Q8_0,F32")
    ap.add_argument("--linear-shapes", default="", help="e.g. 14336x4096")
    ap.add_argument("--linear-tokens", default="", help="e.g. 1,4")
    ap.add_argument("--gemv-path", type=int, default=0, choices=(0, 1, 2),
                    help="decode linear kernel: 0 automatic, 1 CUDA-core GEMV, "
                         "2 int8 tensor-core GEMV where allowed")
    ap.add_argument("--launch-overlap", type=int, default=1, choices=(0, 1),
                    help="1: programmatic dependent launch between kernels (the "
                         "library's default), 0: plain stream order")
    ap.add_argument("--copy-bw", action="store_true",
                    help="pinned host <-> device copy bandwidth (the e2e bound)")
    ap.add_argument("--sweep-ops", default="")
    ap.add_argument("--sweep-hidden", default="")
    ap.add_argument("--sweep-tokens", default="")
    args = ap.parse_args()
    cfg = wl.CONFIGS[args.workload]
    if args.impl != "reference" and not args.prefill:
        import mlb
        mlb.set_launch_overlap(args.launch_overlap)
    if args.copy_bw:
        copy_bandwidth(args)
        return
    if args.sweep:
        sweep(args)
        return
    if args.linear:
        linear_bench(args)
        return
    if args.attention_rows:
        attention_rows_bench(args)
        return
    if args.attention:
        attention_bench(args)
        return
    if args.prefill:
        prefill_bench(args)
        return
    if args.impl == "reference":
        reference_arm(args, cfg)
    else:
        gpu_arm(args, cfg)


if __name__ == "__main__":
    main()
