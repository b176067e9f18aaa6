#!/usr/bin/env python
"""Benchmark: QPS at recall@10 = 0.95 and build Mvec/s, 1M x 128 fp16 (config 2).

Workload (synthetic stand-in for BIGANN): 1,000,000 x 128
SIFT-like integer rows (Gaussian mixture, seed 2), 10,000 queries from the
same mixture (seed 3), L2, R = 64, alpha = 1.2, k = 10.  The graph is built
with jasper_b200 (timed: build Mvec/s), exact ground truth comes from a GPU
brute force, recall is swept over beam widths 16..256 (limit = 2 x bw), and
the two widths bracketing recall 0.95 are timed.  A "step" is one search of
all queries at each of the two bracketing widths; QPS@0.95 is interpolated
log-linearly between them (the reference's protocol).

`value` times the search kernel with inputs resident in HBM (CUDA events on
the launch stream, L2 flushed between steps); `e2e` times the C-ABI call
with host buffers (jb_graph_search_host: H2D queries, search, D2H results).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

With N > 1 (torchrun, one rank per GPU) each rank builds and searches its own
1M-row shard with its own 10,000 queries (weak scaling: per-GPU work fixed,
no data-path collective); times are the max over ranks.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import math
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

BWS = (16, 32, 64, 128, 256)
# DRAM bytes (read + write) of one search launch, from an ncu capture of this
# bench's own launch: (rows, queries, beam width) -> bytes.
SEARCH_TRAFFIC = {(1_000_000, 10_000, 32): 1_374_990_640}
TARGET = 0.95
K = 10
METRIC = "QPS at recall@10=0.95 and build Mvec/s, 1M×128 fp16, at 1/2/4/8 B200"


# ── helpers ───────────────────────────────────────────────────────────────
def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d.get("hbm_gbs", 6650.0)), "measured"
    return 6650.0, "fallback"


_SAMPLER_SRC = r"""
import sys, time, pynvml
pynvml.nvmlInit()
try:
    h = pynvml.nvmlDeviceGetHandleByPciBusId(sys.argv[1])
except Exception:
    h = pynvml.nvmlDeviceGetHandleByIndex(int(sys.argv[2]))
print("max", pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM), flush=True)
period = float(sys.argv[3])
while True:
    try:
        print(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM),
              pynvml.nvmlDeviceGetCurrentClocksEventReasons(h), flush=True)
    except Exception:
        pass
    time.sleep(period)
"""


class ClockSampler:
    """SM clock and clock-event reasons sampled through NVML every ~2 ms by a
    separate process while the timed region runs (a thread in this process
    would compete for the GIL with host-timed loops).  NVML reads only; no
    setting of the GPU is touched."""

    REASONS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
               "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80}

    def __init__(self, device: torch.device, period_s: float = 0.002):
        self.device = device
        self.period = period_s
        self.samples: list[tuple[int, int]] = []
        self.max_mhz = None
        self.proc = None
        self.t = None

    def _read(self):
        for line in self.proc.stdout:
            p = line.split()
            try:
                if p[0] == "max":
                    self.max_mhz = int(p[1])
                else:
                    self.samples.append((int(p[0]), int(p[1])))
            except (ValueError, IndexError):
                pass

    def __enter__(self):
        try:
            props = torch.cuda.get_device_properties(self.device)
            bus = f"{props.pci_domain_id:08X}:{props.pci_bus_id:02X}:{props.pci_device_id:02X}.0"
            self.proc = subprocess.Popen(
                [sys.executable, "-c", _SAMPLER_SRC, bus, str(self.device.index or 0),
                 str(self.period)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            t0 = time.perf_counter()
            while not self.samples and time.perf_counter() - t0 < 5.0:   # sampler running
                time.sleep(0.01)
            self.samples.clear()   # keep only samples taken inside the timed region
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self.t is not None:
            self.t.join(timeout=1.0)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unsampled"]}
        mhz = [m for m, _ in self.samples]
        active = 0
        for _, r in self.samples:
            active |= r
        reasons = sorted(k for k, bit in self.REASONS.items() if active & bit)
        return {"sm_mhz": float(np.median(mhz)), "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(mhz), "sm_mhz_min": int(min(mhz)), "source": "nvml"}


def flush_l2(buf: torch.Tensor):
    buf.add_(1)  # 256 MB write, larger than the 126 MB L2


def exact_gt(base: torch.Tensor, queries: torch.Tensor, k: int) -> torch.Tensor:
    """Exact L2 top-k on the GPU in fp32 (integer rows: every distance exact)."""
    torch.backends.cuda.matmul.allow_tf32 = False
    b = base.float()
    bn = (b * b).sum(1)
    out = []
    for q0 in range(0, queries.size(0), 1000):
        q = queries[q0:q0 + 1000].float()
        d = (q * q).sum(1, keepdim=True) + bn[None, :] - 2.0 * (q @ b.T)
        out.append(d.topk(k, dim=1, largest=False).indices.int())
    return torch.cat(out)


def recall_at_k(res: torch.Tensor, gt: torch.Tensor) -> float:
    r = res.long()
    g = gt.long()
    hit = (r[:, :, None] == g[:, None, :]).any(-1).sum().item()
    return hit / (g.size(0) * g.size(1))


def bracket(recalls: dict[int, float]):
    bws = sorted(recalls)
    for lo, hi in zip(bws, bws[1:]):
        if recalls[lo] < TARGET <= recalls[hi]:
            return lo, hi
    if recalls[bws[0]] >= TARGET:
        return bws[0], bws[0]
    return bws[-1], bws[-1]


def interp_qps(r_lo, q_lo, r_hi, q_hi):
    if r_hi == r_lo:
        return q_hi
    t = (TARGET - r_lo) / (r_hi - r_lo)
    return math.exp(math.log(q_lo) + t * (math.log(q_hi) - math.log(q_lo)))


def load_data(n_base, n_q, rank=0):
    """Config-2 rows for one GPU: rank 0 is config 2 itself (base seed 2,
    query seed 3); rank r builds its own shard from base seed 2 + 100 r with
    queries from the same mixture."""
    from jasper_b200 import synthetic
    bs, qs = 2 + 100 * rank, 3 + 100 * rank
    base = synthetic.sift_like(n_base, 128, bs)
    queries = synthetic.sift_like(n_q, 128, qs, center_seed=bs)
    return base, queries


# ── jasper_b200 arm ───────────────────────────────────────────────────────
def run_jasper(args):
    import jasper_b200 as jasper
    from jasper_b200 import _lib
    ws, rank, local = dist_env()
    dist = None
    if ws > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    dev = torch.device("cuda", torch.cuda.current_device())
    base_np, q_np = load_data(args.n, args.nq, rank)
    base = torch.from_numpy(base_np).to(dev)
    queries = torch.from_numpy(q_np).to(dev)
    q_host = torch.from_numpy(q_np).pin_memory()

    # build (timed on the device)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    g = jasper.Graph.build(base, n_neighbors=64, distance="l2", alpha=1.2)
    torch.cuda.synchronize()
    build_s = time.perf_counter() - t0

    gt = exact_gt(base, queries, K)
    recalls = {}
    for bw in BWS:
        ids, _ = g.search(queries, k=K, beam_width=bw)
        recalls[bw] = recall_at_k(ids, gt)
    lo, hi = bracket(recalls)
    if dist is not None:
        t = torch.tensor([lo, hi], device=dev)
        dist.broadcast(t, 0)
        lo, hi = int(t[0]), int(t[1])
    pair = (lo, hi) if lo != hi else (hi,)

    flush = torch.zeros(64 * 1024 * 1024, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream()

    def step(times):
        for bw in pair:
            flush_l2(flush)
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            g.search(queries, k=K, beam_width=bw)
            e1.record(stream)
            times[bw].append((e0, e1))

    warm = {bw: [] for bw in pair}
    for _ in range(args.warmup):
        step(warm)
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    times = {bw: [] for bw in pair}
    with ClockSampler(dev) as clk:
        t0 = time.perf_counter()
        for _ in range(args.steps):
            step(times)
        torch.cuda.synchronize()
        wall = time.perf_counter() - t0
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    ms = {bw: sum(a.elapsed_time(b) for a, b in times[bw]) / args.steps for bw in pair}
    total_ms = sum(ms.values())
    if dist is not None:
        t = torch.tensor([ms[bw] for bw in pair] + [total_ms, build_s], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        vals = t.tolist()
        ms = {bw: vals[i] for i, bw in enumerate(pair)}
        total_ms, build_s = vals[-2], vals[-1]
    qps = {bw: ws * args.nq / (ms[bw] / 1e3) for bw in pair}
    value = interp_qps(recalls[lo], qps[lo], recalls[hi], qps[hi])

    # e2e: the C ABI with host buffers (copies in, search, copies out)
    out_i = torch.empty(args.nq, K, dtype=torch.int32).pin_memory()
    out_d = torch.empty(args.nq, K, dtype=torch.float32).pin_memory()
    e2e_ms = {}
    with ClockSampler(dev) as clk_e2e:
        for bw in pair:
            for _ in range(max(2, args.warmup)):
                _lib.call("jb_graph_search_host", g._handle, q_host.data_ptr(), args.nq, 128,
                          out_i.data_ptr(), out_d.data_ptr(), K, bw, 2 * bw, stream.cuda_stream)
            ts = []
            for _ in range(max(args.steps, 10)):
                flush_l2(flush)
                torch.cuda.synchronize()
                t1 = time.perf_counter()
                _lib.call("jb_graph_search_host", g._handle, q_host.data_ptr(), args.nq, 128,
                          out_i.data_ptr(), out_d.data_ptr(), K, bw, 2 * bw, stream.cuda_stream)
                ts.append(time.perf_counter() - t1)
            e2e_ms[bw] = 1e3 * float(np.median(ts))
    if dist is not None:
        t = torch.tensor([e2e_ms[bw] for bw in pair], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = {bw: v for bw, v in zip(pair, t.tolist())}
    e2e_qps = {bw: ws * args.nq / (e2e_ms[bw] / 1e3) for bw in pair}
    e2e_value = interp_qps(recalls[lo], e2e_qps[lo], recalls[hi], e2e_qps[hi])

    # roofline numerator: algorithmic bytes of the search at the upper width
    # B_q = 2*dpad (query) + sum_expanded(1 + 4*deg) + 2*dpad*(distinct rows evaluated) + 8k
    _, _, st = g.search_with_stats(queries, k=K, beam_width=hi, distinct=True)
    st = st.long().cpu()
    dpad = 128
    bytes_q = (2 * dpad + st[:, 0] + 4 * st[:, 1] + 2 * dpad * st[:, 4] + 8 * K).sum().item()
    peak, peak_kind = measured_peaks()
    achieved = bytes_q / (ms[hi] / 1e3) / 1e9
    traffic = SEARCH_TRAFFIC.get((args.n, args.nq, hi))
    roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "traffic": traffic,
                "traffic_source": "profiles/search_cfg2_bw32.md (dram__bytes_read.sum + "
                                  "dram__bytes_write.sum, one launch)" if traffic else None,
                "algorithmic_bytes_per_launch": int(bytes_q),
                "peak_source": peak_kind, "kernel": f"beam_search_warp_kernel bw={hi}",
                "bytes_per_query": round(bytes_q / args.nq, 1),
                "expansions_per_query": round(st[:, 0].float().mean().item(), 2),
                "distinct_rows_per_query": round(st[:, 4].float().mean().item(), 2)}

    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(g, base_np, q_np, lo, hi, recalls, args)

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "queries/s",
            "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(total_ms, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16 rows, f32 distances", "data": "synthetic",
            "config": {"workload": "config2: 1M x 128 SIFT-like fp16, L2, R=64, alpha=1.2, "
                                   f"{args.nq} queries/GPU, k=10",
                       "n_base": args.n, "queries_per_gpu": args.nq,
                       "bracket_beam_widths": list(pair), "limit": "2*beam_width",
                       "parallelism": f"independent shards x{ws}" if ws > 1 else "single",
                       "l2": "flushed between timed searches (256 MB write)"},
            "recall_at_10": {str(b): round(r, 4) for b, r in recalls.items()},
            "qps": {str(b): round(v, 1) for b, v in qps.items()},
            "build": {"mvec_per_s": round(ws * args.n / build_s / 1e6, 4),
                      "seconds": round(build_s, 3),
                      "note": (f"{ws} shards of {args.n} rows built concurrently, one per GPU; "
                               "time = max over ranks") if ws > 1 else "single GPU"},
            "e2e": {"value": round(e2e_value, 1), "unit": "queries/s",
                    "h2d_bytes_per_step": int(len(pair) * args.nq * 128 * 2),
                    "d2h_bytes_per_step": int(len(pair) * args.nq * K * 8),
                    "timing": "median host wall time of jb_graph_search_host per call",
                    "clocks": clk_e2e.summary()},
            "roofline": roofline,
            "cpu_baseline": cpu,
            "gpu_launches": args.steps * len(pair),
            "clocks": clk.summary(),
            "wall_s_timed": round(wall, 3),
        }
        print(json.dumps(line), flush=True)
    g.free()
    if dist is not None:
        dist.destroy_process_group()


def cpu_baseline(g, base_np, q_np, lo, hi, recalls, args):
    """The CPU restatement of the reference search (oracle/, a port) timed on
    this host's cores, on a bounded sample of the same queries."""
    from oracle import oracle as O
    from jasper_b200 import _lib
    n, R = base_np.shape[0], 64
    og = O.OracleGraph(base_np, R)
    _lib.call("jb_graph_get_edges", g._handle, og.edges.ctypes.data, og.edist.ctypes.data,
              og.counts.ctypes.data)
    cores = O.max_threads()
    O.set_threads(cores)
    out = {}
    budget_s = args.cpu_seconds / (2 if lo != hi else 1)
    for bw in sorted({lo, hi}):
        done, t_used = 0, 0.0
        sample = 500
        while t_used < budget_s and done < q_np.shape[0]:
            qs = q_np[done:done + sample]
            t0 = time.perf_counter()
            og.search(qs, K, bw, 2 * bw)
            t_used += time.perf_counter() - t0
            done += qs.shape[0]
        out[bw] = done / t_used
    qps = interp_qps(recalls[lo], out[lo], recalls[hi], out[hi])
    return {"value": round(qps, 1), "unit": "queries/s", "cores": cores, "kind": "port",
            "sample": f"first queries of the same set until ~{args.cpu_seconds:.0f} s of CPU time "
                      f"per run, beam widths {sorted({lo, hi})}, all host threads"}


# ── config 5: range-sharded index (one shard per GPU) ─────────────────────
def gen_sift_like_gpu(n: int, dim: int, n_centers: int, seed: int, dev) -> torch.Tensor:
    """SIFT-like rows generated on the GPU (config 5 at 12.5M rows per shard):
    a Gaussian mixture of n_centers centres with uniform integer coordinates
    in [0, 128], uniform cluster choice, per-dimension sigma 12, rounded and
    clipped to [0, 255].  Same distribution as jasper_b200.synthetic.sift_like
    (which draws with numpy); the centres depend on the seed only."""
    gc = torch.Generator(device=dev).manual_seed(1_000_003)
    centers = torch.randint(0, 129, (n_centers, dim), generator=gc, device=dev).float()
    g = torch.Generator(device=dev).manual_seed(seed)
    out = torch.empty(n, dim, dtype=torch.float16, device=dev)
    for i in range(0, n, 1 << 20):
        m = min(1 << 20, n - i)
        c = torch.randint(0, n_centers, (m,), generator=g, device=dev)
        x = centers[c] + 12.0 * torch.randn(m, dim, generator=g, device=dev)
        out[i:i + m] = x.round_().clamp_(0, 255).half()
    return out


def exact_topk_shard(base: torch.Tensor, queries: torch.Tensor, k: int, offset: int):
    """Exact L2 top-k of every query over one shard (fp32; exact for integer
    rows), ids global.  Blocks of 1000 queries x 1M rows bound the scratch."""
    torch.backends.cuda.matmul.allow_tf32 = False
    out_i, out_d = [], []
    for q0 in range(0, queries.size(0), 1000):
        qf = queries[q0:q0 + 1000].float()
        qn = (qf * qf).sum(1, keepdim=True)
        best_d = torch.full((qf.size(0), k), float("inf"), device=base.device)
        best_i = torch.full((qf.size(0), k), -1, dtype=torch.int64, device=base.device)
        for b0 in range(0, base.size(0), 1 << 20):
            b = base[b0:b0 + (1 << 20)].float()
            d = qn + (b * b).sum(1)[None, :] - 2.0 * (qf @ b.T)
            dk, ik = d.topk(k, dim=1, largest=False)
            cd = torch.cat([best_d, dk], 1)
            ci = torch.cat([best_i, ik + b0 + offset], 1)
            best_d, sel = cd.topk(k, dim=1, largest=False)
            best_i = ci.gather(1, sel)
        out_i.append(best_i.int())
        out_d.append(best_d)
    return torch.cat(out_i), torch.cat(out_d)


def run_sharded(args):
    """Config 5: every rank builds a range shard of args.n_shard rows (global
    ids rank * n_shard + i) concurrently; each query batch goes to every
    rank, per-shard top-k are gathered to rank 0 over NCCL and merged there
    (jb_merge_topk).  Weak scaling: the index grows with the number of GPUs."""
    from jasper_b200 import sharded
    ws, rank, local = dist_env()
    dist = None
    if ws > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    dev = torch.device("cuda", torch.cuda.current_device())
    n_shard = args.n_shard
    n_total = n_shard * ws
    offset = rank * n_shard
    base = gen_sift_like_gpu(n_shard, 128, 65536, 8 + 1000 * rank, dev)
    queries = gen_sift_like_gpu(args.nq, 128, 65536, 9, dev)   # identical on every rank

    def barrier():
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(vals):
        t = torch.tensor(vals, device=dev, dtype=torch.float64)
        if dist is not None:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.tolist()

    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    sg = sharded.ShardedGraph.build(base, offset, n_total, n_neighbors=64, distance="l2",
                                    alpha=1.2)
    e1.record()
    barrier()
    (build_s,) = max_over_ranks([e0.elapsed_time(e1) / 1e3])

    gi, gd = exact_topk_shard(base, queries, K, offset)
    if ws > 1:
        got = sharded.gather_topk(gi, gd, root=0)
        gt = sharded.merge_topk(got[0], got[1])[0] if rank == 0 else None
    else:
        gt = gi

    def search(bw):
        if ws > 1:
            return sg.search(queries, k=K, beam_width=bw, root=0)
        return sg.search_local(queries, k=K, beam_width=bw)

    recalls = {}
    for bw in BWS:
        res = search(bw)
        r = recall_at_k(res[0], gt) if rank == 0 else 0.0
        recalls[bw] = r
    t = torch.tensor([recalls[bw] for bw in BWS], device=dev, dtype=torch.float64)
    if dist is not None:
        dist.broadcast(t, 0)
    recalls = {bw: v for bw, v in zip(BWS, t.tolist())}
    lo, hi = bracket(recalls)
    pair = (lo, hi) if lo != hi else (hi,)
    stream = torch.cuda.current_stream()
    for _ in range(args.warmup):
        for bw in pair:
            search(bw)
    barrier()
    times = {bw: [] for bw in pair}
    with ClockSampler(dev) as clk:
        for _ in range(args.steps):
            for bw in pair:
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                search(bw)
                b.record(stream)
                times[bw].append((a, b))
        torch.cuda.synchronize()
    barrier()
    ms_local = [sum(x.elapsed_time(y) for x, y in times[bw]) / args.steps for bw in pair]
    ms = dict(zip(pair, max_over_ranks(ms_local)))
    qps = {bw: args.nq / (ms[bw] / 1e3) for bw in pair}
    value = interp_qps(recalls[lo], qps[lo], recalls[hi], qps[hi])

    # e2e: queries from pinned host memory, the merged top-k back to the host
    q_host = queries.cpu().pin_memory()
    e2e = {}
    clk_e2e = ClockSampler(dev)
    clk_e2e.__enter__()
    for bw in pair:
        ts = []
        for it in range(max(args.steps, 10) + args.warmup):
            barrier()
            t1 = time.perf_counter()
            qd = q_host.to(dev, non_blocking=True)
            res = sg.search(qd, k=K, beam_width=bw, root=0) if ws > 1 else \
                sg.search_local(qd, k=K, beam_width=bw)
            if res is not None:
                res[0].cpu(), res[1].cpu()
            torch.cuda.synchronize()
            if it >= args.warmup:
                ts.append(time.perf_counter() - t1)
        e2e[bw] = float(np.median(ts)) * 1e3
    clk_e2e.__exit__(None, None, None)
    e2e = dict(zip(pair, max_over_ranks([e2e[bw] for bw in pair])))
    e2e_qps = {bw: args.nq / (e2e[bw] / 1e3) for bw in pair}
    e2e_value = interp_qps(recalls[lo], e2e_qps[lo], recalls[hi], e2e_qps[hi])

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "queries/s", "n_gpus": ws,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(sum(ms.values()), 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f16 rows, f32 distances", "data": "synthetic",
            "config": {"workload": f"config5: range-sharded {n_total} x 128 SIFT-like fp16 "
                                   f"({ws} shards x {n_shard}), L2, R=64, alpha=1.2, "
                                   f"{args.nq} queries broadcast, k=10, NCCL gather + device merge",
                       "n_base": n_total, "rows_per_gpu": n_shard, "queries": args.nq,
                       "bracket_beam_widths": list(pair), "limit": "2*beam_width",
                       "parallelism": f"range shards x{ws}",
                       "l2": "inputs larger than L2 (3.2 GB of rows per GPU)"},
            "recall_at_10": {str(b): round(r, 4) for b, r in recalls.items()},
            "qps": {str(b): round(v, 1) for b, v in qps.items()},
            "build": {"mvec_per_s": round(n_total / build_s / 1e6, 4),
                      "seconds": round(build_s, 3),
                      "note": f"{ws} shards built concurrently; time = max over ranks"},
            "e2e": {"value": round(e2e_value, 1), "unit": "queries/s",
                    "h2d_bytes_per_step": int(len(pair) * args.nq * 128 * 2),
                    "d2h_bytes_per_step": int(len(pair) * args.nq * K * 8),
                    "timing": "median host wall time per query batch (upload, search on "
                              "every shard, gather, merge, download), max over ranks",
                    "clocks": clk_e2e.summary()},
            "gpu_launches": args.steps * len(pair) * (2 if ws > 1 else 1),
            "clocks": clk.summary(),
        }
        print(json.dumps(line), flush=True)
    sg.free()
    if dist is not None:
        dist.destroy_process_group()


# ── prerotation GEMM (tensor cores vs the SIMT reference GEMM) ───────────
def run_rotation(args):
    """Times jb_rotate_rows (Y = rows x P^T, fp16 in/out, fp32 accumulation)
    on the tcgen05 kernel and on the SIMT GEMM at the config-3 (D = 128,
    1M rows) and config-4 (D = 960, 250k rows) shapes; one JSON line each."""
    from jasper_b200 import _lib
    torch.cuda.set_device(0)
    peak_tf = 1657.0
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        peak_tf = float(json.loads(p.read_text()).get("bf16_tflops", peak_tf))
    hbm, _ = measured_peaks()
    for dim, n in ((128, 1_000_000), (960, 250_000)):
        dpad = (dim + 7) // 8 * 8
        g = torch.Generator(device="cuda").manual_seed(4)
        x = torch.randn(n, dpad, generator=g, device="cuda").half()
        y = torch.empty_like(x)
        line = {"mode": "rotation", "dim": dim, "rows": n}
        for tc in (1, 0):
            for _ in range(args.warmup):
                _lib.call("jb_rotate_rows", dim, 4, x.data_ptr(), y.data_ptr(), n, tc,
                          torch.cuda.current_stream().cuda_stream)
            ts = []
            for _ in range(args.steps):
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                e0.record()
                _lib.call("jb_rotate_rows", dim, 4, x.data_ptr(), y.data_ptr(), n, tc,
                          torch.cuda.current_stream().cuda_stream)
                e1.record()
                torch.cuda.synchronize()
                ts.append(e0.elapsed_time(e1))
            ms = float(np.median(ts))
            tflops = 2.0 * n * dpad * dpad / ms / 1e9
            gbs = (4.0 * n * dpad + 2.0 * dpad * dpad) / ms / 1e6
            line["tcgen05" if tc else "simt"] = {
                "ms": round(ms, 4), "tflops": round(tflops, 1), "gbs": round(gbs, 1),
                "frac_of_bf16_peak": round(tflops / peak_tf, 4),
                "frac_of_hbm": round(gbs / hbm, 4)}
        print(json.dumps(line), flush=True)


# ── config 3 (directional) and config 4 (RaBitQ) ─────────────────────────
def _timed_qps(fn, nq, steps, warmup):
    """Device time of fn() (CUDA events, median over steps) -> (QPS, ms)."""
    for _ in range(warmup):
        fn()
    ts = []
    for _ in range(steps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        ts.append(a.elapsed_time(b))
    ms = float(np.median(ts))
    return nq / (ms / 1e3), ms


def run_directional(args):
    """Config 3: config-1 rows (100k x 128 N(0,1), seed 0; 1k queries, seed
    1), R = 32, prerotation seed 4; LSH with k_ranks 4 and 16 (32,768
    calibration samples) and PQ with M = k_ranks and M = 32 (4-dim
    subspaces, k-means 20 iterations, seed 5); directional_search /
    pq_search at beam 64 and 128.  One JSON line per estimator."""
    import jasper_b200 as jasper
    from jasper_b200 import _lib, synthetic
    torch.cuda.set_device(0)
    X = torch.from_numpy(synthetic.gaussian(100_000, 128, 0)).cuda()
    Q = torch.from_numpy(synthetic.gaussian(1000, 128, 1)).cuda()
    gt = exact_gt(X, Q, K)
    for kr in (4, 16):
        g = jasper.Graph.build(X, n_neighbors=32, alpha=1.2, build_lsh=True, build_pq=True,
                               k_ranks=kr, prerotate_seed=4, lsh_samples=32768,
                               pq_kmeans_iter=20, pq_seed=5)
        runs = [("lsh", kr, g.directional_search), ("pq", kr, g.pq_search)]
        for name, m, fn in runs:
            line = {"mode": "directional", "config": "config3", "estimator": name,
                    "k_ranks" if name == "lsh" else "pq_m": m}
            for bw in (64, 128):
                ids, _ = fn(Q, k=K, beam_width=bw)
                qps, ms = _timed_qps(lambda: fn(Q, k=K, beam_width=bw), 1000, args.steps, args.warmup)
                line[f"bw{bw}"] = {"recall_at_10": round(recall_at_k(ids, gt), 4),
                                   "qps": round(qps, 1), "ms": round(ms, 4)}
            print(json.dumps(line), flush=True)
        if kr == 4:
            # the 32 x 4-dim codebooks BASELINE asks for (the reference only has M = k_ranks)
            _lib.call("jb_graph_build_pq", g._handle, 32, 40000, 20, 5)
            line = {"mode": "directional", "config": "config3", "estimator": "pq", "pq_m": 32}
            for bw in (64, 128):
                ids, _ = g.pq_search(Q, k=K, beam_width=bw)
                qps, ms = _timed_qps(lambda: g.pq_search(Q, k=K, beam_width=bw), 1000, args.steps,
                                     args.warmup)
                line[f"bw{bw}"] = {"recall_at_10": round(recall_at_k(ids, gt), 4),
                                   "qps": round(qps, 1), "ms": round(ms, 4)}
            print(json.dumps(line), flush=True)
        g.free()


def gen_relu_sphere_gpu(n, dim, n_centers, sigma, seed, center_seed, dev):
    """Config-4 rows on the GPU: Gaussian mixture (centres N(0,1)), per-dim
    sigma, ReLU, L2-normalised, fp16."""
    gc = torch.Generator(device=dev).manual_seed(center_seed)
    centers = torch.randn(n_centers, dim, generator=gc, device=dev)
    g = torch.Generator(device=dev).manual_seed(seed)
    out = torch.empty(n, dim, dtype=torch.float16, device=dev)
    for i in range(0, n, 1 << 18):
        m = min(1 << 18, n - i)
        c = torch.randint(0, n_centers, (m,), generator=g, device=dev)
        x = (centers[c] + sigma * torch.randn(m, dim, generator=g, device=dev)).clamp_(min=0)
        x = x / x.norm(dim=1, keepdim=True).clamp_(min=1e-12)
        out[i:i + m] = x.half()
    return out


def run_rabitq(args):
    """Config 4: 1M x 960 ReLU-clamped, L2-normalised Gaussian-mixture rows
    (256 centres, sigma 0.3, seed 6), 1k queries (seed 7), inner product,
    R = 64, alpha = 1.0; RaBitQ 1-bit codes; k = 10, beam 64 / 128 / 256:
    the exact beam search with the RaBitQ candidate filter (margin 1) and
    without it (exact), with rows read per query."""
    import jasper_b200 as jasper
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    n = args.n
    X = gen_relu_sphere_gpu(n, 960, 256, 0.3, 6, 6, dev)
    Q = gen_relu_sphere_gpu(1000, 960, 256, 0.3, 7, 6, dev)
    torch.backends.cuda.matmul.allow_tf32 = False
    sims = []
    for q0 in range(0, 1000, 250):
        s = Q[q0:q0 + 250].float() @ X.float().T
        sims.append(s.topk(K, dim=1).indices.int())
    gt = torch.cat(sims)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    g = jasper.Graph.build(X, n_neighbors=64, distance="ip", alpha=1.0, build_rabitq=True)
    torch.cuda.synchronize()
    build_s = time.perf_counter() - t0
    line = {"mode": "rabitq", "config": "config4", "rows": n, "dim": 960,
            "build": {"seconds": round(build_s, 3), "mvec_per_s": round(n / build_s / 1e6, 4),
                      "note": "graph construction + prerotation + RaBitQ codes"}}
    from jasper_b200 import _lib
    for bw in (64, 128, 256):
        # margin 1e30: the filter never drops anything (the exact search)
        for name, margin in (("rabitq", 1.0), ("exact", 1e30)):
            ids, _ = g.rabitq_search(Q, k=K, beam_width=bw, margin=margin)
            qps, ms = _timed_qps(lambda: g.rabitq_search(Q, k=K, beam_width=bw, margin=margin),
                                 1000, args.steps, args.warmup)
            st = torch.zeros(1000, 5, dtype=torch.int32, device=dev)
            oi = torch.empty(1000, K, dtype=torch.int32, device=dev)
            od = torch.empty(1000, K, dtype=torch.float32, device=dev)
            _lib.call("jb_graph_search_rabitq", g._handle, Q.data_ptr(), 1000, 960, oi.data_ptr(),
                      od.data_ptr(), K, bw, 2 * bw, float(margin), st.data_ptr(),
                      torch.cuda.current_stream().cuda_stream)
            torch.cuda.synchronize()
            line[f"{name}_bw{bw}"] = {"recall_at_10": round(recall_at_k(ids, gt), 4),
                                      "qps": round(qps, 1), "ms": round(ms, 4),
                                      "rows_read_per_query": round(st[:, 2].float().mean().item(), 1)}
    print(json.dumps(line), flush=True)
    g.free()


# ── reference arm ─────────────────────────────────────────────────────────
def run_reference(args):
    ws, rank, local = dist_env()
    if rank != 0:
        return
    lib = ROOT / "oracle" / "_ref" / "lib" / "libjasper_ffi.so"
    if not lib.exists():
        print(json.dumps({"impl": "reference", "unavailable":
                          "reference library oracle/_ref/lib/libjasper_ffi.so was not built"}))
        return
    import tvm_ffi
    torch.cuda.set_device(local if ws > 1 else 0)
    mod = tvm_ffi.load_module(str(lib))
    base_np, q_np = load_data(args.n, args.nq, 0)
    base = torch.from_numpy(base_np).cuda()
    queries = torch.from_numpy(q_np).cuda()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    h = mod.jasper_construct_f16_r64_l2(base, 128, 1.2, 10 * 10**9, False)
    torch.cuda.synchronize()
    build_s = time.perf_counter() - t0
    gt = exact_gt(base, queries, K)
    search = mod.jasper_search_f16_r64_l2
    oi = torch.empty(args.nq, K, dtype=torch.int32, device="cuda")
    od = torch.empty(args.nq, K, dtype=torch.float32, device="cuda")
    recalls = {}
    for bw in BWS:
        search(h, queries, oi, od, K, bw, 2 * bw, False)
        torch.cuda.synchronize()
        recalls[bw] = recall_at_k(oi, gt)
    lo, hi = bracket(recalls)
    pair = (lo, hi) if lo != hi else (hi,)
    flush = torch.zeros(64 * 1024 * 1024, dtype=torch.float32, device="cuda")
    for _ in range(args.warmup):
        for bw in pair:
            search(h, queries, oi, od, K, bw, 2 * bw, False)
    torch.cuda.synchronize()
    ts = {bw: [] for bw in pair}
    with ClockSampler(torch.device("cuda", 0)) as clk:
        for _ in range(args.steps):
            for bw in pair:
                flush_l2(flush)
                torch.cuda.synchronize()
                t1 = time.perf_counter()
                search(h, queries, oi, od, K, bw, 2 * bw, False)
                torch.cuda.synchronize()
                ts[bw].append(time.perf_counter() - t1)
    ms = {bw: 1e3 * float(np.mean(ts[bw])) for bw in pair}
    qps = {bw: args.nq / (ms[bw] / 1e3) for bw in pair}
    value = interp_qps(recalls[lo], qps[lo], recalls[hi], qps[hi])
    mod.jasper_free_graph(h)
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 1), "unit": "queries/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(sum(ms.values()), 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f16 rows, f32 distances", "data": "synthetic",
        "config": {"workload": "config2: 1M x 128 SIFT-like fp16, L2, R=64, alpha=1.2, "
                               f"{args.nq} queries, k=10",
                   "n_base": args.n, "queries_per_gpu": args.nq, "bracket_beam_widths": list(pair),
                   "limit": "2*beam_width", "parallelism": "single",
                   "l2": "flushed between timed searches (256 MB write)",
                   "implementation": "unmodified reference CUDA sources (ffi/*.cu) compiled for "
                                     "sm_100a by oracle/build_ref.sh, called through its tvm_ffi ops"},
        "recall_at_10": {str(b): round(r, 4) for b, r in recalls.items()},
        "qps": {str(b): round(v, 1) for b, v in qps.items()},
        "build": {"mvec_per_s": round(args.n / build_s / 1e6, 4), "seconds": round(build_s, 3)},
        "cpu_baseline": {"value": round(value, 1), "unit": "queries/s", "cores": 0,
                         "kind": "reference",
                         "sample": "the reference ships no CPU search: this arm runs its own "
                                   "CUDA implementation on the B200 (wall clock incl. its "
                                   "per-call cudaMalloc and stream sync)"},
        "e2e": {"value": round(value, 1), "unit": "queries/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="jasper_b200", choices=["jasper_b200", "reference"])
    ap.add_argument("--n", type=int, default=1_000_000)
    ap.add_argument("--nq", type=int, default=10_000)
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--mode", default="replicas",
                    choices=["replicas", "sharded", "rotation", "directional", "rabitq"],
                    help="replicas: config 2 per GPU (default); sharded: config 5 range "
                         "shards; rotation: the prerotation GEMM alone; directional: "
                         "config 3 (LSH / PQ); rabitq: config 4")
    ap.add_argument("--n-shard", type=int, default=12_500_000,
                    help="rows per GPU in --mode sharded (config 5: 12.5M)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.mode == "sharded":
        run_sharded(args)
    elif args.mode == "rotation":
        run_rotation(args)
    elif args.mode == "directional":
        run_directional(args)
    elif args.mode == "rabitq":
        run_rabitq(args)
    else:
        run_jasper(args)


if __name__ == "__main__":
    main()
