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


class ClockSampler:
    """nvidia-smi samples during the timed region (SM clock, throttle reasons)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        mhz, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            p = [x.strip() for x in ln.split(",")]
            if len(p) < 9:
                continue
            try:
                mhz.append(float(p[1]))
                mx = max(mx, float(p[2]))
            except ValueError:
                continue
            for nm, v in zip(names, p[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        if not mhz:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        return {"sm_mhz": float(np.median(mhz)), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(mhz)}


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
    with ClockSampler(dev.index if ws == 1 else local) as clk:
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
    for bw in pair:
        for _ in range(2):
            _lib.call("jb_graph_search_host", g._handle, q_host.data_ptr(), args.nq, 128,
                      out_i.data_ptr(), out_d.data_ptr(), K, bw, 2 * bw, stream.cuda_stream)
        ts = []
        for _ in range(args.steps):
            flush_l2(flush)
            torch.cuda.synchronize()
            t1 = time.perf_counter()
            _lib.call("jb_graph_search_host", g._handle, q_host.data_ptr(), args.nq, 128,
                      out_i.data_ptr(), out_d.data_ptr(), K, bw, 2 * bw, stream.cuda_stream)
            ts.append(time.perf_counter() - t1)
        e2e_ms[bw] = 1e3 * float(np.mean(ts))
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
    roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "traffic": None,
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
                    "d2h_bytes_per_step": int(len(pair) * args.nq * K * 8)},
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
    with ClockSampler(0) as clk:
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
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_jasper(args)


if __name__ == "__main__":
    main()
