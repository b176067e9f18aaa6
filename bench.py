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
with host buffers (jb_graph_search_host on page-locked buffers: the search
kernel reads the queries from host memory and writes the results there).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

With N > 1 (torchrun, one rank per GPU) every rank holds the same config-2
graph and searches its slice of the same 10,000 queries; the slices' top-k
are gathered to rank 0 over NCCL inside each timed step (strong scaling),
times are the max over ranks.  The run then adds the config-5 range-sharded
leg (one 12.5M-row shard per GPU, queries broadcast, top-k gathered and
merged; weak scaling) under "range_sharded".  After the timed region, rank 0
at N = 1 also reports the CPU baselines and parity with the reference's own
build (oracle/_ref) -- checkers, never on the timed path.

Other modes: --mode config1 | directional (config 3) | rabitq (config 4) |
sharded (config 5 alone) | rotation; --impl reference runs the reference's
CUDA build on the same config (--ref-ndebug: its -DNDEBUG build).
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
SEARCH_TRAFFIC = {(1_000_000, 10_000, 32): 1_719_287_344}
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


def exact_ip_gt(base: torch.Tensor, queries: torch.Tensor, k: int) -> torch.Tensor:
    """Exact maximum-inner-product top-k on the GPU in fp32."""
    torch.backends.cuda.matmul.allow_tf32 = False
    out = []
    for q0 in range(0, queries.size(0), 250):
        s = queries[q0:q0 + 250].float() @ base.float().T
        out.append(s.topk(k, dim=1).indices.int())
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
class stdout_to_stderr:
    """Sends fd 1 to fd 2 while the reference library prints its progress,
    so that this script's stdout carries only its JSON lines."""

    def __enter__(self):
        sys.stdout.flush()
        self.saved = os.dup(1)
        os.dup2(2, 1)
        return self

    def __exit__(self, *exc):
        sys.stdout.flush()
        os.dup2(self.saved, 1)
        os.close(self.saved)


def init_dist():
    ws, rank, local = dist_env()
    dist = None
    if ws > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return ws, rank, dist, torch.device("cuda", torch.cuda.current_device())


def max_over_ranks(dist, vals, dev):
    t = torch.tensor(vals, device=dev, dtype=torch.float64)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def run_jasper(args):
    """Config 2.  N = 1: one GPU searches all 10,000 queries.  N > 1: the
    small-index mode -- every rank holds the same config-2 graph (replica)
    and searches its contiguous slice of the same 10,000 queries; the
    slices' top-k are gathered to rank 0 over NCCL inside the timed step
    (strong scaling: total work fixed)."""
    import jasper_b200 as jasper
    from jasper_b200 import _lib, sharded
    ws, rank, dist, dev = init_dist()
    base_np, q_np = load_data(args.n, args.nq, 0)
    base = torch.from_numpy(base_np).to(dev)
    queries = torch.from_numpy(q_np).to(dev)
    sl = sharded.split_queries(args.nq, ws, rank)
    nloc_max = -(-args.nq // ws)
    q_loc = queries[sl].contiguous()
    nloc = q_loc.shape[0]
    q_loc_host = torch.from_numpy(q_np[sl]).pin_memory()

    # one untimed warm-up build on the first 50k rows: CUDA loads each kernel
    # of the library on its first launch, which is not build work
    jasper.Graph.build(base[:50_000], n_neighbors=64, distance="l2", alpha=1.2).free()
    # build (device time on every replica; max over ranks)
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    t0 = time.perf_counter()
    g = jasper.Graph.build(base, n_neighbors=64, distance="l2", alpha=1.2)
    torch.cuda.synchronize()
    (build_s,) = max_over_ranks(dist, [time.perf_counter() - t0], dev)

    gt = exact_gt(base, queries, K)
    recalls, full = {}, {}
    for bw in BWS:     # every replica holds the same graph: identical sweeps
        ids, dd = g.search(queries, k=K, beam_width=bw)
        recalls[bw] = recall_at_k(ids, gt)
        full[bw] = (ids, dd)
    lo, hi = bracket(recalls)
    pair = (lo, hi) if lo != hi else (hi,)

    flush = torch.zeros(64 * 1024 * 1024, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream()
    gbuf = torch.empty(ws, 2, nloc_max, K, dtype=torch.int32, device=dev) if ws > 1 else None
    pad_i = torch.full((nloc_max, K), -1, dtype=torch.int32, device=dev)
    pad_d = torch.full((nloc_max, K), 1e30, dtype=torch.float32, device=dev)

    def one(bw):
        ids, dd = g.search(q_loc, k=K, beam_width=bw)
        if dist is None:
            return ids, dd
        if nloc < nloc_max:
            pad_i[:nloc].copy_(ids)
            pad_d[:nloc].copy_(dd)
            ids, dd = pad_i, pad_d
        return sharded.gather_topk(ids, dd, root=0, out=gbuf)

    def step(times):
        for bw in pair:
            flush_l2(flush)
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            one(bw)
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
    ms_l = [sum(a.elapsed_time(b) for a, b in times[bw]) / args.steps for bw in pair]
    ms = dict(zip(pair, max_over_ranks(dist, ms_l, dev)))
    total_ms = sum(ms.values())
    qps = {bw: args.nq / (ms[bw] / 1e3) for bw in pair}
    value = interp_qps(recalls[lo], qps[lo], recalls[hi], qps[hi])

    # the split-and-gathered results equal one GPU's search of all queries
    split_ok = None
    if dist is not None:
        got = one(hi)
        if rank == 0:
            gi = torch.cat([got[0][r, :sharded.shard_range(args.nq, ws, r)[1]] for r in range(ws)])
            gd = torch.cat([got[1][r, :sharded.shard_range(args.nq, ws, r)[1]] for r in range(ws)])
            split_ok = bool(torch.equal(gi, full[hi][0]) and
                            torch.equal(gd.view(torch.int32), full[hi][1].view(torch.int32)))

    # e2e: the C ABI with page-locked host buffers (queries read and results
    # written by the search kernel over the host link), each rank on its
    # slice; max over ranks of the median call
    out_i = torch.empty(nloc, K, dtype=torch.int32).pin_memory()
    out_d = torch.empty(nloc, K, dtype=torch.float32).pin_memory()
    e2e_ms = {}
    with ClockSampler(dev) as clk_e2e:
        for bw in pair:
            for _ in range(max(2, args.warmup)):
                _lib.call("jb_graph_search_host", g._handle, q_loc_host.data_ptr(), nloc, 128,
                          out_i.data_ptr(), out_d.data_ptr(), K, bw, 2 * bw, stream.cuda_stream)
            ts = []
            for _ in range(max(args.steps, 10)):
                flush_l2(flush)
                torch.cuda.synchronize()
                if dist is not None:
                    dist.barrier()
                t1 = time.perf_counter()
                _lib.call("jb_graph_search_host", g._handle, q_loc_host.data_ptr(), nloc, 128,
                          out_i.data_ptr(), out_d.data_ptr(), K, bw, 2 * bw, stream.cuda_stream)
                ts.append(time.perf_counter() - t1)
            e2e_ms[bw] = 1e3 * float(np.median(ts))
    # the host results of the last call (upper width) against the device search
    e2e_ok = bool(torch.equal(out_i, full[pair[-1]][0][sl].cpu()) and
                  torch.equal(out_d.view(torch.int32), full[pair[-1]][1][sl].cpu().view(torch.int32)))
    e2e_ms = dict(zip(pair, max_over_ranks(dist, [e2e_ms[bw] for bw in pair], dev)))
    e2e_qps = {bw: args.nq / (e2e_ms[bw] / 1e3) for bw in pair}
    e2e_value = interp_qps(recalls[lo], e2e_qps[lo], recalls[hi], e2e_qps[hi])

    # roofline numerator: algorithmic bytes of this rank's search at the upper
    # width, B_q = 2*dpad (query) + sum_expanded(1 + 4*deg) + 2*dpad*(distinct
    # rows evaluated) + 8k, over the search-only kernel time
    _, _, st = g.search_with_stats(q_loc, k=K, beam_width=hi, distinct=True)
    st = st.long().cpu()
    dpad = 128
    bytes_q = (2 * dpad + st[:, 0] + 4 * st[:, 1] + 2 * dpad * st[:, 4] + 8 * K).sum().item()
    kt = []
    for _ in range(max(args.steps, 5)):
        flush_l2(flush)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        g.search(q_loc, k=K, beam_width=hi)
        b.record(stream)
        kt.append((a, b))
    torch.cuda.synchronize()
    kernel_ms = float(np.mean([a.elapsed_time(b) for a, b in kt]))
    peak, peak_kind = measured_peaks()
    achieved = bytes_q / (kernel_ms / 1e3) / 1e9
    traffic = SEARCH_TRAFFIC.get((args.n, nloc, hi))
    roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "traffic": traffic,
                "traffic_source": "profiles/search_cfg2_bw32.md (dram__bytes_read.sum + "
                                  "dram__bytes_write.sum, one launch)" if traffic else None,
                "algorithmic_bytes_per_launch": int(bytes_q), "kernel_ms": round(kernel_ms, 4),
                "peak_source": peak_kind, "kernel": f"beam_search_warp_kernel bw={hi}",
                "queries_per_launch": nloc,
                "bytes_per_query": round(bytes_q / nloc, 1),
                "expansions_per_query": round(st[:, 0].float().mean().item(), 2),
                "distinct_rows_per_query": round(st[:, 4].float().mean().item(), 2)}

    cpu = parity = None
    if rank == 0 and ws == 1:
        if not args.no_cpu_baseline:
            cpu = cpu_baseline(g, base_np, q_np, lo, hi, recalls, args)
        if not args.no_parity:
            parity = parity_leg(g, base, queries, gt, recalls, args)
    g.free()
    del base, queries, flush, gbuf, pad_i, pad_d, full
    torch.cuda.empty_cache()

    shard_res = None
    if not args.no_sharded:
        shard_res = sharded_leg(args, ws, rank, dist, dev)

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "queries/s",
            "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(total_ms, 4), "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None, "dtype": "f16 rows, f32 distances", "data": "synthetic",
            "config": {"workload": "config2: 1M x 128 SIFT-like fp16, L2, R=64, alpha=1.2, "
                                   f"{args.nq} queries, k=10",
                       "n_base": args.n, "queries": args.nq, "queries_per_gpu": nloc_max,
                       "bracket_beam_widths": list(pair), "limit": "2*beam_width",
                       "parallelism": (f"replicated graph x{ws}, queries split, top-k gathered "
                                       "to rank 0 over NCCL inside the timed step")
                       if ws > 1 else "single",
                       "l2": "flushed between timed searches (256 MB write)"},
            "recall_at_10": {str(b): round(r, 4) for b, r in recalls.items()},
            "qps": {str(b): round(v, 1) for b, v in qps.items()},
            "split_gather_identical_to_one_gpu": split_ok,
            "build": {"mvec_per_s": round(args.n / build_s / 1e6, 4),
                      "seconds": round(build_s, 3),
                      "note": (f"the same graph built on each of {ws} replicas; time = max over "
                               "ranks (build scaling: range_sharded)") if ws > 1 else "single GPU"},
            "e2e": {"value": round(e2e_value, 1), "unit": "queries/s",
                    "h2d_bytes_per_step": int(len(pair) * args.nq * 128 * 2),
                    "d2h_bytes_per_step": int(len(pair) * args.nq * K * 8),
                    "timing": ("median host wall time of jb_graph_search_host per call"
                               + (" on each rank's query slice, max over ranks" if ws > 1 else "")),
                    "transfer": ("page-locked host buffers: the search kernel reads each query "
                                 "row from host memory once and writes the results to host "
                                 "memory (no separate copy before or after the search)"),
                    "identical_to_device_search": e2e_ok,
                    "clocks": clk_e2e.summary()},
            "roofline": roofline,
            "cpu_baseline": cpu,
            "parity_vs_reference": parity,
            "range_sharded": shard_res,
            "gpu_launches": args.steps * len(pair),
            "clocks": clk.summary(),
            "wall_s_timed": round(wall, 3),
        }
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.destroy_process_group()


def cpu_baseline(g, base_np, q_np, lo, hi, recalls, args):
    """The CPU baselines on this host's cores, on bounded samples of the same
    queries.  Headline: exact brute-force k-NN (oracle/bruteforce.c: fp16
    rows widened to fp32, all host threads, per-thread top-k; recall 1 by
    construction).  Beside it: the CPU restatement of the reference's beam
    search on this graph (a correctness oracle, timed for information)."""
    from oracle import oracle as O
    from jasper_b200 import _lib
    cores = os.cpu_count() or 1
    bf_base = base_np.astype(np.float32)
    bf_q = q_np.astype(np.float32)
    t0 = time.perf_counter()
    O.bruteforce_knn(bf_base, bf_q[:4 * cores], K, threads=cores)
    est = 4 * cores / (time.perf_counter() - t0)
    m = int(min(q_np.shape[0], max(4 * cores, est * args.cpu_seconds)))
    t0 = time.perf_counter()
    bi, _ = O.bruteforce_knn(bf_base, bf_q[:m], K, threads=cores)
    bf_qps = m / (time.perf_counter() - t0)
    exact = exact_gt(torch.from_numpy(base_np).cuda(), torch.from_numpy(q_np[:m]).cuda(), K)
    bf_recall = recall_at_k(torch.from_numpy(bi), exact.cpu())
    del bf_base

    n, R = base_np.shape[0], 64
    og = O.OracleGraph(base_np, R)
    _lib.call("jb_graph_get_edges", g._handle, og.edges.ctypes.data, og.edist.ctypes.data,
              og.counts.ctypes.data)
    O.set_threads(cores)
    port = {}
    budget_s = args.cpu_seconds / 2 / (2 if lo != hi else 1)
    for bw in sorted({lo, hi}):
        done, t_used = 0, 0.0
        while t_used < budget_s and done < q_np.shape[0]:
            qs = q_np[done:done + 500]
            t0 = time.perf_counter()
            og.search(qs, K, bw, 2 * bw)
            t_used += time.perf_counter() - t0
            done += qs.shape[0]
        port[bw] = done / t_used
    return {"value": round(bf_qps, 1), "unit": "queries/s", "cores": cores, "kind": "port",
            "algorithm": "exact brute-force k-NN (oracle/bruteforce.c), fp16 rows as fp32",
            "recall_at_10": round(bf_recall, 4),
            "sample": f"the first {m} of the {q_np.shape[0]} queries against all "
                      f"{base_np.shape[0]} rows (~{args.cpu_seconds:.0f} s), {cores} threads",
            "beam_search_port": {
                "value": round(interp_qps(recalls[lo], port[lo], recalls[hi], port[hi]), 1),
                "unit": "queries/s", "cores": cores,
                "note": "CPU restatement of the reference's beam search on this graph "
                        f"(a correctness oracle), beam widths {sorted({lo, hi})}"}}


def parity_leg(g, base, queries, gt, recalls, args):
    """The checker, after the timed region: parity with the reference's own
    CUDA build (oracle/_ref) on config 2.  (1) Same graph: this graph is
    saved, loaded by the reference, and searched there at every beam width;
    its ids and distance bits are compared with this library's search.
    (2) Build: the reference builds its own graph from the same rows; its
    recall@10 at every width is set beside this build's."""
    lib = ROOT / "oracle" / "_ref" / "lib" / "libjasper_ffi.so"
    try:
        import tvm_ffi
    except ImportError:
        return {"unavailable": "tvm_ffi not importable"}
    if not lib.exists():
        return {"unavailable": "reference library oracle/_ref not built"}
    import tempfile
    mod = tvm_ffi.load_module(str(lib))
    nq = queries.shape[0]
    oi = torch.empty(nq, K, dtype=torch.int32, device=queries.device)
    od = torch.empty(nq, K, dtype=torch.float32, device=queries.device)
    mism, total, max_rel = 0, 0, 0.0
    with tempfile.TemporaryDirectory() as td:
        path = os.path.join(td, "g.graph")
        g.save(path)
        with stdout_to_stderr():
            rh = mod.jasper_load_f16_r64_l2(path, 128, False)
    try:
        for bw in BWS:
            ji, jd = g.search(queries, k=K, beam_width=bw)
            with stdout_to_stderr():
                mod.jasper_search_f16_r64_l2(rh, queries, oi, od, K, bw, 2 * bw, False)
            torch.cuda.synchronize()
            bad = (ji != oi).any(1) | (jd.view(torch.int32) != od.view(torch.int32)).any(1)
            mism += int(bad.sum())
            total += nq
            rel = ((jd - od).abs() / od.abs().clamp(min=1e-30)).max().item()
            max_rel = max(max_rel, rel)
    finally:
        mod.jasper_free_graph(rh)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    with stdout_to_stderr():
        rh = mod.jasper_construct_f16_r64_l2(base, 128, 1.2, 10 * 10**9, False)
    torch.cuda.synchronize()
    ref_build_s = time.perf_counter() - t0
    ref_rec = {}
    try:
        for bw in BWS:
            with stdout_to_stderr():
                mod.jasper_search_f16_r64_l2(rh, queries, oi, od, K, bw, 2 * bw, False)
            torch.cuda.synchronize()
            ref_rec[bw] = recall_at_k(oi, gt)
    finally:
        mod.jasper_free_graph(rh)
    diff = max(abs(recalls[bw] - ref_rec[bw]) for bw in BWS)
    return {"same_graph_search": {"mismatched_queries": mism, "query_searches": total,
                                  "beam_widths": list(BWS), "max_rel_dist_err": max_rel,
                                  "compare": "ids and distance bits, this build's graph searched "
                                             "by the reference (jasper_search_f16_r64_l2)"},
            "build_recall": {"reference": {str(b): round(r, 4) for b, r in ref_rec.items()},
                             "here": {str(b): round(r, 4) for b, r in recalls.items()},
                             "max_abs_diff": round(diff, 4), "within_0.005": diff <= 0.005},
            "reference_build_s": round(ref_build_s, 3)}


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


def sharded_leg(args, ws, rank, dist, dev):
    """Config 5: every rank builds a range shard of args.n_shard rows (global
    ids rank * n_shard + i) concurrently; each query batch goes to every
    rank, per-shard top-k are gathered to rank 0 with one NCCL gather and
    merged there (jb_merge_topk_strided).  Weak scaling: the index grows
    with the number of GPUs.  Returns the result dict on rank 0."""
    from jasper_b200 import sharded
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

    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    sg = sharded.ShardedGraph.build(base, offset, n_total, n_neighbors=64, distance="l2",
                                    alpha=1.2)
    e1.record()
    barrier()
    own_build_s = e0.elapsed_time(e1) / 1e3
    (build_s,) = max_over_ranks(dist, [own_build_s], dev)
    build_each = [own_build_s]
    if dist is not None:
        t = torch.zeros(ws, device=dev, dtype=torch.float64)
        t[rank] = own_build_s
        dist.all_reduce(t)
        build_each = t.tolist()

    gi, gd = exact_topk_shard(base, queries, K, offset)
    if ws > 1:
        got = sharded.gather_topk(gi, gd, root=0)
        gt = sharded.merge_topk(got[0], got[1])[0] if rank == 0 else None
    else:
        gt = gi
    del base
    torch.cuda.empty_cache()

    def search(bw, phases=None):
        if ws > 1:
            return sg.search(queries, k=K, beam_width=bw, root=0, phases=phases)
        return sg.search_local(queries, k=K, beam_width=bw)

    recalls = {}
    for bw in BWS:
        res = search(bw)
        recalls[bw] = recall_at_k(res[0], gt) if rank == 0 else 0.0
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
    phases = {bw: [] for bw in pair}
    with ClockSampler(dev) as clk:
        for _ in range(args.steps):
            for bw in pair:
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                search(bw, phases[bw] if ws > 1 else None)
                b.record(stream)
                times[bw].append((a, b))
        torch.cuda.synchronize()
    barrier()
    ms_local = [sum(x.elapsed_time(y) for x, y in times[bw]) / args.steps for bw in pair]
    ms = dict(zip(pair, max_over_ranks(dist, ms_local, dev)))
    qps = {bw: args.nq / (ms[bw] / 1e3) for bw in pair}
    value = interp_qps(recalls[lo], qps[lo], recalls[hi], qps[hi])
    # per phase (median over steps): local search, gather (includes waiting
    # for the slowest shard), merge; every rank's numbers
    phase_ms = None
    if ws > 1:
        loc = []
        for bw in pair:
            ev = phases[bw]
            loc += [float(np.median([e[0].elapsed_time(e[1]) for e in ev])),
                    float(np.median([e[1].elapsed_time(e[2]) for e in ev])),
                    float(np.median([e[2].elapsed_time(e[3]) for e in ev]))]
        t = torch.zeros(ws, len(loc), device=dev, dtype=torch.float64)
        t[rank] = torch.tensor(loc, dtype=torch.float64)
        dist.all_reduce(t)
        allp = t.tolist()
        phase_ms = {}
        for i, bw in enumerate(pair):
            phase_ms[str(bw)] = {
                "search_ms_by_rank": [round(r[3 * i], 4) for r in allp],
                "gather_ms_by_rank": [round(r[3 * i + 1], 4) for r in allp],
                "merge_ms_rank0": round(allp[0][3 * i + 2], 4)}

    # e2e: queries from pinned host memory, the merged top-k back to the host
    # (ShardedGraph.search_host: page-locked buffers, see its docstring)
    q_host = queries.cpu().pin_memory()
    oi_host = torch.empty(args.nq, K, dtype=torch.int32).pin_memory()
    od_host = torch.empty(args.nq, K, dtype=torch.float32).pin_memory()
    e2e = {}
    for bw in pair:
        ts = []
        for it in range(max(args.steps, 10) + args.warmup):
            barrier()
            t1 = time.perf_counter()
            sg.search_host(q_host, oi_host, od_host, k=K, beam_width=bw, root=0)
            if it >= args.warmup:
                ts.append(time.perf_counter() - t1)
        e2e[bw] = float(np.median(ts)) * 1e3
    # the host results of the last call against the device-buffer search
    ref = sg.search(queries, k=K, beam_width=pair[-1], root=0) if ws > 1 else \
        sg.search_local(queries, k=K, beam_width=pair[-1])
    e2e_ok = None if ref is None else bool(
        torch.equal(oi_host, ref[0].cpu()) and
        torch.equal(od_host.view(torch.int32), ref[1].cpu().view(torch.int32)))
    e2e = dict(zip(pair, max_over_ranks(dist, [e2e[bw] for bw in pair], dev)))
    e2e_qps = {bw: args.nq / (e2e[bw] / 1e3) for bw in pair}
    e2e_value = interp_qps(recalls[lo], e2e_qps[lo], recalls[hi], e2e_qps[hi])
    sg.free()
    del queries, gi, gd
    torch.cuda.empty_cache()
    if rank != 0:
        return None
    return {
        "value": round(value, 1), "unit": "queries/s", "n_gpus": ws, "scaling": "weak",
        "ms_per_step": round(sum(ms.values()), 4),
        "workload": f"config5: range-sharded {n_total} x 128 SIFT-like fp16 ({ws} shards x "
                    f"{n_shard}), L2, R=64, alpha=1.2, {args.nq} queries broadcast, k=10, one "
                    "NCCL gather + device merge",
        "rows_per_gpu": n_shard, "bracket_beam_widths": list(pair),
        "recall_at_10": {str(b): round(r, 4) for b, r in recalls.items()},
        "qps": {str(b): round(v, 1) for b, v in qps.items()},
        "phases": phase_ms,
        "build": {"mvec_per_s": round(n_total / build_s / 1e6, 4), "seconds": round(build_s, 3),
                  "seconds_by_rank": [round(x, 3) for x in build_each],
                  "note": f"{ws} shards built concurrently; time = max over ranks"},
        "e2e": {"value": round(e2e_value, 1), "unit": "queries/s",
                "h2d_bytes_per_step": int(len(pair) * args.nq * 128 * 2),
                "d2h_bytes_per_step": int(len(pair) * args.nq * K * 8),
                "timing": ("median host wall time per query batch through "
                           "ShardedGraph.search_host (page-locked buffers; one shard: the "
                           "kernel reads the queries and writes the results in place; "
                           "several: upload, search on every shard, gather, merge, "
                           "download), max over ranks"),
                "identical_to_device_search": e2e_ok},
        "gpu_launches": args.steps * len(pair) * (2 if ws > 1 else 1),
        "clocks": clk.summary(),
    }


def run_sharded(args):
    """--mode sharded: the config-5 leg alone, as its own JSON line."""
    ws, rank, dist, dev = init_dist()
    r = sharded_leg(args, ws, rank, dist, dev)
    if rank == 0:
        line = {"metric": METRIC, "value": r["value"], "unit": r["unit"], "n_gpus": ws,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": r["ms_per_step"],
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "f16 rows, f32 distances", "data": "synthetic",
                "config": {"workload": r["workload"], "n_base": r["rows_per_gpu"] * ws,
                           "rows_per_gpu": r["rows_per_gpu"], "queries": args.nq,
                           "parallelism": f"range shards x{ws}",
                           "l2": "inputs larger than L2 (3.2 GB of rows per GPU)"}}
        line.update({k: v for k, v in r.items() if k not in line and k != "workload"})
        print(json.dumps(line), flush=True)
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
    gt = exact_ip_gt(X, Q, K)
    jasper.Graph.build(X[:50_000], n_neighbors=64, distance="ip", alpha=1.0,
                       build_rabitq=True).free()   # untimed warm-up (kernel loading)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    g = jasper.Graph.build(X, n_neighbors=64, distance="ip", alpha=1.0, build_rabitq=True)
    torch.cuda.synchronize()
    build_s = time.perf_counter() - t0
    line = {"mode": "rabitq", "config": "config4", "rows": n, "dim": 960,
            "build": {"seconds": round(build_s, 3), "mvec_per_s": round(n / build_s / 1e6, 4),
                      "note": "graph construction + prerotation + RaBitQ codes"}}
    from jasper_b200 import _lib
    for bw in (64, 128, 256, 512):
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
    g.free()
    for name in ("rabitq", "exact"):
        rec = {bw: line[f"{name}_bw{bw}"]["recall_at_10"] for bw in (64, 128, 256, 512)}
        qp = {bw: line[f"{name}_bw{bw}"]["qps"] for bw in (64, 128, 256, 512)}
        lo, hi = bracket(rec)
        line[f"{name}_qps_at_0.95"] = (round(interp_qps(rec[lo], qp[lo], rec[hi], qp[hi]), 1)
                                       if rec[hi] >= TARGET else None)
    if not args.no_cpu_baseline:
        line["cpu_baseline"] = bruteforce_baseline(X.cpu().numpy(), Q.cpu().numpy(), 1, gt.cpu(),
                                                   args)
    print(json.dumps(line), flush=True)


def bruteforce_baseline(base_np, q_np, metric, gt, args):
    """Exact brute-force k-NN on all host cores (oracle/bruteforce.c, fp16
    rows as fp32) over a bounded prefix of the queries."""
    from oracle import oracle as O
    cores = os.cpu_count() or 1
    b = base_np.astype(np.float32)
    q = q_np.astype(np.float32)
    t0 = time.perf_counter()
    O.bruteforce_knn(b, q[:cores], K, metric, threads=cores)
    est = cores / (time.perf_counter() - t0)
    m = int(min(q.shape[0], max(cores, est * args.cpu_seconds)))
    t0 = time.perf_counter()
    ids, _ = O.bruteforce_knn(b, q[:m], K, metric, threads=cores)
    qps = m / (time.perf_counter() - t0)
    return {"value": round(qps, 1), "unit": "queries/s", "cores": cores, "kind": "port",
            "algorithm": "exact brute-force k-NN (oracle/bruteforce.c), fp16 rows as fp32",
            "recall_at_10": round(recall_at_k(torch.from_numpy(ids), gt[:m]), 4),
            "sample": f"the first {m} of the {q.shape[0]} queries against all {b.shape[0]} rows "
                      f"(~{args.cpu_seconds:.0f} s), {cores} threads"}


def run_config1(args):
    """Config 1: 100k x 128 N(0,1) rows (seed 0), 1k queries (seed 1), L2,
    R = 32, alpha = 1.2, k = 10, beam widths 16..256 (the config names 64).
    The index (25.6 MB of rows + 12.8 MB of ids) stays in the 126 MB L2, so
    the search's bytes are set against an L2 read bandwidth measured here
    (a torch reduction over an L2-resident 48 MB buffer)."""
    import jasper_b200 as jasper
    from jasper_b200 import synthetic
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    X = synthetic.gaussian(100_000, 128, 0)
    Q = synthetic.gaussian(1000, 128, 1)
    Xd = torch.from_numpy(X).to(dev)
    Qd = torch.from_numpy(Q).to(dev)
    gt = exact_gt(Xd, Qd, K)
    jasper.Graph.build(Xd[:20_000], n_neighbors=32, distance="l2", alpha=1.2).free()  # warm-up
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    g = jasper.Graph.build(Xd, n_neighbors=32, distance="l2", alpha=1.2)
    torch.cuda.synchronize()
    build_s = time.perf_counter() - t0
    # L2 read bandwidth: sum over a 48 MB buffer that stays in L2
    buf = torch.ones(12 * 1024 * 1024, dtype=torch.float32, device=dev)
    for _ in range(5):
        buf.sum()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(50):
        buf.sum()
    b.record()
    torch.cuda.synchronize()
    l2_gbs = 50 * buf.numel() * 4 / (a.elapsed_time(b) / 1e3) / 1e9
    del buf
    line = {"mode": "config1", "config": "config1", "rows": 100_000, "dim": 128, "R": 32,
            "build": {"seconds": round(build_s, 3), "mvec_per_s": round(0.1 / build_s, 4)},
            "l2_read_gbs_measured": round(l2_gbs, 1)}
    for bw in BWS:
        ids, _ = g.search(Qd, k=K, beam_width=bw)
        qps, ms = _timed_qps(lambda: g.search(Qd, k=K, beam_width=bw), 1000, args.steps,
                             args.warmup)
        _, _, st = g.search_with_stats(Qd, k=K, beam_width=bw, distinct=True)
        st = st.long().cpu()
        bytes_q = (2 * 128 + st[:, 0] + 4 * st[:, 1] + 2 * 128 * st[:, 4] + 8 * K).sum().item()
        gbs = bytes_q / (ms / 1e3) / 1e9
        line[f"bw{bw}"] = {"recall_at_10": round(recall_at_k(ids, gt), 4), "qps": round(qps, 1),
                           "ms": round(ms, 4), "algorithmic_gbs": round(gbs, 1),
                           "frac_of_l2_read": round(gbs / l2_gbs, 4)}
    g.free()
    if not args.no_cpu_baseline:
        line["cpu_baseline"] = bruteforce_baseline(X, Q, 0, gt.cpu(), args)
    print(json.dumps(line), flush=True)


# ── reference arm ─────────────────────────────────────────────────────────
def ref_library(args):
    name = "libjasper_ffi_ndebug.so" if args.ref_ndebug else "libjasper_ffi.so"
    return ROOT / "oracle" / "_ref" / "lib" / name


def ref_plain_sweep(mod, cfg, base, queries, dim, alpha, bws, gt, args):
    """The reference's own build + search (tvm_ffi ops) for one plain config:
    build time (after one untimed warm-up build on the first 50k rows, as
    the other arm does), recall@10 per beam width, wall-clock QPS per width
    (its call includes its per-call cudaMalloc and stream sync), L2 flushed
    between timed calls.  Returns (build_s, recalls, qps, clocks)."""
    with stdout_to_stderr():
        mod.jasper_free_graph(getattr(mod, f"jasper_construct_{cfg}")(
            base[:50_000].contiguous(), dim, alpha, 10 * 10**9, False))
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    with stdout_to_stderr():
        h = getattr(mod, f"jasper_construct_{cfg}")(base, dim, alpha, 10 * 10**9, False)
    torch.cuda.synchronize()
    build_s = time.perf_counter() - t0
    search = getattr(mod, f"jasper_search_{cfg}")
    nq = queries.shape[0]
    oi = torch.empty(nq, K, dtype=torch.int32, device="cuda")
    od = torch.empty(nq, K, dtype=torch.float32, device="cuda")
    flush = torch.zeros(64 * 1024 * 1024, dtype=torch.float32, device="cuda")
    recalls, qps = {}, {}
    try:
        with ClockSampler(torch.device("cuda", torch.cuda.current_device())) as clk:
            for bw in bws:
                search(h, queries, oi, od, K, bw, 2 * bw, False)
                torch.cuda.synchronize()
                recalls[bw] = recall_at_k(oi, gt)
                for _ in range(args.warmup):
                    search(h, queries, oi, od, K, bw, 2 * bw, False)
                ts = []
                for _ in range(args.steps):
                    flush_l2(flush)
                    torch.cuda.synchronize()
                    t1 = time.perf_counter()
                    search(h, queries, oi, od, K, bw, 2 * bw, False)
                    torch.cuda.synchronize()
                    ts.append(time.perf_counter() - t1)
                qps[bw] = nq / float(np.mean(ts))
    finally:
        mod.jasper_free_graph(h)
    return build_s, recalls, qps, clk.summary()


def run_reference(args):
    """The reference's own CUDA implementation (unmodified sources compiled
    for sm_100a, oracle/_ref) through its tvm_ffi ops, on the config the
    other arm runs: config 2 by default, config 1 (--mode config1),
    config 4's plain inner-product search (--mode rabitq; the reference has
    no RaBitQ search), config 3 (--mode directional)."""
    ws, rank, local = dist_env()
    if rank != 0:
        return
    lib = ref_library(args)
    if not lib.exists():
        print(json.dumps({"impl": "reference", "unavailable":
                          f"reference library {lib.relative_to(ROOT)} was not built"}))
        return
    import tvm_ffi
    torch.cuda.set_device(local if ws > 1 else 0)
    mod = tvm_ffi.load_module(str(lib))
    variant = ("-DNDEBUG build (device asserts compiled out)" if args.ref_ndebug
               else "default build (device asserts on, as the reference ships)")
    if args.mode == "directional":
        return run_reference_directional(args, mod, variant)
    if args.mode == "config1":
        from jasper_b200 import synthetic
        base = torch.from_numpy(synthetic.gaussian(100_000, 128, 0)).cuda()
        queries = torch.from_numpy(synthetic.gaussian(1000, 128, 1)).cuda()
        cfg, dim, alpha, bws = "f16_r32_l2", 128, 1.2, BWS
        workload = ("config1: 100k x 128 N(0,1) fp16, L2, R=32, alpha=1.2, 1000 queries, k=10")
        gt = exact_gt(base, queries, K)
    elif args.mode == "rabitq":
        dev = torch.device("cuda", torch.cuda.current_device())
        base = gen_relu_sphere_gpu(args.n, 960, 256, 0.3, 6, 6, dev)
        queries = gen_relu_sphere_gpu(1000, 960, 256, 0.3, 7, 6, dev)
        cfg, dim, alpha, bws = "f16_r64_ip", 960, 1.0, (64, 128, 256, 512)
        workload = (f"config4 (plain IP search; the reference has no RaBitQ search): {args.n} x "
                    "960 ReLU-sphere fp16, IP, R=64, alpha=1.0, 1000 queries, k=10")
        gt = exact_ip_gt(base, queries, K)
    else:
        base_np, q_np = load_data(args.n, args.nq, 0)
        base = torch.from_numpy(base_np).cuda()
        queries = torch.from_numpy(q_np).cuda()
        cfg, dim, alpha, bws = "f16_r64_l2", 128, 1.2, BWS
        workload = ("config2: 1M x 128 SIFT-like fp16, L2, R=64, alpha=1.2, "
                    f"{args.nq} queries, k=10")
        gt = exact_gt(base, queries, K)
    nq = queries.shape[0]
    n = base.shape[0]
    build_s, recalls, qps, clk = ref_plain_sweep(mod, cfg, base, queries, dim, alpha, bws, gt,
                                                 args)
    lo, hi = bracket(recalls)
    pair = (lo, hi) if lo != hi else (hi,)
    reached = recalls[hi] >= TARGET
    value = interp_qps(recalls[lo], qps[lo], recalls[hi], qps[hi])
    ms = {bw: 1e3 * nq / qps[bw] for bw in pair}
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 1), "unit": "queries/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(sum(ms.values()), 4), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f16 rows, f32 distances", "data": "synthetic",
        "config": {"workload": workload, "n_base": n, "queries": nq,
                   "bracket_beam_widths": list(pair), "limit": "2*beam_width",
                   "parallelism": "single", "l2": "flushed between timed searches (256 MB write)",
                   "implementation": "unmodified reference CUDA sources (ffi/*.cu) compiled for "
                                     f"sm_100a by oracle/build_ref.sh, {variant}, called "
                                     "through its tvm_ffi ops"},
        "recall_at_10": {str(b): round(r, 4) for b, r in recalls.items()},
        "qps": {str(b): round(v, 1) for b, v in qps.items()},
        "recall_0.95_reached": reached,
        "build": {"mvec_per_s": round(n / build_s / 1e6, 4), "seconds": round(build_s, 3)},
        "cpu_baseline": {"value": round(value, 1), "unit": "queries/s", "cores": 0,
                         "kind": "reference",
                         "sample": "the reference ships no CPU search: this arm runs its own "
                                   "CUDA implementation on the B200 (wall clock incl. its "
                                   "per-call cudaMalloc and stream sync)"},
        "e2e": {"value": round(value, 1), "unit": "queries/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "clocks": clk,
    }
    print(json.dumps(line), flush=True)


def run_reference_directional(args, mod, variant):
    """Config 3 on the reference: its own prerotated directional build
    (seed 4) and PQ codebooks (k-means 20 iterations, seed 5; M = k_ranks,
    the only PQ the reference has); its LSH payload builder is not run (it
    stops on a failing device assert on this GPU), so the LSH payload is
    computed by the CPU restatement (oracle/directional.py) on the
    reference's own graph and rows.  Graph, payloads and PQ codebooks go
    into a legacy-layout directional file that the reference loads and
    searches with directional_search / pq_search."""
    import tempfile
    from jasper_b200 import synthetic
    from oracle import directional as D
    X = synthetic.gaussian(100_000, 128, 0)
    Q = synthetic.gaussian(1000, 128, 1)
    Xd = torch.from_numpy(X).cuda()
    Qd = torch.from_numpy(Q).cuda()
    gt = exact_gt(Xd, Qd, K)
    for kr in (4, 16):
        cfg = f"f16_r32_l2_k{kr}_d128"
        with stdout_to_stderr():
            h = getattr(mod, f"jasper_construct_directional_{cfg}")(Xd.clone(), 128, 1.2,
                                                                   10 * 10**9, False, True, 4)
            getattr(mod, f"jasper_build_pq_{cfg}")(h, 40000, 20, 5)
        with tempfile.TemporaryDirectory() as td:
            p1 = os.path.join(td, "g.graph")
            with stdout_to_stderr():
                getattr(mod, f"jasper_save_directional_{cfg}")(h, p1)
            mod.jasper_free_graph(h)
            rows, edges, edist, counts, medoid, pq = D.read_directional_file(p1, 128, 32)
            packed, mag = D.lsh_edges(rows, edges, counts, kr)
            c, nd = D.lsh_globals(rows, edges, counts, kr, n_samples=32768, seed=42)
            p2 = os.path.join(td, "legacy.graph")
            D.write_legacy_directional(p2, rows, edges, edist, counts, medoid, 32, kr, packed, mag,
                                       c, nd, pq["centroids"], pq["codes"], D.norms(rows))
            with stdout_to_stderr():
                h = getattr(mod, f"jasper_load_directional_{cfg}")(p2, 128, False, True, 4)
        try:
            flags = getattr(mod, f"jasper_get_directional_flags_{cfg}")(h)
            for name in ("directional_search", "pq_search"):
                fn = getattr(mod, f"jasper_{name}_{cfg}")
                line = {"impl": "reference", "mode": "directional", "config": "config3",
                        "estimator": "lsh" if name == "directional_search" else "pq",
                        "k_ranks" if name == "directional_search" else "pq_m": kr,
                        "flags": int(flags), "variant": variant}
                oi = torch.empty(1000, K, dtype=torch.int32, device="cuda")
                od = torch.empty(1000, K, dtype=torch.float32, device="cuda")
                for bw in (64, 128):
                    with stdout_to_stderr():
                        fn(h, Qd, oi, od, K, bw, 2 * bw, False)
                    torch.cuda.synchronize()
                    r = recall_at_k(oi, gt)
                    ts = []
                    for it in range(args.warmup + args.steps):
                        torch.cuda.synchronize()
                        t1 = time.perf_counter()
                        with stdout_to_stderr():
                            fn(h, Qd, oi, od, K, bw, 2 * bw, False)
                        torch.cuda.synchronize()
                        if it >= args.warmup:
                            ts.append(time.perf_counter() - t1)
                    line[f"bw{bw}"] = {"recall_at_10": round(r, 4),
                                       "qps": round(1000 / float(np.mean(ts)), 1)}
                print(json.dumps(line), flush=True)
        finally:
            mod.jasper_free_graph(h)


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
    ap.add_argument("--ref-ndebug", action="store_true",
                    help="--impl reference: use the -DNDEBUG build of the reference")
    ap.add_argument("--no-parity", action="store_true",
                    help="skip the parity check against the reference build (oracle/_ref)")
    ap.add_argument("--no-sharded", action="store_true",
                    help="skip the config-5 range-sharded leg of the default run")
    ap.add_argument("--mode", default="replicas",
                    choices=["replicas", "sharded", "rotation", "directional", "rabitq", "config1"],
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
    elif args.mode == "config1":
        run_config1(args)
    else:
        run_jasper(args)


if __name__ == "__main__":
    main()
