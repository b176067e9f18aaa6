"""Golden fixtures for directional (LSH / PQ) search from the reference's CUDA build.

Runs on a GPU box with oracle/_ref/lib/libjasper_ffi.so.  The reference's own
LSH builder cannot be run here: populate_lsh walks all R edge slots
(include/jasper/lsh/lsh_kernels.cuh:46-49) and, in the shipped assert-enabled
build, trips the device assert `neighbor_idx < edge_counts` of
graph_segment::get_neighbor (include/jasper/index/graph.cuh:426) on any node
with fewer than R edges.  So the graph is built by jasper_b200 (bit-identical
to the reference's construction), the LSH / PQ / norm artifacts are computed
by the numpy restatement in oracle/directional.py, and everything is written
as a directional file whose base section uses the legacy record layout -- the
layout at which the reference's loader (graph.cuh:1961-1964) looks for the
trailer.  The reference then loads that file (jasper_load_directional_<cfg>,
prerotate off) and answers directional_search and pq_search; those answers,
with the artifacts, are the fixture.

    python tests/golden/make_golden_directional.py [out_dir]
"""
from __future__ import annotations

import hashlib
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

from jasper_b200.synthetic import gaussian, relu_sphere  # noqa: E402

# name: (generator, n, dim, nq, seed_base, seed_q, R, metric, k_ranks, alpha, bws)
CASES = {
    "dir_l2_r32_k4": (gaussian, 3000, 128, 150, 20, 21, 32, "l2", 4, 1.2, (64, 128)),
    "dir_ip_r32_k16": (relu_sphere, 3000, 128, 150, 22, 23, 32, "ip", 16, 1.0, (64,)),
    "dir_l2_r64_k16_d256": (gaussian, 2000, 256, 100, 24, 25, 64, "l2", 16, 1.2, (64,)),
}
BUDGET = 10 * 10**9


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def main(out_dir: str) -> None:
    import ctypes as C
    import torch
    import tvm_ffi
    from oracle import directional as D
    import jb_testlib as T

    out = Path(out_dir)
    out.mkdir(parents=True, exist_ok=True)
    mod = tvm_ffi.load_module(str(ROOT / "oracle" / "_ref" / "lib" / "libjasper_ffi.so"))
    tmp = Path(tempfile.mkdtemp())
    for name, (gen, n, dim, nq, sb, sq, R, metric, kr, alpha, bws) in CASES.items():
        X = gen(n, dim, sb)
        Q = gen(nq, dim, sq) if gen is gaussian else gen(nq, dim, sq, center_seed=sb)
        m = 0 if metric == "l2" else 1
        h = T.construct(X, R, m, alpha)
        edges, edist, counts = T.get_edges(h, n, R)
        T.free(h)
        packed, mag = D.lsh_edges(X, edges, counts, kr)
        c, nd = D.lsh_globals(X, edges, counts, kr, n_samples=4096, seed=42)
        cent = D.pq_train(X, edges, counts, kr, n_train=4096, iters=6, seed=123)
        codes = D.pq_codes(X, edges, counts, cent)
        nrm = D.norms(X)
        cfg = f"f16_r{R}_{metric}_k{kr}_{'d128' if dim <= 128 else 'd32678'}"
        path = tmp / f"{name}.graph"
        D.write_legacy_directional(str(path), X, edges, edist, counts, 0, R, kr, packed, mag, c,
                                   nd, cent, codes, nrm)
        h = getattr(mod, f"jasper_load_directional_{cfg}")(str(path), dim, False, False, 42)
        flags = getattr(mod, f"jasper_get_directional_flags_{cfg}")(h)
        assert flags == 3, flags
        res = {}
        qt = torch.from_numpy(Q.copy()).cuda()
        for kind in ("directional_search", "pq_search"):
            for bw in bws:
                oi = torch.empty(nq, 10, dtype=torch.int32, device="cuda")
                od = torch.empty(nq, 10, dtype=torch.float32, device="cuda")
                getattr(mod, f"jasper_{kind}_{cfg}")(h, qt, oi, od, 10, bw, 2 * bw, False)
                torch.cuda.synchronize()
                res[f"{kind}_idx_bw{bw}"] = oi.cpu().numpy()
                res[f"{kind}_dist_bw{bw}"] = od.cpu().numpy()
        mod.jasper_free_graph(h)
        np.savez_compressed(out / f"{name}.npz", n=n, dim=dim, nq=nq, seed_base=sb,
                            seed_queries=sq, R=R, metric=metric, k_ranks=kr, alpha=alpha,
                            bws=np.array(bws), x_sha=sha(X), q_sha=sha(Q),
                            generator=gen.__name__, medoid=0, counts=counts, edges=edges,
                            dists=edist, lsh_packed=packed, lsh_mag_sq=mag, lsh_c=c,
                            lsh_norm_denom=nd, pq_centroids=cent, pq_codes=codes, norms=nrm,
                            **res)
        print("wrote", name, flush=True)


if __name__ == "__main__":
    sys.path.insert(0, str(ROOT / "tests"))
    main(sys.argv[1] if len(sys.argv) > 1 else str(HERE))
