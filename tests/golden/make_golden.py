"""Generate golden fixtures from the reference's own CUDA build.

Runs on a GPU box with oracle/_ref/lib/libjasper_ffi.so (built from the
unmodified reference sources by oracle/build_ref.sh).  It calls the
reference's tvm_ffi ops exactly as the reference Python package does
(python/jasper/__init__.py:399-403, 504-507): construct, save, search with
limit = 2 * beam_width.  Outputs tests/golden/<case>.npz (adjacency of the
reference-built graph and its search results) and, for the file-format case,
the raw graph file the reference wrote.

Inputs are regenerated from seeds (see CASES); each fixture stores the
SHA-256 of its fp16 inputs so a test can prove it rebuilt the same data.

    python tests/golden/make_golden.py [out_dir]
"""
from __future__ import annotations

import hashlib
import struct
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

from jasper_b200.synthetic import gaussian, sift_like  # noqa: E402

# name: (generator, n, dim, n_queries, seed_base, seed_queries, R, metric, alpha, beam widths)
CASES = {
    "gauss_l2_r32": (gaussian, 3000, 128, 200, 10, 11, 32, "l2", 1.2, (16, 64, 128)),
    "int_l2_r64": (sift_like, 3000, 128, 200, 12, 13, 64, "l2", 1.2, (32, 64)),
    "gauss_ip_r32": (gaussian, 2000, 96, 100, 14, 15, 32, "ip", 1.0, (64,)),
}
FILE_CASE = ("gauss_l2_r16_file", gaussian, 600, 32, 16, 16, "l2", 1.2)
BUDGET = 10 * 10**9


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def parse_graph_file(path: str, dim: int, R: int):
    """Read the reference's current layout (graph.cuh:1653-1788)."""
    raw = Path(path).read_bytes()
    total, n, medoid, bpn = struct.unpack_from("<4Q", raw, 0)
    assert bpn == 2 * dim + 1 + 6 * R + 4, (bpn, dim, R)
    rec = np.frombuffer(raw, dtype=np.uint8, count=n * bpn, offset=32).reshape(n, bpn)
    o = 2 * dim
    counts = rec[:, o].copy()
    edges = rec[:, o + 1:o + 1 + 4 * R].copy().view("<u4").reshape(n, R)
    dists = rec[:, o + 1 + 4 * R:o + 1 + 6 * R].copy().view("<u2").reshape(n, R)
    ids = rec[:, o + 1 + 6 * R:o + 5 + 6 * R].copy().view("<u4").reshape(n)
    return dict(n=n, medoid=medoid, total=total, counts=counts, edges=edges, dists=dists, ids=ids)


def main(out_dir: str) -> None:
    import torch
    import tvm_ffi

    out = Path(out_dir)
    out.mkdir(parents=True, exist_ok=True)
    mod = tvm_ffi.load_module(str(ROOT / "oracle" / "_ref" / "lib" / "libjasper_ffi.so"))
    tmp = Path(tempfile.mkdtemp())
    for name, (gen, n, dim, nq, sb, sq, R, metric, alpha, bws) in CASES.items():
        X = gen(n, dim, sb)
        Q = gen(nq, dim, sq) if gen is gaussian else gen(nq, dim, sq, center_seed=sb)
        cfg = f"f16_r{R}_{metric}"
        xt = torch.from_numpy(X.copy()).cuda()
        h = getattr(mod, f"jasper_construct_{cfg}")(xt, dim, alpha, BUDGET, False)
        gpath = tmp / f"{name}.graph"
        getattr(mod, f"jasper_save_{cfg}")(h, str(gpath))
        gr = parse_graph_file(str(gpath), dim, R)
        res = {}
        qt = torch.from_numpy(Q.copy()).cuda()
        for bw in bws:
            oi = torch.empty(nq, 10, dtype=torch.int32, device="cuda")
            od = torch.empty(nq, 10, dtype=torch.float32, device="cuda")
            getattr(mod, f"jasper_search_{cfg}")(h, qt, oi, od, 10, bw, 2 * bw, False)
            torch.cuda.synchronize()
            res[f"idx_bw{bw}"] = oi.cpu().numpy()
            res[f"dist_bw{bw}"] = od.cpu().numpy()
        mod.jasper_free_graph(h)
        np.savez_compressed(out / f"{name}.npz", n=n, dim=dim, nq=nq, seed_base=sb, seed_queries=sq,
                            R=R, metric=metric, alpha=alpha, bws=np.array(bws),
                            x_sha=sha(X), q_sha=sha(Q), generator=gen.__name__,
                            medoid=gr["medoid"], counts=gr["counts"], edges=gr["edges"],
                            dists=gr["dists"], **res)
        print("wrote", name, "mean degree", gr["counts"].mean())
    # raw file written by the reference, for the loader test
    name, gen, n, dim, R, sb, metric, alpha = FILE_CASE
    X = gen(n, dim, sb)
    cfg = f"f16_r{R}_{metric}"
    h = getattr(mod, f"jasper_construct_{cfg}")(torch.from_numpy(X.copy()).cuda(), dim, alpha,
                                                 BUDGET, False)
    getattr(mod, f"jasper_save_{cfg}")(h, str(out / f"{name}.graph"))
    mod.jasper_free_graph(h)
    print("wrote", name)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else str(HERE))
