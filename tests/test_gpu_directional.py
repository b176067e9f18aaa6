"""Directional (LSH / PQ) search parity: the CUDA kernel against the CPU
restatement (bit for bit) on graphs with restated artifacts, and against the
reference's own directional_search / pq_search outputs (golden fixtures)."""
from pathlib import Path

import numpy as np
import pytest

from jasper_b200 import synthetic
from oracle import oracle as O
from oracle import directional as D
import jb_testlib as T

pytestmark = pytest.mark.gpu
DIR_GOLDEN = Path(__file__).resolve().parent / "golden" / "directional"


@pytest.mark.parametrize("path", sorted(DIR_GOLDEN.glob("*.npz")), ids=lambda p: p.stem)
def test_directional_matches_reference_golden(cuda, path):
    from test_oracle import regen, oracle_from_golden
    z = np.load(path)
    X, Q = regen(z)
    g = oracle_from_golden(z, X)
    h = T.create_graph(g)
    try:
        T.set_artifacts(h, z, int(z["k_ranks"]))
        for kind, key in (("lsh", "directional_search"), ("pq", "pq_search")):
            for bw in z["bws"]:
                bw = int(bw)
                ji, jd = T.dir_search(h, kind, Q, 10, bw)
                T.assert_same_results(ji, jd, z[f"{key}_idx_bw{bw}"], z[f"{key}_dist_bw{bw}"],
                                      msg=f"{kind} bw={bw}")
    finally:
        T.free(h)


CASES = [
    # kind of data, n, dim, R, metric, k_ranks
    ("gaussian", 2500, 128, 32, 0, 4),
    ("gaussian", 2000, 96, 16, 0, 16),
    ("relu_sphere", 2000, 128, 32, 1, 4),
    ("gaussian", 1500, 256, 64, 0, 4),
    ("gaussian", 1500, 192, 32, 1, 16),
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"{c[0]}-d{c[2]}-R{c[3]}-m{c[4]}-k{c[5]}")
def test_directional_matches_oracle(cuda, case):
    kind_data, n, dim, R, metric, kr = case
    X = getattr(synthetic, kind_data)(n, dim, 61)
    gen = getattr(synthetic, kind_data)
    Q = gen(80, dim, 62) if kind_data == "gaussian" else gen(80, dim, 62, center_seed=61)
    g = O.OracleGraph(X, R, metric=metric)
    g.build(1.2 if metric == 0 else 1.0, max(1, n // 50))
    packed, mag = D.lsh_edges(X, g.edges, g.counts, kr)
    c, nd = D.lsh_globals(X, g.edges, g.counts, kr, n_samples=2048)
    cent = D.pq_train(X, g.edges, g.counts, kr, n_train=1024, iters=3)
    codes = D.pq_codes(X, g.edges, g.counts, cent)
    art = dict(lsh_packed=packed, lsh_mag_sq=mag, lsh_c=c, lsh_norm_denom=nd,
               pq_centroids=cent, pq_codes=codes, norms=D.norms(X), k_ranks=kr)
    h = T.create_graph(g)
    try:
        T.set_artifacts(h, art, kr)
        for kind in ("lsh", "pq"):
            for k, bw, limit in [(10, 64, 128), (10, 16, 32), (40, 24, 48), (10, 200, 400)]:
                oi, od = O.dir_search(g, kind, art, Q, k, bw, limit)
                ji, jd = T.dir_search(h, kind, Q, k, bw, limit)
                T.assert_same_results(ji, jd, oi, od, msg=f"{kind} k={k} bw={bw}")
    finally:
        T.free(h)


def test_directional_requires_artifacts(cuda):
    X = synthetic.gaussian(300, 32, 63)
    h = T.construct(X, 16, 0, 1.2)
    try:
        with pytest.raises(Exception, match="no LSH"):
            T.dir_search(h, "lsh", X[:4], 10, 16)
        with pytest.raises(Exception, match="no PQ"):
            T.dir_search(h, "pq", X[:4], 10, 16)
    finally:
        T.free(h)
