"""Build parity: jasper_b200's batched construction against the CPU
restatement, and both against graphs built by the reference's CUDA code.

The construction is deterministic in both implementations (same batch ramp,
same search, same (distance, id) candidate order, same RobustPrune), so the
adjacency must match exactly: ids, bf16 edge distances and counts.
"""
from pathlib import Path

import numpy as np
import pytest

from jasper_b200 import synthetic
from oracle import oracle as O
import jb_testlib as T

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"

CASES = [
    # kind, n, dim, R, metric, alpha
    ("gaussian", 3000, 128, 32, 0, 1.2),
    ("sift_like", 3000, 128, 64, 0, 1.2),
    ("gaussian", 2500, 96, 16, 0, 1.2),
    ("gaussian", 2000, 128, 32, 1, 1.0),
    ("gaussian", 1200, 40, 8, 0, 1.2),
    ("gaussian", 30, 16, 8, 0, 1.2),     # n < 50: one row per batch
    ("relu_sphere", 1500, 320, 32, 1, 1.0),
    # batches of 400 rows: hub targets collect more than 256 + R candidates
    ("sift_like", 20000, 128, 64, 0, 1.2),
    # exact duplicate rows (zero pair distances) and near ties on the prune
    # threshold: exercises the exact fallback of the Gram-filtered prune
    ("dup_sift", 4000, 128, 32, 0, 1.2),
    ("dup_sift", 3000, 64, 16, 1, 1.0),
    # rows near the fp16 limit, large-norm near-duplicates and three scales
    # in one candidate list: where the Gram filter's error band is thinnest
    ("adversarial", 3000, 128, 32, 0, 1.2),
    ("adversarial", 2000, 64, 16, 1, 1.0),
]


def adversarial(n, dim, seed):
    """Thirds of the rows at three scales: uniform in +-60000 (squared
    norms near 4.6e11 at 128 dims), in +-64 and in +-0.01; a quarter of the
    rows are near-duplicates of another row of their scale (a few
    coordinates moved by one or two fp16 steps), in shuffled order."""
    rng = np.random.default_rng(seed)
    scales = np.array([60000.0, 64.0, 0.01])
    X = (rng.uniform(-1.0, 1.0, size=(n, dim)) * scales[np.arange(n) % 3, None]).astype(np.float16)
    dup = rng.random(n) < 0.25
    src = rng.integers(0, n, size=n)
    src = src - (src % 3) + (np.arange(n) % 3)          # same scale as the copy
    src = np.minimum(src, n - 1)
    X[dup] = X[src[dup]]
    bits = X.view(np.uint16)
    for i in np.flatnonzero(dup):
        cols = rng.integers(0, dim, size=3)
        bits[i, cols] = bits[i, cols] + rng.integers(1, 3, size=3).astype(np.uint16)
    X = bits.view(np.float16)
    assert np.isfinite(X.astype(np.float32)).all()
    return X[rng.permutation(n)]


def dup_sift(n, dim, seed):
    """sift_like rows, each repeated four times (some with one coordinate
    nudged by one step), in shuffled order."""
    base = synthetic.sift_like((n + 3) // 4, dim, seed)
    X = np.repeat(base, 4, axis=0)[:n].copy()
    rng = np.random.default_rng(seed)
    nudge = rng.random(n) < 0.3
    cols = rng.integers(0, dim, size=n)
    X[nudge, cols[nudge]] += np.float16(1.0)
    return X[rng.permutation(n)]


def assert_graph_equal(e, d, c, g, msg=""):
    np.testing.assert_array_equal(c, g.counts, err_msg=msg)
    for i in range(g.n):
        k = int(c[i])
        np.testing.assert_array_equal(e[i, :k], g.edges[i, :k], err_msg=f"{msg} row {i}")
        np.testing.assert_array_equal(d[i, :k], g.edist[i, :k], err_msg=f"{msg} row {i}")


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"{c[0]}-n{c[1]}-d{c[2]}-R{c[3]}-m{c[4]}")
def test_build_matches_oracle(cuda, case):
    kind, n, dim, R, metric, alpha = case
    if kind == "dup_sift":
        X = dup_sift(n, dim, 31)
    elif kind == "adversarial":
        X = adversarial(n, dim, 31)
    else:
        X = getattr(synthetic, kind)(n, dim, 31)
    budget = 10 * 10**9
    g = O.OracleGraph(X, R, metric=metric)
    g.build(alpha, max(1, O.reference_max_batch_size(budget, n, R)))
    h = T.construct(X, R, metric, alpha, budget)
    try:
        e, d, c = T.get_edges(h, n, R)
        assert_graph_equal(e, d, c, g, msg=str(case))
    finally:
        T.free(h)


def golden_cases():
    return sorted(GOLDEN.glob("*.npz"))


@pytest.mark.parametrize("path", golden_cases(), ids=lambda p: p.stem)
def test_golden_build_and_search_match_reference(cuda, path):
    from test_oracle import regen
    z = np.load(path)
    X, Q = regen(z)
    R = int(z["R"])
    metric = 0 if str(z["metric"]) == "l2" else 1
    h = T.construct(X, R, metric, float(z["alpha"]))
    try:
        e, d, c = T.get_edges(h, int(z["n"]), R)
        ref = O.OracleGraph(X, R, metric=metric, medoid=int(z["medoid"]))
        ref.edges[:] = z["edges"]
        ref.edist[:] = z["dists"]
        ref.counts[:] = z["counts"]
        assert_graph_equal(e, d, c, ref, msg=path.stem)
    finally:
        T.free(h)
    # search on the reference's own graph
    h = T.create_graph(ref)
    try:
        for bw in z["bws"]:
            bw = int(bw)
            ji, jd = T.search(h, Q, 10, bw)
            T.assert_same_results(ji, jd, z[f"idx_bw{bw}"], z[f"dist_bw{bw}"], msg=f"bw={bw}")
    finally:
        T.free(h)
