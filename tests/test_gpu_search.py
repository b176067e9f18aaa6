"""Search parity: jasper_b200's CUDA search against the CPU restatement.

Both run on the same graph and queries; ids and distances must agree bit for
bit (the kernel reproduces the reference's fp32 summation order and its
(distance, id) ordering).  Graphs are built by the oracle so the test does not
depend on the GPU build.
"""
import numpy as np
import pytest

from jasper_b200 import synthetic
from oracle import oracle as O
import jb_testlib as T

pytestmark = pytest.mark.gpu


@pytest.fixture(params=[1, 4], ids=["warp_per_query", "cta_per_query"], autouse=True)
def kernel_mode(request, cuda):
    """Every test runs on both query-search kernels (jb_search_set_warps_per_query:
    1 = a warp per query, 4 = a CTA per query)."""
    from jasper_b200 import _lib
    _lib.call("jb_search_set_warps_per_query", request.param)
    yield request.param
    _lib.call("jb_search_set_warps_per_query", 0)

_GRAPHS = {}


def oracle_graph(kind, n, dim, R, metric, alpha, seed):
    key = (kind, n, dim, R, metric, alpha, seed)
    if key not in _GRAPHS:
        X = getattr(synthetic, kind)(n, dim, seed)
        g = O.OracleGraph(X, R, metric=metric)
        g.build(alpha, max(1, n // 50))
        _GRAPHS[key] = (X, g)
    return _GRAPHS[key]


def queries(kind, nq, dim, seed, base_seed):
    gen = getattr(synthetic, kind)
    return gen(nq, dim, seed) if kind == "gaussian" else gen(nq, dim, seed, center_seed=base_seed)


CASES = [
    # kind, n, dim, R, metric, alpha, bws
    ("gaussian", 4000, 128, 32, 0, 1.2, (16, 32, 64, 128, 256)),
    ("sift_like", 4000, 128, 64, 0, 1.2, (16, 64, 128)),
    ("gaussian", 3000, 96, 16, 0, 1.2, (32, 64)),
    ("gaussian", 2000, 200, 32, 0, 1.2, (64,)),
    ("gaussian", 2000, 40, 8, 0, 1.2, (64,)),
    ("gaussian", 2000, 128, 32, 1, 1.0, (64, 128)),
    ("relu_sphere", 2000, 320, 32, 1, 1.0, (64,)),
    ("gaussian", 1500, 512, 64, 0, 1.2, (64,)),
    ("relu_sphere", 1500, 960, 32, 1, 1.0, (64, 128)),
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"{c[0]}-n{c[1]}-d{c[2]}-R{c[3]}-m{c[4]}")
def test_search_matches_oracle(cuda, case):
    kind, n, dim, R, metric, alpha, bws = case
    X, g = oracle_graph(kind, n, dim, R, metric, alpha, 21)
    Q = queries(kind, 150, dim, 22, 21)
    h = T.create_graph(g)
    try:
        for bw in bws:
            oi, od, _, _ = g.search(Q, 10, bw, 2 * bw)
            ji, jd = T.search(h, Q, 10, bw)
            T.assert_same_results(ji, jd, oi, od, msg=f"bw={bw}")
    finally:
        T.free(h)


def test_k_larger_than_beam_and_odd_limits(cuda):
    X, g = oracle_graph("gaussian", 4000, 128, 32, 0, 1.2, 21)
    Q = queries("gaussian", 64, 128, 23, 21)
    h = T.create_graph(g)
    try:
        for k, bw, limit in [(40, 16, 32), (1, 8, 0), (10, 64, 7), (100, 256, 600), (10, 1000, 2000)]:
            oi, od, _, _ = g.search(Q, k, bw, limit)
            ji, jd = T.search(h, Q, k, bw, limit)
            T.assert_same_results(ji, jd, oi, od, msg=f"k={k} bw={bw} limit={limit}")
    finally:
        T.free(h)


def test_deleted_rows_are_skipped(cuda):
    import ctypes as C
    from jasper_b200 import _lib
    X, g = oracle_graph("gaussian", 4000, 128, 32, 0, 1.2, 21)
    Q = queries("gaussian", 100, 128, 24, 21)
    h = T.create_graph(g)
    try:
        ji, _ = T.search(h, Q, 10, 64)
        dead = np.unique(ji[:, :3].ravel()).astype(np.int32)
        _lib.call("jb_graph_mark_deleted", h, dead.ctypes.data, dead.size)
        words = np.zeros((g.n + 31) // 32, np.uint32)
        for i in dead:
            words[i >> 5] |= np.uint32(1 << (int(i) & 31))
        g.deleted = words
        try:
            oi, od, _, _ = g.search(Q, 10, 64, 128)
        finally:
            g.deleted = None
        ji2, jd2 = T.search(h, Q, 10, 64)
        T.assert_same_results(ji2, jd2, oi, od)
        assert not np.isin(ji2, dead).any()
    finally:
        T.free(h)


def test_global_offset_shard(cuda):
    """A shard holding ids [off, off + n) searches like the local graph."""
    off = 1_000_000
    X, g = oracle_graph("gaussian", 3000, 96, 16, 0, 1.2, 21)
    Q = queries("gaussian", 80, 96, 25, 21)
    h = T.create_graph(g)
    from jasper_b200 import _lib
    try:
        _lib.call("jb_graph_apply_global_offset", h, off)
        gi = O.OracleGraph(X, g.R, medoid=off, global_offset=off)
        gi.edges[:] = np.where(g.edges == 0xFFFFFFFF, g.edges, g.edges + off)
        gi.edist[:] = g.edist
        gi.counts[:] = g.counts
        oi, od, _, _ = gi.search(Q, 10, 64, 128)
        ji, jd = T.search(h, Q, 10, 64)
        T.assert_same_results(ji, jd, oi, od)
        assert (ji >= off).all()
    finally:
        T.free(h)


def test_stats_count_expansions(cuda):
    X, g = oracle_graph("gaussian", 4000, 128, 32, 0, 1.2, 21)
    Q = queries("gaussian", 50, 128, 26, 21)
    h = T.create_graph(g)
    try:
        _, _, ne, _ = g.search(Q, 10, 64, 128)
        _, _, st = T.search(h, Q, 10, 64, stats=True)
        np.testing.assert_array_equal(st[:, 0], ne)
    finally:
        T.free(h)
