"""The CPU restatement (oracle/) pinned against the reference's own answers.

* known-answer distances of the reference's gtest suite
  (tests/test_distance.cu:32-136), through the same summation order;
* the golden fixtures written by the reference's CUDA build
  (tests/golden/make_golden.py): the oracle must reproduce the reference's
  search results on the reference's graph, and the reference's graph from the
  same rows;
* self-consistency: on a fully connected graph the beam search is exact kNN.
"""
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O
from jasper_b200 import synthetic

GOLDEN = Path(__file__).resolve().parent / "golden"


# ── tests/test_distance.cu known answers (float rows, 4-lane tile) ─────────
def test_l2_identical_is_zero():
    assert O.distance_f32(0, [1, 2, 3, 4], [1, 2, 3, 4], 4) == 0.0


def test_l2_known_distance():
    assert O.distance_f32(0, [0, 0, 0, 0], [3, 4, 0, 0], 4) == 25.0


def test_l2_larger_dim():
    assert O.distance_f32(0, [1.0] * 16, [0.0] * 16, 16) == 16.0


def test_l2_symmetric():
    a, b = [1, 2, 3, 4], [5, 6, 7, 8]
    assert O.distance_f32(0, a, b, 4) == O.distance_f32(0, b, a, 4)


def test_ip_orthogonal_zero():
    assert abs(O.distance_f32(1, [1, 0, 0, 0], [0, 1, 0, 0], 4)) == 0.0


def test_ip_known_value():
    assert O.distance_f32(1, [1, 2, 3, 4], [2, 3, 4, 5], 4) == -40.0


def test_ip_self_dot_negative():
    assert O.distance_f32(1, [3, 4, 0, 0], [3, 4, 0, 0], 2) == -25.0


def test_fp16_distance_matches_float64_on_exact_values():
    rng = np.random.default_rng(0)
    a = rng.integers(0, 256, 128).astype(np.float16)
    b = rng.integers(0, 256, 128).astype(np.float16)
    exact = float(((a.astype(np.float64) - b.astype(np.float64)) ** 2).sum())
    assert O.distance_f16(0, a, b) == exact  # integer terms: exact in any order
    assert O.distance_f16(1, a, b) == -float((a.astype(np.float64) * b).sum())


def test_bf16_rounding_is_nearest_even():
    import ctypes
    L = O.lib()
    for f in [1.0, 1.00390625, 1.005859375, 3.14159, -2.5e-3, 65504.0, 1e30]:
        got = L.orc_float_to_bf16(ctypes.c_float(f))
        u = np.array([f], np.float32).view(np.uint32)[0]
        lsb = (u >> 16) & 1
        want = ((int(u) + 0x7FFF + int(lsb)) >> 16) & 0xFFFF
        assert got == want


# ── self-consistency ─────────────────────────────────────────────────────
def test_complete_graph_search_is_exact_knn():
    rng = np.random.default_rng(1)
    n = 64
    X = rng.standard_normal((n, 16)).astype(np.float16)
    Q = rng.standard_normal((20, 16)).astype(np.float16)
    g = O.OracleGraph(X, 64)
    for i in range(n):
        nb = [j for j in range(n) if j != i]
        g.edges[i, :len(nb)] = nb
        g.counts[i] = len(nb)
    oi, od, _, _ = g.search(Q, 10, 64, 128)
    bi, bd = O.bruteforce(X, Q, 10)
    np.testing.assert_array_equal(oi, bi)
    np.testing.assert_array_equal(od, bd)


def test_empty_graph_returns_sentinels():
    X = np.zeros((1, 8), np.float16)
    g = O.OracleGraph(X, 8)
    oi, od, _, _ = g.search(np.ones((2, 8), np.float16), 5, 16, 32)
    assert (oi[:, 0] == 0).all() and (oi[:, 1:] == -1).all()
    assert (od[:, 1:] == np.float32(1e30)).all()


def test_build_small_is_connected_and_degree_bounded():
    X = synthetic.gaussian(500, 32, 5)
    g = O.OracleGraph(X, 16)
    g.build(1.2, 10)
    assert g.counts.max() <= 16 and g.counts.min() >= 1
    Q = synthetic.gaussian(50, 32, 6)
    oi, _, _, _ = g.search(Q, 10, 64, 128)
    bi, _ = O.bruteforce(X, Q, 10)
    rec = np.mean([len(set(oi[i]) & set(bi[i])) / 10 for i in range(50)])
    assert rec > 0.9


# ── golden fixtures from the reference's CUDA build ─────────────────────
def golden_cases():
    return sorted(GOLDEN.glob("*.npz"))


def regen(z):
    gen = getattr(synthetic, str(z["generator"]))
    n, dim, nq = int(z["n"]), int(z["dim"]), int(z["nq"])
    sb, sq = int(z["seed_base"]), int(z["seed_queries"])
    X = gen(n, dim, sb)
    Q = gen(nq, dim, sq) if gen is synthetic.gaussian else gen(nq, dim, sq, center_seed=sb)
    import hashlib
    assert hashlib.sha256(X.tobytes()).hexdigest() == str(z["x_sha"]), "base rows differ"
    assert hashlib.sha256(Q.tobytes()).hexdigest() == str(z["q_sha"]), "queries differ"
    return X, Q


def oracle_from_golden(z, X):
    metric = 0 if str(z["metric"]) == "l2" else 1
    g = O.OracleGraph(X, int(z["R"]), metric=metric, medoid=int(z["medoid"]))
    g.edges[:] = z["edges"]
    g.edist[:] = z["dists"]
    g.counts[:] = z["counts"]
    return g


@pytest.mark.parametrize("path", golden_cases(), ids=lambda p: p.stem)
def test_golden_search_oracle_matches_reference(path):
    z = np.load(path)
    X, Q = regen(z)
    g = oracle_from_golden(z, X)
    for bw in z["bws"]:
        bw = int(bw)
        oi, od, _, _ = g.search(Q, 10, bw, 2 * bw)
        ri, rd = z[f"idx_bw{bw}"], z[f"dist_bw{bw}"]
        np.testing.assert_array_equal(oi, ri, err_msg=f"bw={bw}")
        np.testing.assert_array_equal(od.view(np.uint32), rd.view(np.uint32), err_msg=f"bw={bw}")


def golden_graph_equal(g, z):
    """Edge lists equal up to the reference's uninitialised slots >= count."""
    np.testing.assert_array_equal(g.counts, z["counts"])
    for i in range(g.n):
        c = int(g.counts[i])
        np.testing.assert_array_equal(g.edges[i, :c], z["edges"][i, :c], err_msg=f"row {i}")
        np.testing.assert_array_equal(g.edist[i, :c], z["dists"][i, :c], err_msg=f"row {i}")


@pytest.mark.parametrize("path", golden_cases(), ids=lambda p: p.stem)
def test_golden_build_oracle_matches_reference(path):
    z = np.load(path)
    X, _ = regen(z)
    metric = 0 if str(z["metric"]) == "l2" else 1
    g = O.OracleGraph(X, int(z["R"]), metric=metric)
    g.build(float(z["alpha"]), O.reference_max_batch_size(10 * 10**9, int(z["n"]), int(z["R"])))
    golden_graph_equal(g, z)


# ── directional fixtures (reference search on restated artifacts) ───────
DIR_GOLDEN = GOLDEN / "directional"


def dir_cases():
    return sorted(DIR_GOLDEN.glob("*.npz"))


@pytest.mark.parametrize("path", dir_cases(), ids=lambda p: p.stem)
def test_golden_directional_oracle_matches_reference(path):
    z = np.load(path)
    X, Q = regen(z)
    g = oracle_from_golden(z, X)
    for kind, key in (("lsh", "directional_search"), ("pq", "pq_search")):
        for bw in z["bws"]:
            bw = int(bw)
            oi, od = O.dir_search(g, kind, z, Q, 10, bw, 2 * bw)
            np.testing.assert_array_equal(oi, z[f"{key}_idx_bw{bw}"], err_msg=f"{kind} bw={bw}")
            np.testing.assert_array_equal(od.view(np.uint32), z[f"{key}_dist_bw{bw}"].view(np.uint32),
                                          err_msg=f"{kind} bw={bw}")


def test_oracle_append_wires_new_rows():
    """orc_append_range (append_batch, construct.cuh:1169-1265): appended
    rows get edges and are found by a search for themselves; ids continue
    the slot sequence."""
    from jasper_b200 import synthetic
    X = synthetic.gaussian(1600, 32, 95)
    g = O.OracleGraph(X[:1200], 16)
    g.build(1.2, 24)
    ids = g.append(X[1200:], 1.2)
    np.testing.assert_array_equal(ids, np.arange(1200, 1600))
    assert g.n == 1600 and (g.counts[1200:] > 0).all()
    # appended rows find themselves about as often as the built rows do
    base, _, _, _ = g.search(X[:400], 1, 32, 64)
    oi, _, _, _ = g.search(X[1200:], 1, 32, 64)
    assert np.mean(oi[:, 0] == np.arange(1200, 1600)) >= np.mean(base[:, 0] == np.arange(400)) - 0.03
