"""Directional payload builders on the GPU (LSH sketches + calibration, PQ
codebooks + codes, exact norms), prerotated construction and the directional
file trailer.

Exact parts (edge sketches, magnitudes, codes for given centroids, norms) are
compared bit for bit with the CPU restatement; the sampled parts (LSH
calibration, k-means codebooks) are random by design in the reference too
(cuRAND sampling, float atomics) and are checked against population
statistics with the tolerances stated in each test."""
import ctypes as C
from pathlib import Path

import numpy as np
import pytest

from jasper_b200 import _lib, synthetic
from oracle import oracle as O
from oracle import directional as D
import jb_testlib as T

pytestmark = pytest.mark.gpu
DIR_GOLDEN = Path(__file__).resolve().parent / "golden" / "directional"

CASES = [
    # data, n, dim, R, metric, k_ranks (= PQ subquantizers)
    ("gaussian", 2000, 128, 32, 0, 4),
    ("gaussian", 1500, 96, 16, 0, 16),
    ("relu_sphere", 1500, 128, 32, 1, 4),
    ("gaussian", 1200, 256, 64, 0, 16),
    ("gaussian", 1000, 200, 32, 1, 4),
]


def _data(kind, n, dim, seed):
    return getattr(synthetic, kind)(n, dim, seed)


def _population_c(g: O.OracleGraph, k_ranks: int) -> np.ndarray:
    """E over (uniform node with edges, uniform edge) of |Δ|_(r) / |Δ| --
    the quantity accumulate_rank_sums (lsh_globals.cuh:17-158) samples."""
    X = g.vec.view(np.float16).astype(np.float32)
    per_node = []
    for u in range(g.n):
        c = int(g.counts[u])
        if c == 0:
            continue
        nb = g.edges[u, :c].astype(np.int64) - g.global_offset
        d = (g.vec.view(np.float16)[nb] - g.vec.view(np.float16)[u][None]).astype(np.float32)
        nrm = np.sqrt((d * d).sum(1))
        ok = nrm > 0
        mags = -np.sort(-np.abs(d[ok]), axis=1)[:, :k_ranks] / nrm[ok, None]
        if len(mags):
            per_node.append(mags.mean(0))
    del X
    return np.mean(per_node, axis=0)


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"{c[0]}-d{c[2]}-R{c[3]}-m{c[4]}-k{c[5]}")
def test_builders_match_oracle(cuda, case):
    kind, n, dim, R, metric, kr = case
    X = _data(kind, n, dim, 71)
    h = T.construct(X, R, metric, 1.2 if metric == 0 else 1.0)
    try:
        _lib.call("jb_graph_build_lsh", h, kr, 16384, 42)
        _lib.call("jb_graph_build_pq", h, kr, 4000, 6, 123)
        g = T.oracle_from_handle(h, n, dim, R, metric)
        art = T.get_artifacts(h, n, R, g.dpad)
        # edge sketches and magnitudes: bit-exact
        packed, mag = O.lsh_edges_exact(g, kr)
        np.testing.assert_array_equal(art["lsh_packed"], packed)
        np.testing.assert_array_equal(art["lsh_mag_sq"], mag)
        # calibration: mean of 16384 sampled ratios vs the population mean
        # (standard error well below 1 %; tolerance 3 %)
        pop = _population_c(g, kr)
        np.testing.assert_allclose(art["lsh_c"], pop, rtol=0.03)
        c = art["lsh_c"]
        assert abs(float(art["lsh_norm_denom"]) - float((c.astype(np.float64) ** 2).sum())) < 1e-5
        # PQ codes for the trained centroids, and norms: bit-exact
        np.testing.assert_array_equal(art["pq_codes"], O.pq_codes_exact(g, art["pq_centroids"]))
        np.testing.assert_array_equal(art["norms"].view(np.uint32),
                                      O.row_norms_exact(g).view(np.uint32))
        # codebook quality: quantisation error of the edge residuals within
        # 15 % of a numpy Lloyd codebook trained the same way
        cent_np = D.pq_train(X, g.edges, g.counts, kr, n_train=4000, iters=6, seed=5)
        codes_np = O.pq_codes_exact(g, cent_np)
        err_gpu = _pq_error(g, art["pq_centroids"], art["pq_codes"])
        err_np = _pq_error(g, cent_np, codes_np)
        assert err_gpu <= 1.15 * err_np, (err_gpu, err_np)
        # the directional searches run bit-exact on the built payloads
        Q = _data(kind, 64, dim, 72)
        for which in ("lsh", "pq"):
            oi, od = O.dir_search(g, which, art, Q, 10, 64, 128)
            ji, jd = T.dir_search(h, which, Q, 10, 64, 128)
            T.assert_same_results(ji, jd, oi, od, msg=which)
    finally:
        T.free(h)


def _pq_error(g, cent, codes):
    M, _, dsub = cent.shape
    V = g.vec.view(np.float16)
    tot, cnt = 0.0, 0
    for u in range(0, g.n, 7):
        c = int(g.counts[u])
        if c == 0:
            continue
        r = (V[g.edges[u, :c].astype(np.int64)] - V[u][None]).astype(np.float32)
        for j in range(M):
            rec = cent[j][codes[u, j * g.R:j * g.R + c]]
            tot += float(((r[:, j * dsub:(j + 1) * dsub] - rec) ** 2).sum())
        cnt += c
    return tot / cnt


def test_builders_are_deterministic(cuda):
    X = synthetic.gaussian(1500, 128, 73)
    h1 = T.construct(X, 32, 0, 1.2)
    h2 = T.construct(X, 32, 0, 1.2)
    try:
        for h in (h1, h2):
            _lib.call("jb_graph_build_lsh", h, 4, 8192, 7)
            _lib.call("jb_graph_build_pq", h, 4, 3000, 4, 9)
        a1, a2 = T.get_artifacts(h1, 1500, 32, 128), T.get_artifacts(h2, 1500, 32, 128)
        for key in ("lsh_packed", "lsh_mag_sq", "lsh_c", "pq_centroids", "pq_codes", "norms"):
            np.testing.assert_array_equal(np.asarray(a1[key]).view(np.uint8),
                                          np.asarray(a2[key]).view(np.uint8), err_msg=key)
    finally:
        T.free(h1)
        T.free(h2)


@pytest.mark.parametrize("metric", [0, 1])
def test_prerotated_construct_and_search(cuda, metric):
    n, dim, R, kr = 3000, 128, 32, 4
    gen = synthetic.gaussian if metric == 0 else synthetic.relu_sphere
    X = gen(n, dim, 74)
    Q = gen(100, dim, 75) if metric == 0 else gen(100, dim, 75, center_seed=74)
    h = T.construct_directional(X, R, metric, 1.2 if metric == 0 else 1.0, True, seed=42)
    try:
        # stored rows are the rotated rows y = P^T x (fp16 rounding of an
        # fp32-accumulated product; tolerance 2 fp16 ulps of the row scale)
        P = np.zeros((dim, dim), np.float32)
        _lib.call("jb_rotation_matrix", dim, 42, P.ctypes.data)
        # column-major P: y_i = sum_k P[k + i * dim] x_k, so row i of the
        # row-major view is the i-th output's weights
        A = P.astype(np.float16).astype(np.float32)
        Y_ref = X.astype(np.float32) @ A.T
        Y = T.get_rows(h, n, dim).astype(np.float32)
        tol = 2 * np.float32(2.0 ** -10) * np.maximum(np.abs(Y_ref), 2.0 ** -14)
        assert (np.abs(Y - Y_ref) <= tol + 1e-3).mean() > 0.999
        # the graph over the rotated rows is exactly the oracle's build of them
        g = T.oracle_from_handle(h, n, dim, R, metric)
        g2 = O.OracleGraph(Y.astype(np.float16), R, metric=metric)
        g2.build(1.2 if metric == 0 else 1.0, O.reference_max_batch_size(10 * 10**9, n, R))
        np.testing.assert_array_equal(g.edges, g2.edges)
        np.testing.assert_array_equal(g.counts, g2.counts)
        _lib.call("jb_graph_build_lsh", h, kr, 16384, 42)
        _lib.call("jb_graph_build_pq", h, kr, 5000, 8, 123)
        art = T.get_artifacts(h, n, R, g.dpad)
        Yh = Y.astype(np.float16)
        c_np, nd_np = D.lsh_globals(Yh, g.edges, g.counts, kr, n_samples=16384)
        cent_np = D.pq_train(Yh, g.edges, g.counts, kr, n_train=5000, iters=8)
        art_np = dict(art, lsh_c=c_np, lsh_norm_denom=nd_np, pq_centroids=cent_np,
                      pq_codes=O.pq_codes_exact(g, cent_np))
        # queries are rotated inside the search kernel's prologue, in the
        # SIMT rotation GEMM's order: the results equal the restatement's
        # search of the queries rotated by that GEMM, bit for bit
        Qr = T.rotate_on_device(Q, dim, 42)
        Qf = (Q.astype(np.float32) @ A.T).astype(np.float16)
        assert np.mean(np.abs(Qr.astype(np.float32) - Qf.astype(np.float32)) <=
                       2 * 2.0 ** -10 * np.maximum(np.abs(Qf.astype(np.float32)), 2.0 ** -14)
                       + 1e-3) > 0.999
        for which in ("lsh", "pq"):
            ji, jd = T.dir_search(h, which, Q, 10, 64)
            oi, od = O.dir_search(g, which, art, Qr, 10, 64, 128)
            T.assert_same_results(ji, jd, oi, od, msg=which)
            # estimator quality: recall@10 with the device-built payloads is
            # no worse (within 0.05) than with payloads built by the numpy
            # restatement of the same builders on the same graph
            gt, _ = O.bruteforce(X, Q, 10, metric)
            rec = np.mean([len(set(a) & set(b)) / 10 for a, b in zip(ji, gt)])
            ni, _ = O.dir_search(g, which, art_np, Qr, 10, 64, 128)
            rec_np = np.mean([len(set(a) & set(b)) / 10 for a, b in zip(ni, gt)])
            assert rec >= rec_np - 0.05, (which, rec, rec_np)
    finally:
        T.free(h)


def test_directional_file_round_trip(cuda, tmp_path):
    n, dim, R, kr = 2000, 96, 32, 16
    X = synthetic.gaussian(n, dim, 76)
    Q = synthetic.gaussian(50, dim, 77)
    h = T.construct_directional(X, R, 0, 1.2, True, seed=3)
    path = str(tmp_path / "dir.graph")
    try:
        _lib.call("jb_graph_build_lsh", h, kr, 4096, 1)
        _lib.call("jb_graph_build_pq", h, kr, 2000, 3, 2)
        _lib.call("jb_graph_save_directional", h, path.encode())
        h2 = C.c_int64(-1)
        _lib.call("jb_graph_load_directional", path.encode(), dim, R, 0, kr, 0, 1, 3, C.byref(h2))
        try:
            a1, a2 = T.get_artifacts(h, n, R, 96), T.get_artifacts(h2.value, n, R, 96)
            for key in ("lsh_packed", "lsh_mag_sq", "lsh_c", "pq_centroids", "pq_codes", "norms"):
                np.testing.assert_array_equal(np.asarray(a1[key]).view(np.uint8),
                                              np.asarray(a2[key]).view(np.uint8), err_msg=key)
            for which in ("lsh", "pq"):
                T.assert_same_results(*T.dir_search(h, which, Q, 10, 32),
                                      *T.dir_search(h2.value, which, Q, 10, 32), msg=which)
            # a wrong rank count is rejected, as in the reference loader
            with pytest.raises(Exception, match="k_ranks"):
                h3 = C.c_int64(-1)
                _lib.call("jb_graph_load_directional", path.encode(), dim, R, 0, 4, 0, 1, 3,
                          C.byref(h3))
        finally:
            T.free(h2.value)
    finally:
        T.free(h)


@pytest.mark.parametrize("path", sorted(DIR_GOLDEN.glob("*.npz")), ids=lambda p: p.stem)
def test_load_legacy_directional_file_matches_reference(cuda, tmp_path, path):
    """The legacy-layout directional file the reference itself loaded to make
    the golden outputs: loading it here gives the reference's results."""
    from test_oracle import regen, oracle_from_golden
    z = np.load(path)
    X, Q = regen(z)
    g = oracle_from_golden(z, X)
    kr = int(z["k_ranks"])
    f = str(tmp_path / "legacy.graph")
    D.write_legacy_directional(f, X, g.edges, g.edist, g.counts, g.medoid, g.R, kr,
                               packed=z["lsh_packed"], mag=z["lsh_mag_sq"], c=z["lsh_c"],
                               norm_denom=z["lsh_norm_denom"], cent=z["pq_centroids"],
                               codes=z["pq_codes"], nrm=z["norms"])
    h = C.c_int64(-1)
    _lib.call("jb_graph_load_directional", f.encode(), g.dim, g.R, g.metric, kr, 0, 0, 0,
              C.byref(h))
    try:
        for kind, key in (("lsh", "directional_search"), ("pq", "pq_search")):
            for bw in z["bws"]:
                bw = int(bw)
                ji, jd = T.dir_search(h.value, kind, Q, 10, bw)
                T.assert_same_results(ji, jd, z[f"{key}_idx_bw{bw}"], z[f"{key}_dist_bw{bw}"],
                                      msg=f"{kind} bw={bw}")
    finally:
        T.free(h.value)


def test_python_graph_directional_surface(cuda, tmp_path):
    import torch
    import jasper_b200 as jasper
    X = torch.from_numpy(synthetic.gaussian(3000, 128, 78)).cuda()
    Q = torch.from_numpy(synthetic.gaussian(64, 128, 79)).cuda()
    g = jasper.Graph.build(X, n_neighbors=32, build_lsh=True, build_pq=True, k_ranks=4,
                           lsh_samples=4096, pq_train=3000, pq_kmeans_iter=4)
    with pytest.raises(RuntimeError, match="directional graph"):
        g.search(Q)
    li, ld = g.directional_search(Q, k=10, beam_width=64)
    pi, pd = g.pq_search(Q, k=10, beam_width=64)
    assert li.shape == (64, 10) and li.dtype == torch.int32 and pd.dtype == torch.float32
    path = str(tmp_path / "g.graph")
    g.save(path)
    g2 = jasper.Graph.load(path, dim=128, n_neighbors=32, k_ranks=4, prerotate=True)
    for a, b in ((g2.directional_search(Q, k=10, beam_width=64), (li, ld)),
                 (g2.pq_search(Q, k=10, beam_width=64), (pi, pd))):
        T.assert_same_results(a[0].cpu().numpy(), a[1].cpu().numpy(), b[0].cpu().numpy(),
                              b[1].cpu().numpy())
    # loaded without the trailer's PQ / LSH: the search is refused
    g3 = jasper.Graph.load(path, dim=128, n_neighbors=32)
    with pytest.raises(RuntimeError, match="build_lsh"):
        g3.directional_search(Q)
    gt, _ = O.bruteforce(X.cpu().numpy(), Q.cpu().numpy(), 10, 0)
    for ids in (li, pi):
        rec = np.mean([len(set(a) & set(b)) / 10 for a, b in zip(ids.cpu().numpy(), gt)])
        assert rec > 0.2, rec   # iid gaussian 128-d, 4 ranks: a smoke bound only
    for h in (g, g2, g3):
        h.free()
