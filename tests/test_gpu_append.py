"""Live append (jb_graph_append; reference append_batch,
include/jasper/index/construct.cuh:1169-1265, and its check in
cmd/test_append.cu: appended ids are [N, N+M) and each appended vector finds
itself).  The appended graph is compared bit for bit with the CPU
restatement's append (oracle/jasper_oracle.c: orc_append_range)."""
from __future__ import annotations

import numpy as np
import pytest

from jasper_b200 import _lib, synthetic
from oracle import oracle as O
import jb_testlib as T

pytestmark = pytest.mark.gpu


def _append(h, rows, alpha):
    import torch
    x = np.ascontiguousarray(rows, dtype=np.float16)
    ids = np.full(x.shape[0], -7, np.int32)
    _lib.call("jb_graph_append", h, x.ctypes.data, x.shape[0], x.shape[1], float(alpha),
              ids.ctypes.data, torch.cuda.current_stream().cuda_stream)
    return ids


@pytest.mark.parametrize("case", [
    # data, n0, appended per round, rounds, dim, R, metric
    ("gaussian", 2000, 1000, 1, 64, 32, 0),
    ("sift_like", 1500, 700, 2, 128, 64, 0),
    ("gaussian", 1200, 333, 2, 100, 16, 1),   # padded rows, inner product
])
def test_append_matches_oracle(cuda, case):
    kind, n0, m, rounds, dim, R, metric = case
    total = n0 + m * rounds
    X = getattr(synthetic, kind)(total, dim, 91)
    alpha = 1.2 if metric == 0 else 1.0
    h = T.construct(X[:n0], R, metric, alpha)
    try:
        g = O.OracleGraph(X[:n0], R, metric=metric)
        g.build(alpha, O.reference_max_batch_size(10 * 10**9, n0, R))
        for r in range(rounds):
            lo = n0 + r * m
            ids = _append(h, X[lo:lo + m], alpha)
            oids = g.append(X[lo:lo + m], alpha)
            np.testing.assert_array_equal(ids, np.arange(lo, lo + m, dtype=np.int32))
            np.testing.assert_array_equal(ids, oids)
            e, d, c = T.get_edges(h, lo + m, R)
            np.testing.assert_array_equal(c, g.counts, err_msg=f"round {r}: edge counts")
            for i in range(lo + m):
                k = int(c[i])
                np.testing.assert_array_equal(e[i, :k], g.edges[i, :k], err_msg=f"row {i}")
                np.testing.assert_array_equal(d[i, :k], g.edist[i, :k], err_msg=f"row {i}")
        # appended vectors find themselves (cmd/test_append.cu) about as
        # often as built ones do (L2; under IP a row need not be its own
        # nearest neighbour)
        lo = n0
        ji, jd = T.search(h, X[lo:], 10, 64)
        if metric == 0:
            bi, _ = T.search(h, X[:300], 10, 64)
            assert np.mean(ji[:, 0] == np.arange(lo, total)) >= \
                np.mean(bi[:, 0] == np.arange(300)) - 0.03
        oi, od, _, _ = g.search(X[lo:lo + 100], 10, 64, 128)
        T.assert_same_results(ji[:100], jd[:100], oi, od)
    finally:
        T.free(h)


def test_append_python_api_and_rejections(cuda):
    import torch
    import jasper_b200 as jasper
    X = synthetic.sift_like(6000, 128, 92)
    Xd = torch.from_numpy(X).cuda()
    g = jasper.Graph.build(Xd[:5000], n_neighbors=32)
    try:
        ids = g.append(Xd[5000:], alpha=1.2)
        assert ids.dtype == torch.int32 and ids.device.type == "cpu"
        assert ids.tolist() == list(range(5000, 6000))
        assert g.n_vectors == 6000
        found, _ = g.search(Xd[5000:], k=1, beam_width=64)
        base, _ = g.search(Xd[:500], k=1, beam_width=64)
        own = (base[:, 0].cpu() == torch.arange(500)).float().mean().item()
        assert (found[:, 0].cpu() == ids).float().mean().item() >= own - 0.03
        with pytest.raises(ValueError):
            g.append(Xd[:3, :64])
        with pytest.raises(ValueError):
            g.append(Xd[:3].cpu())
        empty = g.append(Xd[:0])
        assert empty.numel() == 0 and g.n_vectors == 6000
    finally:
        g.free()
    gd = jasper.Graph.build(Xd[:3000], n_neighbors=32, build_lsh=True, lsh_samples=2048)
    try:
        with pytest.raises(Exception, match="plain graphs"):
            gd.append(Xd[3000:3100])
    finally:
        gd.free()
