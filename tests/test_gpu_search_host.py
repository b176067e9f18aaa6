"""jb_graph_search_host (queries and results in host memory) returns exactly
what jb_graph_search returns for the same queries on device buffers, for
page-locked and pageable host buffers, padded query rows and mixed cases,
over repeated calls."""
import numpy as np
import pytest
import torch

from jasper_b200 import _lib, synthetic
from oracle import oracle as O
import jb_testlib as T

pytestmark = pytest.mark.gpu


def _host_search(h, q: torch.Tensor, k, bw, out_i: torch.Tensor, out_d: torch.Tensor):
    _lib.call("jb_graph_search_host", h, q.data_ptr(), q.shape[0], q.shape[1], out_i.data_ptr(),
              out_d.data_ptr(), k, bw, 2 * bw, torch.cuda.current_stream().cuda_stream)
    return out_i.numpy(), out_d.numpy()


@pytest.mark.parametrize("metric", [0, 1])
def test_search_host_matches_device_search(cuda, metric):
    n, dim, k = 4000, 128, 10
    X = synthetic.gaussian(n, dim, 61)
    Q = synthetic.gaussian(777, dim, 62)
    h = T.construct(X, 32, metric, 1.2 if metric == 0 else 1.0)
    try:
        for bw in (16, 64):
            ri, rd = T.search(h, Q, k, bw)
            qp = torch.from_numpy(O.pad_rows(Q))
            cases = {
                "pinned": (qp.pin_memory(), True, True),
                "pageable": (qp.clone(), False, False),
                "pinned-in": (qp.pin_memory(), False, False),
                "pinned-out": (qp.clone(), True, True),
                "mixed-out": (qp.pin_memory(), True, False),
            }
            for name, (q, pin_i, pin_d) in cases.items():
                oi = torch.full((Q.shape[0], k), 7, dtype=torch.int32)
                od = torch.full((Q.shape[0], k), 7.0, dtype=torch.float32)
                oi = oi.pin_memory() if pin_i else oi
                od = od.pin_memory() if pin_d else od
                for _ in range(2):
                    gi, gd = _host_search(h, q, k, bw, oi, od)
                    T.assert_same_results(gi, gd, ri, rd, msg=f"{name} bw={bw}")
            # padded rows (row stride > dim) from pinned memory take the copy path
            qw = np.zeros((Q.shape[0], dim + 24), np.float16)
            qw[:, :dim] = Q
            oi = torch.empty(Q.shape[0], k, dtype=torch.int32).pin_memory()
            od = torch.empty(Q.shape[0], k, dtype=torch.float32).pin_memory()
            gi, gd = _host_search(h, torch.from_numpy(qw).pin_memory(), k, bw, oi, od)
            T.assert_same_results(gi, gd, ri, rd, msg=f"padded bw={bw}")
    finally:
        T.free(h)


def test_search_host_large_batch(cuda):
    """A batch larger than the device's resident warps (9001 queries): the
    results equal the device search, call after call, with the outputs
    refilled in between."""
    n, dim, k, bw = 3000, 64, 10, 32
    X = synthetic.gaussian(n, dim, 71)
    Q = synthetic.gaussian(9001, dim, 72)
    h = T.construct(X, 16, 0, 1.2)
    try:
        ri, rd = T.search(h, Q, k, bw)
        qp = torch.from_numpy(O.pad_rows(Q))
        for q, pinned in ((qp.pin_memory(), True), (qp.clone(), False)):
            oi = torch.empty(Q.shape[0], k, dtype=torch.int32)
            od = torch.empty(Q.shape[0], k, dtype=torch.float32)
            if pinned:
                oi, od = oi.pin_memory(), od.pin_memory()
            for _ in range(3):
                oi.fill_(7)
                od.fill_(7.0)
                gi, gd = _host_search(h, q, k, bw, oi, od)
                T.assert_same_results(gi, gd, ri, rd, msg=f"pinned={pinned}")
    finally:
        T.free(h)


@pytest.mark.parametrize("dim", [200, 960])
@pytest.mark.parametrize("metric", [0, 1])
def test_search_host_pinned_wide_rows(cuda, dim, metric):
    """Page-locked buffers are read and written in place by the search
    kernel, which stages each query row in shared memory before building its
    query layout: the lane-per-row layout (dim 200) and the shared-memory
    query (dim 960), for both the warp-per-query kernel (2500 queries) and
    the CTA-per-query kernel (300 queries)."""
    n, k, bw = 3000, 10, 32
    X = synthetic.gaussian(n, dim, 81 + dim)
    h = T.construct(X, 16, metric, 1.2 if metric == 0 else 1.0)
    try:
        for nq in (2500, 300):
            Q = synthetic.gaussian(nq, dim, 82 + dim)
            ri, rd = T.search(h, Q, k, bw)
            q = torch.from_numpy(O.pad_rows(Q)).pin_memory()
            oi = torch.full((nq, k), 7, dtype=torch.int32).pin_memory()
            od = torch.full((nq, k), 7.0, dtype=torch.float32).pin_memory()
            for _ in range(2):
                gi, gd = _host_search(h, q, k, bw, oi, od)
                T.assert_same_results(gi, gd, ri, rd, msg=f"dim={dim} nq={nq}")
    finally:
        T.free(h)
