"""jb_graph_search_noalloc: the search entry point for callers that cannot let
a search allocate device memory (a fixed pre-reserved budget, an allocator
they own, or no allocator traffic while other GPU work runs).  It must give
exactly the results of jb_graph_search -- the same bit-exact bar as every
other search test -- on consecutive calls that reuse its fixed scratch, and
must refuse, with a clear error, queries whose repacking would not fit.

Collected last on purpose (file name), and self-contained, so it passes both
alone in a fresh process and after the rest of the suite."""
import ctypes as C

import numpy as np
import pytest

from jasper_b200 import _lib, synthetic
import jb_testlib as T

pytestmark = pytest.mark.gpu


def _noalloc(h, q, nq, stride, k, bw):
    import torch
    oi = torch.full((nq, k), -7, dtype=torch.int32, device="cuda")
    od = torch.full((nq, k), -7.0, dtype=torch.float32, device="cuda")
    _lib.call("jb_graph_search_noalloc", h, q.data_ptr(), nq, stride, oi.data_ptr(),
              od.data_ptr(), k, bw, 2 * bw, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return oi.cpu().numpy(), od.cpu().numpy()


def _alloc(h, q, nq, stride, k, bw):
    import torch
    oi = torch.empty((nq, k), dtype=torch.int32, device="cuda")
    od = torch.empty((nq, k), dtype=torch.float32, device="cuda")
    _lib.call("jb_graph_search", h, q.data_ptr(), nq, stride, oi.data_ptr(), od.data_ptr(),
              k, bw, 2 * bw, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return oi.cpu().numpy(), od.cpu().numpy()


def test_noalloc_matches_search_on_consecutive_calls(cuda):
    import torch
    X = synthetic.gaussian(3000, 128, 51)
    h = T.construct(X, 32, 0, 1.2)
    try:
        for seed, bw in [(52, 64), (53, 32)]:  # two calls in a row, different inputs
            Q = torch.from_numpy(synthetic.gaussian(300, 128, seed)).cuda()
            a = _alloc(h, Q, 300, 128, 10, bw)
            b = _noalloc(h, Q, 300, 128, 10, bw)
            T.assert_same_results(b[0], b[1], a[0], a[1], msg=f"seed={seed}")
    finally:
        T.free(h)


def test_noalloc_repacks_unpadded_queries_and_rejects_oversize(cuda):
    import torch
    X = synthetic.gaussian(2000, 100, 54)       # dim % 8 != 0: padded stride is 104
    h = T.construct(X, 16, 0, 1.2)
    try:
        Q = torch.from_numpy(synthetic.gaussian(200, 100, 55)).cuda()   # stride 100
        a = _alloc(h, Q, 200, 100, 10, 64)
        for _ in range(2):
            b = _noalloc(h, Q, 200, 100, 10, 64)
            T.assert_same_results(b[0], b[1], a[0], a[1])
        big = torch.zeros((21000, 100), dtype=torch.float16, device="cuda")  # 21000*104*2 > 4 MiB
        with pytest.raises(ValueError, match="scratch"):
            _noalloc(h, big, 21000, 100, 10, 16)
    finally:
        T.free(h)
