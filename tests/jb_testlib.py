"""Helpers shared by the tests: calls into libjasper_b200 through its C ABI."""
from __future__ import annotations

import ctypes as C

import numpy as np

from jasper_b200 import _lib
from oracle import oracle as O


def create_graph(g: "O.OracleGraph") -> int:
    """Upload an oracle graph (rows + adjacency) into a jasper_b200 handle."""
    rows = np.ascontiguousarray(g.vec)
    h = C.c_int64(-1)
    _lib.call("jb_graph_create", rows.ctypes.data, g.n, g.dim, g.dpad, g.R, g.metric, 0, C.byref(h))
    _lib.call("jb_graph_set_edges", h.value, g.edges.ctypes.data, g.edist.ctypes.data,
              g.counts.ctypes.data, g.medoid)
    return h.value


def get_edges(h: int, n: int, R: int):
    e = np.zeros((n, R), np.uint32)
    d = np.zeros((n, R), np.uint16)
    c = np.zeros(n, np.uint8)
    _lib.call("jb_graph_get_edges", h, e.ctypes.data, d.ctypes.data, c.ctypes.data)
    return e, d, c


def search(h: int, Q: np.ndarray, k: int, bw: int, limit: int | None = None, stats: bool = False):
    import torch
    q = torch.from_numpy(O.pad_rows(Q)).cuda()
    nq = q.shape[0]
    oi = torch.empty(nq, k, dtype=torch.int32, device="cuda")
    od = torch.empty(nq, k, dtype=torch.float32, device="cuda")
    limit = 2 * bw if limit is None else limit
    st = torch.cuda.current_stream().cuda_stream
    if stats:
        s = torch.zeros(nq, 5, dtype=torch.int32, device="cuda")
        info = _lib.GraphInfo()
        _lib.call("jb_graph_get_info", h, C.byref(info))
        seen = torch.zeros(nq * ((info.n_vectors + 31) // 32), dtype=torch.int32, device="cuda")
        _lib.call("jb_graph_search_stats", h, q.data_ptr(), nq, q.shape[1], oi.data_ptr(),
                  od.data_ptr(), k, bw, limit, s.data_ptr(), seen.data_ptr(), st)
        torch.cuda.synchronize()
        return oi.cpu().numpy(), od.cpu().numpy(), s.cpu().numpy()
    _lib.call("jb_graph_search", h, q.data_ptr(), nq, q.shape[1], oi.data_ptr(), od.data_ptr(),
              k, bw, limit, st)
    torch.cuda.synchronize()
    return oi.cpu().numpy(), od.cpu().numpy()


def construct(X: np.ndarray, R: int, metric: int, alpha: float, budget: int = 10 * 10**9) -> int:
    x = np.ascontiguousarray(X, dtype=np.float16)
    h = C.c_int64(-1)
    _lib.call("jb_graph_construct", x.ctypes.data, x.shape[0], x.shape[1], x.shape[1], R, metric,
              float(alpha), budget, 0, None, C.byref(h))
    return h.value


def free(h: int) -> None:
    _lib.call("jb_graph_free", h)


def assert_same_results(ai, ad, bi, bd, msg=""):
    """Bit-exact ids and distances."""
    np.testing.assert_array_equal(ai, bi, err_msg=msg)
    np.testing.assert_array_equal(np.asarray(ad, np.float32).view(np.uint32),
                                  np.asarray(bd, np.float32).view(np.uint32), err_msg=msg)


def set_artifacts(h: int, art: dict, k_ranks: int) -> None:
    """Attach LSH and PQ payloads (numpy arrays, oracle/directional.py layout)."""
    packed = np.ascontiguousarray(art["lsh_packed"])
    mag = np.ascontiguousarray(art["lsh_mag_sq"], np.uint16)
    c = np.ascontiguousarray(art["lsh_c"], np.float32)
    _lib.call("jb_graph_set_lsh", h, k_ranks, packed.dtype.itemsize, packed.ctypes.data,
              mag.ctypes.data, c.ctypes.data, float(art["lsh_norm_denom"]))
    cent = np.ascontiguousarray(art["pq_centroids"], np.float32)
    codes = np.ascontiguousarray(art["pq_codes"], np.uint8)
    nrm = np.ascontiguousarray(art["norms"], np.float32)
    M = k_ranks
    _lib.call("jb_graph_set_pq", h, M, cent.size // (M * 256), cent.ctypes.data, codes.ctypes.data,
              nrm.ctypes.data)


def dir_search(h: int, kind: str, Q: np.ndarray, k: int, bw: int, limit: int | None = None):
    import torch
    q = torch.from_numpy(O.pad_rows(Q)).cuda()
    nq = q.shape[0]
    oi = torch.empty(nq, k, dtype=torch.int32, device="cuda")
    od = torch.empty(nq, k, dtype=torch.float32, device="cuda")
    limit = 2 * bw if limit is None else limit
    _lib.call("jb_graph_directional_search", h, 0 if kind == "lsh" else 1, q.data_ptr(), nq,
              q.shape[1], oi.data_ptr(), od.data_ptr(), k, bw, limit,
              torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return oi.cpu().numpy(), od.cpu().numpy()
