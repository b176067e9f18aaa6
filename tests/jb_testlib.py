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


def get_artifacts(h: int, n: int, R: int, dpad: int) -> dict:
    """Read back LSH and PQ payloads (whichever the graph carries)."""
    flags = C.c_int32(0)
    _lib.call("jb_graph_get_directional_flags", h, C.byref(flags))
    art = {}
    if flags.value & 1:
        kr, pb, nd = C.c_uint32(0), C.c_uint32(0), C.c_float(0)
        _lib.call("jb_graph_get_lsh", h, C.byref(kr), C.byref(pb), None, None, None, C.byref(nd))
        packed = np.zeros((n, R * kr.value), np.uint8 if pb.value == 1 else np.uint16)
        mag = np.zeros((n, R), np.uint16)
        c = np.zeros(kr.value, np.float32)
        _lib.call("jb_graph_get_lsh", h, None, None, packed.ctypes.data, mag.ctypes.data,
                  c.ctypes.data, C.byref(nd))
        art.update(lsh_packed=packed, lsh_mag_sq=mag, lsh_c=c, lsh_norm_denom=np.float32(nd.value),
                   k_ranks=kr.value)
    if flags.value & 2:
        m, ds = C.c_uint32(0), C.c_uint32(0)
        _lib.call("jb_graph_get_pq", h, C.byref(m), C.byref(ds), None, None, None)
        cent = np.zeros((m.value, 256, ds.value), np.float32)
        codes = np.zeros((n, m.value * R), np.uint8)
        nrm = np.zeros(n, np.float32)
        _lib.call("jb_graph_get_pq", h, None, None, cent.ctypes.data, codes.ctypes.data,
                  nrm.ctypes.data)
        art.update(pq_centroids=cent, pq_codes=codes, norms=nrm, k_ranks=m.value)
    return art


def get_rows(h: int, n: int, dim: int) -> np.ndarray:
    """All stored rows (identity ids) as fp16 [n, dim]."""
    out = np.zeros((n, dim), np.float16)
    for i in range(n):
        _lib.call("jb_graph_get_vector", h, i, out[i:].ctypes.data)
    return out


def construct_directional(X: np.ndarray, R: int, metric: int, alpha: float, prerotate: bool,
                          seed: int = 42, budget: int = 10 * 10**9) -> int:
    x = np.ascontiguousarray(X, dtype=np.float16)
    h = C.c_int64(-1)
    _lib.call("jb_graph_construct_directional", x.ctypes.data, x.shape[0], x.shape[1], x.shape[1],
              R, metric, float(alpha), budget, 0, int(prerotate), seed, None, C.byref(h))
    return h.value


def oracle_from_handle(h: int, n: int, dim: int, R: int, metric: int) -> "O.OracleGraph":
    """Copy a handle's rows and adjacency into an oracle graph."""
    info = _lib.GraphInfo()
    _lib.call("jb_graph_get_info", h, C.byref(info))
    g = O.OracleGraph(get_rows(h, n, dim), R, metric=metric, medoid=info.medoid)
    e, d, c = get_edges(h, n, R)
    g.edges[:], g.edist[:], g.counts[:] = e, d, c
    return g


def dir_search_kind(h: int, kind: int, Q: np.ndarray, k: int, bw: int, limit: int | None = None):
    """jb_graph_directional_search with an explicit kind (0 LSH, 1 PQ, 2 RaBitQ)."""
    import torch
    q = torch.from_numpy(O.pad_rows(Q)).cuda()
    nq = q.shape[0]
    oi = torch.empty(nq, k, dtype=torch.int32, device="cuda")
    od = torch.empty(nq, k, dtype=torch.float32, device="cuda")
    limit = 2 * bw if limit is None else limit
    _lib.call("jb_graph_directional_search", h, kind, q.data_ptr(), nq, q.shape[1], oi.data_ptr(),
              od.data_ptr(), k, bw, limit, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return oi.cpu().numpy(), od.cpu().numpy()


def rotate_on_device(Q: np.ndarray, dim: int, seed: int, tensor_cores: bool = False) -> np.ndarray:
    """Rows rotated on the device, as fp16 [n, dim].  By default in the SIMT
    GEMM's summation order, which is the order the search kernels use when
    they rotate each query in their prologue; tensor_cores=True gives the
    tcgen05 GEMM that rotates a graph's rows."""
    import torch
    x = torch.from_numpy(O.pad_rows(Q)).cuda()
    y = torch.empty_like(x)
    _lib.call("jb_rotate_rows", dim, seed, x.data_ptr(), y.data_ptr(), x.shape[0],
              1 if tensor_cores else 0, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return y.cpu().numpy().view(np.float16)[:, :dim]
