"""ctypes wrapper of the CPU restatement (jasper_oracle.c).

TEST INFRASTRUCTURE ONLY.  tests/, __graft_entry__.smoke() and the
cpu_baseline leg of bench.py use it as the checker; the jasper_b200 product
never imports it.  Build with ``make -C oracle`` (or __graft_entry__.build()).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libjasper_oracle.so"


class _Graph(C.Structure):
    _fields_ = [
        ("n", C.c_uint32), ("dim", C.c_uint32), ("dpad", C.c_uint32), ("R", C.c_uint32),
        ("metric", C.c_int), ("medoid", C.c_uint32), ("global_offset", C.c_uint32),
        ("vec", C.c_void_p), ("edges", C.c_void_p), ("edist", C.c_void_p),
        ("counts", C.c_void_p), ("deleted", C.c_void_p),
    ]


_lib = None


def build() -> Path:
    srcs = [HERE / "jasper_oracle.c", HERE / "bruteforce.c"]
    if not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < max(s.stat().st_mtime for s in srcs):
        subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        L = C.CDLL(str(LIB_PATH))
        P = C.c_void_p
        L.orc_distance_f32.argtypes = [C.c_int, P, P, C.c_int]
        L.orc_distance_f32.restype = C.c_float
        L.orc_distance_f16.argtypes = [C.c_int, P, P, C.c_int]
        L.orc_distance_f16.restype = C.c_float
        L.orc_half_to_float.argtypes = [C.c_uint16]
        L.orc_half_to_float.restype = C.c_float
        L.orc_float_to_bf16.argtypes = [C.c_float]
        L.orc_float_to_bf16.restype = C.c_uint16
        L.orc_search.argtypes = [C.POINTER(_Graph), P, C.c_uint32, C.c_uint32, C.c_uint32,
                                 C.c_uint32, C.c_uint32, P, P, P, P]
        L.orc_search.restype = None
        L.orc_search_one.argtypes = [C.POINTER(_Graph), P, C.c_uint32, C.c_uint32, C.c_uint32,
                                     C.c_uint32, P, P, P, P, P]
        L.orc_search_one.restype = C.c_uint32
        L.orc_build.argtypes = [C.POINTER(_Graph), C.c_float, C.c_uint32]
        L.orc_build.restype = None
        L.orc_bruteforce.argtypes = [P, C.c_uint32, P, C.c_uint32, C.c_uint32, C.c_int,
                                     C.c_uint32, P, P]
        L.orc_bruteforce.restype = None
        L.orc_set_threads.argtypes = [C.c_int]
        L.orc_set_threads.restype = None
        L.orc_max_threads.argtypes = []
        L.orc_max_threads.restype = C.c_int
        _lib = L
    return _lib


def set_threads(n: int) -> None:
    lib().orc_set_threads(int(n))


def max_threads() -> int:
    return int(lib().orc_max_threads())


def _p(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def pad_rows(x: np.ndarray) -> np.ndarray:
    """fp16 [n, dim] -> uint16 bit patterns [n, dpad] with zero pad lanes."""
    x = np.ascontiguousarray(x, dtype=np.float16)
    n, d = x.shape
    dpad = (d + 7) // 8 * 8
    out = np.zeros((n, dpad), dtype=np.uint16)
    out[:, :d] = x.view(np.uint16)
    return out


class OracleGraph:
    """A graph in the oracle's flat layout (numpy arrays, CPU)."""

    def __init__(self, vectors: np.ndarray, R: int, metric: int = 0, medoid: int = 0,
                 global_offset: int = 0):
        v = np.ascontiguousarray(vectors, dtype=np.float16)
        self.n, self.dim = v.shape
        self.vec = pad_rows(v)
        self.dpad = self.vec.shape[1]
        self.R = R
        self.metric = metric
        self.medoid = medoid
        self.global_offset = global_offset
        self.edges = np.full((self.n, R), 0xFFFFFFFF, dtype=np.uint32)
        self.edist = np.zeros((self.n, R), dtype=np.uint16)
        self.counts = np.zeros(self.n, dtype=np.uint8)
        self.deleted: np.ndarray | None = None

    def _struct(self) -> _Graph:
        return _Graph(self.n, self.dim, self.dpad, self.R, self.metric, self.medoid,
                      self.global_offset, _p(self.vec), _p(self.edges), _p(self.edist),
                      _p(self.counts), _p(self.deleted))

    def build(self, alpha: float, max_batch_size: int) -> None:
        g = self._struct()
        lib().orc_build(C.byref(g), float(alpha), int(max_batch_size))

    def append(self, vectors: np.ndarray, alpha: float, max_batch: int = 0) -> np.ndarray:
        """Live append (orc_append_range): the rows join at slots [n, n + m)
        and are wired in batches of min(m, 100000) rows (or max_batch).
        Returns the new rows' slots (their ids while no compaction ran)."""
        v = pad_rows(np.ascontiguousarray(vectors, dtype=np.float16))
        assert v.shape[1] == self.dpad
        old, m = self.n, v.shape[0]
        self.vec = np.ascontiguousarray(np.concatenate([self.vec, v]))
        self.edges = np.ascontiguousarray(np.concatenate(
            [self.edges, np.full((m, self.R), 0xFFFFFFFF, np.uint32)]))
        self.edist = np.ascontiguousarray(np.concatenate(
            [self.edist, np.zeros((m, self.R), np.uint16)]))
        self.counts = np.ascontiguousarray(np.concatenate([self.counts, np.zeros(m, np.uint8)]))
        if self.deleted is not None:
            words = (old + m + 31) // 32
            d = np.zeros(words, np.uint32)
            d[:self.deleted.shape[0]] = self.deleted
            self.deleted = d
        self.n = old + m
        g = self._struct()
        L = lib()
        L.orc_append_range.argtypes = [C.POINTER(_Graph), C.c_uint32, C.c_uint32, C.c_float,
                                       C.c_uint32]
        L.orc_append_range(C.byref(g), old, m, float(alpha), int(max_batch))
        return np.arange(old, old + m, dtype=np.int32)

    def search(self, queries: np.ndarray, k: int, beam_width: int, limit: int,
               max_result_size: int = 2048):
        q = pad_rows(queries)
        assert q.shape[1] == self.dpad
        nq = q.shape[0]
        oi = np.zeros((nq, k), dtype=np.uint32)
        od = np.zeros((nq, k), dtype=np.float32)
        ne = np.zeros(nq, dtype=np.uint32)
        ev = np.zeros(nq, dtype=np.uint64)
        g = self._struct()
        lib().orc_search(C.byref(g), _p(q), nq, k, beam_width, limit, max_result_size,
                         _p(oi), _p(od), _p(ne), _p(ev))
        return oi.view(np.int32), od, ne, ev

    def search_visited(self, query: np.ndarray, k: int, beam_width: int, limit: int,
                       max_result_size: int):
        """One query with its expansion order (the build's search)."""
        q = pad_rows(query.reshape(1, -1))
        oi = np.zeros(k, dtype=np.uint32)
        od = np.zeros(k, dtype=np.float32)
        vi = np.zeros(max_result_size, dtype=np.uint32)
        vd = np.zeros(max_result_size, dtype=np.float32)
        g = self._struct()
        n = lib().orc_search_one(C.byref(g), _p(q), k, beam_width, limit, max_result_size,
                                 _p(oi), _p(od), _p(vi), _p(vd), None)
        return oi.view(np.int32), od, vi[:n].view(np.int32), vd[:n]


def distance_f32(metric: int, a, b, dim: int) -> float:
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    return float(lib().orc_distance_f32(metric, _p(a), _p(b), dim))


def distance_f16(metric: int, a, b, dim: int | None = None) -> float:
    a = pad_rows(np.asarray(a, dtype=np.float16).reshape(1, -1))[0]
    b = pad_rows(np.asarray(b, dtype=np.float16).reshape(1, -1))[0]
    return float(lib().orc_distance_f16(metric, _p(a), _p(b), a.shape[0] if dim is None else dim))


def bruteforce(base: np.ndarray, queries: np.ndarray, k: int, metric: int = 0):
    b = pad_rows(base)
    q = pad_rows(queries)
    nq = q.shape[0]
    oi = np.zeros((nq, k), dtype=np.uint32)
    od = np.zeros((nq, k), dtype=np.float32)
    lib().orc_bruteforce(_p(b), b.shape[0], _p(q), nq, b.shape[1], metric, k, _p(oi), _p(od))
    return oi.view(np.int32), od


def bruteforce_knn(base: np.ndarray, queries: np.ndarray, k: int, metric: int = 0,
                   threads: int | None = None):
    """The timed CPU baseline (oracle/bruteforce.c): exact k-NN of fp32
    rows over fp32 queries on `threads` host threads (default: all), distance
    ascending then id.  Returns (ids int32 [nq, k], distances float32)."""
    b = np.ascontiguousarray(base, dtype=np.float32)
    q = np.ascontiguousarray(queries, dtype=np.float32)
    assert b.ndim == 2 and q.ndim == 2 and b.shape[1] == q.shape[1]
    L = lib()
    L.orc_bruteforce_knn.argtypes = [C.c_void_p, C.c_uint64, C.c_void_p, C.c_uint64, C.c_uint32,
                                     C.c_uint32, C.c_int, C.c_int, C.c_void_p, C.c_void_p]
    L.orc_bruteforce_knn.restype = C.c_int
    nq = q.shape[0]
    oi = np.empty((nq, k), dtype=np.int32)
    od = np.empty((nq, k), dtype=np.float32)
    rc = L.orc_bruteforce_knn(_p(b), b.shape[0], _p(q), nq, b.shape[1], k, metric,
                              int(threads or os.cpu_count() or 1), _p(oi), _p(od))
    if rc != 0:
        raise ValueError("orc_bruteforce_knn: bad arguments")
    return oi, od


def reference_max_batch_size(budget_bytes: int, n: int, R: int) -> int:
    """graph_construct_workspace::max_batch_size_for_budget (construct.cuh:233-258)
    capped at n / 50 (ffi/jasper_ffi_common.cuh:245-248)."""
    L, mrs = 64, 256
    per_item = 8 * L + 8 * mrs + 4 + 8 * (mrs + R) + 4 + 8 * R + 4 * R + 4 * R
    b = 0 if budget_bytes <= 4 else (budget_bytes - 4) // per_item
    return min(b, n // 50)


# ── directional search ──────────────────────────────────────────────────
class _Dir(C.Structure):
    _fields_ = [
        ("kind", C.c_int), ("k_ranks", C.c_uint32), ("packed_bytes", C.c_uint32),
        ("packed", C.c_void_p), ("mag_sq", C.c_void_p), ("c", C.c_void_p),
        ("norm_denom", C.c_float), ("pq_m", C.c_uint32), ("pq_dsub", C.c_uint32),
        ("centroids", C.c_void_p), ("codes", C.c_void_p), ("norms", C.c_void_p),
    ]


def set_dir_mode(m: int) -> None:
    L = lib()
    L.orc_set_dir_mode.argtypes = [C.c_int]
    L.orc_set_dir_mode(int(m))


def dir_search(g: OracleGraph, kind: str, art: dict, queries: np.ndarray, k: int,
               beam_width: int, limit: int):
    """directional_search ('lsh') or pq_search ('pq') given the artifacts."""
    L = lib()
    L.orc_dir_search.argtypes = [C.POINTER(_Graph), C.POINTER(_Dir), C.c_void_p, C.c_uint32,
                                 C.c_uint32, C.c_uint32, C.c_uint32, C.c_void_p, C.c_void_p]
    L.orc_dir_search.restype = None
    keep = {}
    def arr(name, dtype):
        a = np.ascontiguousarray(art[name], dtype=dtype)
        keep[name] = a
        return _p(a)
    d = _Dir()
    if kind == "lsh":
        packed = np.ascontiguousarray(art["lsh_packed"])
        keep["packed"] = packed
        d.kind, d.k_ranks, d.packed_bytes = 0, int(art["k_ranks"]), packed.dtype.itemsize
        d.packed, d.mag_sq, d.c = _p(packed), arr("lsh_mag_sq", np.uint16), arr("lsh_c", np.float32)
        d.norm_denom = float(art["lsh_norm_denom"])
    else:
        cent = np.ascontiguousarray(art["pq_centroids"], np.float32)
        keep["cent"] = cent
        M = int(art["k_ranks"])
        d.kind, d.pq_m, d.pq_dsub = 1, M, cent.size // (M * 256)
        d.centroids, d.codes, d.norms = _p(cent), arr("pq_codes", np.uint8), arr("norms", np.float32)
    q = pad_rows(queries)
    nq = q.shape[0]
    oi = np.zeros((nq, k), np.uint32)
    od = np.zeros((nq, k), np.float32)
    gs = g._struct()
    L.orc_dir_search(C.byref(gs), C.byref(d), _p(q), nq, k, beam_width, limit, _p(oi), _p(od))
    return oi.view(np.int32), od


# ── directional artifact builders (the exact, sampling-free parts) ───────
def lsh_edges_exact(g: OracleGraph, k_ranks: int):
    """populate_lsh per edge: words [n, R * k_ranks] (uint8 for dpad <= 128,
    else uint16) and bf16 |Δ|² [n, R], bit-exact to the device builder."""
    L = lib()
    L.orc_lsh_edges.argtypes = [C.POINTER(_Graph), C.c_uint32, C.c_int, C.c_void_p, C.c_void_p]
    L.orc_lsh_edges.restype = None
    pb = 1 if g.dpad <= 128 else 2
    packed = np.zeros((g.n, g.R * k_ranks), np.uint8 if pb == 1 else np.uint16)
    mag = np.zeros((g.n, g.R), np.uint16)
    gs = g._struct()
    L.orc_lsh_edges(C.byref(gs), int(k_ranks), pb, _p(packed), _p(mag))
    return packed, mag


def pq_codes_exact(g: OracleGraph, centroids: np.ndarray):
    """pq_populate: codes [n, M * R] (subspace-major) for given centroids."""
    L = lib()
    L.orc_pq_codes.argtypes = [C.POINTER(_Graph), C.c_uint32, C.c_void_p, C.c_void_p]
    L.orc_pq_codes.restype = None
    cent = np.ascontiguousarray(centroids, np.float32)
    M = cent.shape[0]
    codes = np.zeros((g.n, M * g.R), np.uint8)
    gs = g._struct()
    L.orc_pq_codes(C.byref(gs), M, _p(cent), _p(codes))
    return codes


def row_norms_exact(g: OracleGraph):
    """pq_compute_vector_norms: exact |x|² per row, block-reduction order."""
    L = lib()
    L.orc_row_norms.argtypes = [C.POINTER(_Graph), C.c_void_p]
    L.orc_row_norms.restype = None
    out = np.zeros(g.n, np.float32)
    gs = g._struct()
    L.orc_row_norms(C.byref(gs), _p(out))
    return out


# ── RaBitQ (1 bit per dimension) ─────────────────────────────────────────
def rabitq_code_bytes(dim: int) -> int:
    return ((dim + 7) // 8 + 3) // 4 * 4


def rabitq_quantize(rows: np.ndarray, centroid: np.ndarray, ip: bool, with_err: bool = False):
    """rabitq_quantize_kernel<1> restated: rows [n, dim] float32 (already
    rotated) -> node store [n, code_bytes + 8] uint8 (and, with_err, the
    per-row error scale of the estimate used by the search filter)."""
    L = lib()
    L.orc_rabitq_quantize.argtypes = [C.c_void_p, C.c_uint64, C.c_uint64, C.c_uint32, C.c_void_p,
                                      C.c_int, C.c_void_p, C.c_void_p]
    L.orc_rabitq_quantize.restype = None
    x = np.ascontiguousarray(rows, np.float32)
    n, dim = x.shape
    c = np.ascontiguousarray(centroid, np.float32)
    out = np.zeros((n, rabitq_code_bytes(dim) + 8), np.uint8)
    err = np.zeros(n, np.float32) if with_err else None
    L.orc_rabitq_quantize(_p(x), n, dim, dim, _p(c), int(bool(ip)), _p(out), _p(err))
    return (out, err) if with_err else out


def set_rabitq_filter(store=None, centroid=None, err=None, margin: float = 0.0) -> None:
    """Make OracleGraph.search apply the RaBitQ candidate filter (None: off).
    The arrays must stay alive while it is set."""
    L = lib()
    L.orc_set_rabitq_filter.argtypes = [C.c_void_p, C.c_uint32, C.c_void_p, C.c_void_p, C.c_float,
                                        C.c_int]
    L.orc_set_rabitq_filter.restype = None
    if store is None:
        L.orc_set_rabitq_filter(None, 0, None, None, 0.0, 0)
        return
    L.orc_set_rabitq_filter(_p(store), store.shape[1], _p(centroid), _p(err), float(margin), 1)


def rabitq_centroid(g: "OracleGraph") -> np.ndarray:
    """Column means of the graph rows, double accumulation in row order."""
    L = lib()
    L.orc_rabitq_centroid.argtypes = [C.c_void_p, C.c_uint64, C.c_uint32, C.c_uint32, C.c_void_p]
    L.orc_rabitq_centroid.restype = None
    out = np.zeros(g.dim, np.float32)
    L.orc_rabitq_centroid(_p(g.vec), g.n, g.dim, g.dpad, _p(out))
    return out
