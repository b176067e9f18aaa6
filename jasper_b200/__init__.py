"""jasper_b200 -- B200-native Vamana graph index with Jasper's Python surface.

Drop-in for ``jasper`` (saltsystemslab/Jasper, python/jasper/__init__.py):
the same ``Graph`` class (build / load / save / search / get_vector / ...),
config ids, defaults and helpers, backed by libjasper_b200.so (hand-written
sm_100a kernels behind the C ABI of include/jasper_b200.h) instead of the
reference's tvm_ffi module.  Torch tensors exist only at this boundary.
"""
from __future__ import annotations

import ctypes as C
import re
import struct
from enum import Enum

import numpy as np
import torch

from . import _lib
from ._lib import GraphInfo, JasperError

__all__ = [
    "DistanceFunc", "DataType", "Graph", "JasperError", "parse_storage_size", "read_bin",
    "read_groundtruth", "get_recall", "generate_groundtruth", "save_groundtruth",
]


class DistanceFunc(str, Enum):
    L2 = "l2"
    INNER_PRODUCT = "ip"


class DataType(str, Enum):
    FLOAT16 = "f16"


# Config registry of the reference (python/jasper/__init__.py:29-38).
_CONFIGS: dict[tuple[DataType, int, DistanceFunc], str] = {
    (DataType.FLOAT16, r, f): f"f16_r{r}_{f.value}"
    for f in (DistanceFunc.L2, DistanceFunc.INNER_PRODUCT) for r in (8, 16, 32, 64)
}

# Directional registry (python/jasper/__init__.py:66-84): key adds k_ranks and
# whether dim <= 128 (7-bit vs 15-bit packed LSH coordinates).
_DIRECTIONAL_CONFIGS: dict[tuple[DataType, int, DistanceFunc, int, bool], str] = {
    (DataType.FLOAT16, r, f, kr, le): f"f16_r{r}_{f.value}_k{kr}_{'d128' if le else 'd32678'}"
    for f in (DistanceFunc.L2, DistanceFunc.INNER_PRODUCT) for r in (32, 64)
    for kr in (4, 16) for le in (True, False)
}

_DTYPE_MAP = {DataType.FLOAT16: torch.float16}
_METRIC = {DistanceFunc.L2: 0, DistanceFunc.INNER_PRODUCT: 1}


def _resolve_config(data_type: DataType, n_neighbors: int, distance: DistanceFunc) -> str:
    key = (data_type, n_neighbors, distance)
    if key not in _CONFIGS:
        supported = "\n  ".join(f"({d.value}, R={r}, {f.value})" for (d, r, f) in _CONFIGS)
        raise ValueError(
            f"Unsupported config: data_type={data_type.value}, n_neighbors={n_neighbors}, "
            f"distance={distance.value}\nSupported configs:\n  {supported}")
    return _CONFIGS[key]


def _resolve_directional_config(data_type: DataType, n_neighbors: int, distance: DistanceFunc,
                                k_ranks: int, dim: int) -> str:
    key = (data_type, n_neighbors, distance, k_ranks, dim <= 128)
    if key not in _DIRECTIONAL_CONFIGS:
        raise ValueError(
            f"Unsupported directional config: data_type={data_type.value}, "
            f"n_neighbors={n_neighbors}, distance={distance.value}, k_ranks={k_ranks}, dim={dim}")
    return _DIRECTIONAL_CONFIGS[key]


# Storage sizes (python/jasper/__init__.py:152-171): SI and IEC units.
STORAGE_SIZE_RE = re.compile(r"^\s*([\d.]+)\s*([KMGTP]?i?B)\s*$", re.IGNORECASE)
STORAGE_UNITS = {"B": 1, "KB": 10**3, "MB": 10**6, "GB": 10**9, "TB": 10**12,
                 "KIB": 2**10, "MIB": 2**20, "GIB": 2**30, "TIB": 2**40}


def parse_storage_size(s: str) -> int:
    m = STORAGE_SIZE_RE.match(s)
    if not m:
        raise ValueError(f"Invalid storage size: {s}")
    value, unit = m.groups()
    if unit.upper() not in STORAGE_UNITS:
        raise ValueError(f"Invalid storage size: {s}")
    return int(float(value) * STORAGE_UNITS[unit.upper()])


def _stream_ptr(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _ptr(t: torch.Tensor) -> int:
    return t.data_ptr()


class Graph:
    """A GPU-resident Vamana graph index (same surface as ``jasper.Graph``)."""

    def __init__(self, handle: int, config_id: str, data_type: DataType, distance: DistanceFunc,
                 n_neighbors: int, dim: int, *, is_directional: bool = False,
                 k_ranks: int | None = None, has_lsh: bool = False, has_pq: bool = False,
                 prerotate: bool = False, prerotate_seed: int = 42):
        self._handle = handle
        self._config_id = config_id
        self._data_type = data_type
        self._distance = distance
        self._n_neighbors = n_neighbors
        self._dim = dim
        self._torch_dtype = _DTYPE_MAP[data_type]
        self._is_directional = is_directional
        self._k_ranks = k_ranks
        self._has_lsh = has_lsh
        self._has_pq = has_pq
        self._prerotate = prerotate
        self._prerotate_seed = prerotate_seed
        self._has_rabitq = False

    # ── construction / persistence ─────────────────────────────────────
    @classmethod
    def load(cls, path: str, dim: int, n_neighbors: int = 32,
             data_type: DataType | str = DataType.FLOAT16,
             distance: DistanceFunc | str = DistanceFunc.L2, on_host: bool = False,
             k_ranks: int | None = None, prerotate: bool = False,
             prerotate_seed: int = 42) -> "Graph":
        """Load a graph file (the reference's on-disk layout).  With ``k_ranks``
        the file is read as a directional graph: its LSH / PQ trailer, if any,
        is attached, and ``prerotate`` / ``prerotate_seed`` must repeat the
        build's (they are not stored in the file, as in the reference)."""
        data_type = DataType(data_type)
        distance = DistanceFunc(distance)
        h = C.c_int64(-1)
        if k_ranks is None:
            config_id = _resolve_config(data_type, n_neighbors, distance)
            _lib.call("jb_graph_load", str(path).encode(), dim, n_neighbors, _METRIC[distance],
                      int(on_host), C.byref(h))
            return cls(h.value, config_id, data_type, distance, n_neighbors, dim)
        config_id = _resolve_directional_config(data_type, n_neighbors, distance, k_ranks, dim)
        _lib.call("jb_graph_load_directional", str(path).encode(), dim, n_neighbors,
                  _METRIC[distance], int(k_ranks), int(on_host), int(bool(prerotate)),
                  int(prerotate_seed), C.byref(h))
        flags = C.c_int32(0)
        _lib.call("jb_graph_get_directional_flags", h.value, C.byref(flags))
        return cls(h.value, config_id, data_type, distance, n_neighbors, dim,
                   is_directional=True, k_ranks=k_ranks, has_lsh=bool(flags.value & 1),
                   has_pq=bool(flags.value & 2), prerotate=prerotate,
                   prerotate_seed=prerotate_seed)

    def save(self, path: str) -> None:
        """Write this graph in the reference's on-disk layout."""
        self._check_alive()
        fn = "jb_graph_save_directional" if self._is_directional else "jb_graph_save"
        _lib.call(fn, self._handle, str(path).encode())

    @classmethod
    def build(cls, vectors: torch.Tensor, n_neighbors: int = 32,
              distance: DistanceFunc | str = DistanceFunc.L2, alpha: float = 1.2,
              workspace_budget: str = "10GB", on_host: bool = False, build_lsh: bool = False,
              build_pq: bool = False, k_ranks: int = 4, prerotate: bool | None = None,
              prerotate_seed: int = 42, lsh_samples: int = 32768, lsh_seed: int = 42,
              pq_train: int = 40000, pq_kmeans_iter: int = 12, pq_seed: int = 123,
              build_rabitq: bool = False) -> "Graph":
        """Construct a graph from [n, dim] float16 vectors (CUDA or host tensor).

        ``build_lsh`` / ``build_pq`` / ``build_rabitq`` build a directional
        graph (prerotated unless ``prerotate=False``) with the corresponding
        estimator payloads; ``build_rabitq`` (1-bit RaBitQ codes of the rows,
        an addition of this package) enables :meth:`rabitq_search`."""
        distance = DistanceFunc(distance)
        budget = parse_storage_size(workspace_budget)
        if vectors.ndim != 2:
            raise ValueError(f"vectors must be 2D, got {vectors.ndim}D")
        if vectors.dtype != torch.float16:
            raise ValueError(f"Unsupported tensor dtype: {vectors.dtype}. Use torch.float16.")
        vectors = vectors.contiguous()
        n, dim = vectors.shape
        h = C.c_int64(-1)
        stream = _stream_ptr(vectors.device) if vectors.is_cuda else 0
        if vectors.is_cuda:
            torch.cuda.set_device(vectors.device)
        if not (build_lsh or build_pq or build_rabitq):
            config_id = _resolve_config(DataType.FLOAT16, n_neighbors, distance)
            _lib.call("jb_graph_construct", _ptr(vectors), n, dim, dim, n_neighbors,
                      _METRIC[distance], float(alpha), budget, int(on_host), stream, C.byref(h))
            return cls(h.value, config_id, DataType.FLOAT16, distance, n_neighbors, dim)
        config_id = _resolve_directional_config(DataType.FLOAT16, n_neighbors, distance, k_ranks,
                                                dim)
        resolved_prerotate = True if prerotate is None else bool(prerotate)
        _lib.call("jb_graph_construct_directional", _ptr(vectors), n, dim, dim, n_neighbors,
                  _METRIC[distance], float(alpha), budget, int(on_host),
                  int(resolved_prerotate), int(prerotate_seed), stream, C.byref(h))
        g = cls(h.value, config_id, DataType.FLOAT16, distance, n_neighbors, dim,
                is_directional=True, k_ranks=k_ranks, has_lsh=build_lsh, has_pq=build_pq,
                prerotate=resolved_prerotate, prerotate_seed=prerotate_seed)
        if build_lsh:
            _lib.call("jb_graph_build_lsh", h.value, int(k_ranks), int(lsh_samples), int(lsh_seed))
        if build_pq:
            _lib.call("jb_graph_build_pq", h.value, int(k_ranks), int(pq_train),
                      int(pq_kmeans_iter), int(pq_seed))
        if build_rabitq:
            _lib.call("jb_graph_build_rabitq", h.value)
            g._has_rabitq = True
        return g

    # ── properties ─────────────────────────────────────────────────────
    def _info(self) -> GraphInfo:
        self._check_alive()
        info = GraphInfo()
        _lib.call("jb_graph_get_info", self._handle, C.byref(info))
        return info

    @property
    def dim(self) -> int:
        return self._dim

    @property
    def n_vectors(self) -> int:
        return int(self._info().n_vectors)

    @property
    def n_neighbors(self) -> int:
        return self._n_neighbors

    @property
    def data_type(self) -> DataType:
        return self._data_type

    @property
    def distance(self) -> DistanceFunc:
        return self._distance

    @property
    def n_tombstoned(self) -> int:
        return int(self._info().n_deleted)

    @property
    def n_live(self) -> int:
        info = self._info()
        return int(info.n_vectors - info.n_deleted)

    # ── search ─────────────────────────────────────────────────────────
    def _check_queries(self, queries: torch.Tensor) -> torch.Tensor:
        if not queries.is_cuda:
            raise ValueError("queries must be a CUDA tensor")
        if queries.dtype != self._torch_dtype:
            raise ValueError(f"queries must be {self._torch_dtype}, got {queries.dtype}")
        if queries.ndim != 2:
            raise ValueError(f"queries must be 2D, got {queries.ndim}D")
        if queries.size(1) != self._dim:
            raise ValueError(f"query dim ({queries.size(1)}) != graph dim ({self._dim})")
        return queries.contiguous()

    def search(self, queries: torch.Tensor, k: int = 10, beam_width: int = 64,
               print_throughput: bool = False) -> tuple[torch.Tensor, torch.Tensor]:
        """Beam search; returns (int32 [nq, k] stable ids, float32 [nq, k] distances).

        ``limit`` is 2 x beam_width as in the reference (python/jasper/__init__.py:500-501).
        """
        self._check_alive()
        if self._is_directional:
            raise RuntimeError("search() is not available on a directional graph")
        queries = self._check_queries(queries)
        nq = queries.size(0)
        out_i = torch.empty(nq, k, dtype=torch.int32, device=queries.device)
        out_d = torch.empty(nq, k, dtype=torch.float32, device=queries.device)
        limit = beam_width * 2
        stream = _stream_ptr(queries.device)
        if print_throughput:
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
        _lib.call("jb_graph_search", self._handle, _ptr(queries), nq, self._dim, _ptr(out_i),
                  _ptr(out_d), k, beam_width, limit, stream)
        if print_throughput:
            e1.record()
            e1.synchronize()
            ms = e0.elapsed_time(e1)
            print(f"[beam_search] duration={ms}ms, throughput={nq * 1000.0 / max(ms, 1e-9)}")
        return out_i, out_d

    def search_with_stats(self, queries: torch.Tensor, k: int = 10, beam_width: int = 64,
                          limit: int | None = None, distinct: bool = False):
        """search() plus per-query counters [nq, 5]: expansions, expanded degree
        sum, distance evaluations, visited-table resets, distinct rows
        evaluated (exact only with ``distinct=True``, which needs
        nq * n_vectors / 8 bytes of scratch)."""
        self._check_alive()
        queries = self._check_queries(queries)
        nq = queries.size(0)
        out_i = torch.empty(nq, k, dtype=torch.int32, device=queries.device)
        out_d = torch.empty(nq, k, dtype=torch.float32, device=queries.device)
        stats = torch.zeros(nq, 5, dtype=torch.int32, device=queries.device)
        seen = None
        if distinct:
            words = (self.n_vectors + 31) // 32
            seen = torch.zeros(nq * words, dtype=torch.int32, device=queries.device)
        limit = beam_width * 2 if limit is None else limit
        _lib.call("jb_graph_search_stats", self._handle, _ptr(queries), nq, self._dim, _ptr(out_i),
                  _ptr(out_d), k, beam_width, limit, _ptr(stats),
                  None if seen is None else _ptr(seen), _stream_ptr(queries.device))
        return out_i, out_d, stats

    def _dir_search(self, kind: int, name: str, queries: torch.Tensor, k: int, beam_width: int,
                    limit: int | None, print_throughput: bool):
        queries = self._check_queries(queries)
        nq = queries.size(0)
        out_i = torch.empty(nq, k, dtype=torch.int32, device=queries.device)
        out_d = torch.empty(nq, k, dtype=torch.float32, device=queries.device)
        limit = beam_width * 2 if limit is None else limit
        if print_throughput:
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
        _lib.call("jb_graph_directional_search", self._handle, kind, _ptr(queries), nq,
                  self._dim, _ptr(out_i), _ptr(out_d), k, beam_width, limit,
                  _stream_ptr(queries.device))
        if print_throughput:
            e1.record()
            e1.synchronize()
            ms = e0.elapsed_time(e1)
            print(f"[{name}] duration={ms}ms, throughput={nq * 1000.0 / max(ms, 1e-9)}")
        return out_i, out_d

    def directional_search(self, queries: torch.Tensor, k: int = 10, beam_width: int = 64,
                           limit: int | None = None, print_throughput: bool = False):
        """Beam search scored by the cross-polytope LSH estimator (reference:
        python/jasper/__init__.py:525-567).  Queries are rotated in the call
        when the graph was prerotated.  ``limit`` defaults to 2 x beam_width."""
        self._check_alive()
        if not self._is_directional or not self._has_lsh:
            raise RuntimeError("directional_search() requires a graph built with build_lsh=True "
                               "(or loaded with LSH artifacts present)")
        return self._dir_search(0, "directional_search", queries, k, beam_width, limit,
                                print_throughput)

    def pq_search(self, queries: torch.Tensor, k: int = 10, beam_width: int = 64,
                  limit: int | None = None, print_throughput: bool = False):
        """Beam search scored by the PQ ADC estimator (reference:
        python/jasper/__init__.py:569-611)."""
        self._check_alive()
        if not self._is_directional or not self._has_pq:
            raise RuntimeError("pq_search() requires a graph built with build_pq=True "
                               "(or loaded with PQ artifacts present)")
        return self._dir_search(1, "pq_search", queries, k, beam_width, limit, print_throughput)

    def rabitq_search(self, queries: torch.Tensor, k: int = 10, beam_width: int = 128,
                      limit: int | None = None, margin: float = 1.0,
                      print_throughput: bool = False):
        """Beam search with exact distances where RaBitQ 1-bit estimates
        (codes built with ``build_rabitq=True``) skip neighbours that cannot
        enter the full beam: a neighbour is read only if its estimate minus
        ``margin`` error scales is below the beam's worst distance.  An
        addition of this package (the reference has no RaBitQ search).
        Returns (int32 [nq, k] ids, float32 [nq, k] exact distances)."""
        self._check_alive()
        if not self._is_directional or not self._has_rabitq:
            raise RuntimeError("rabitq_search() requires a graph built with build_rabitq=True")
        queries = self._check_queries(queries)
        nq = queries.size(0)
        out_i = torch.empty(nq, k, dtype=torch.int32, device=queries.device)
        out_d = torch.empty(nq, k, dtype=torch.float32, device=queries.device)
        limit = beam_width * 2 if limit is None else limit
        if print_throughput:
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
        _lib.call("jb_graph_search_rabitq", self._handle, _ptr(queries), nq, self._dim,
                  _ptr(out_i), _ptr(out_d), k, beam_width, limit, float(margin), None,
                  _stream_ptr(queries.device))
        if print_throughput:
            e1.record()
            e1.synchronize()
            ms = e0.elapsed_time(e1)
            print(f"[rabitq_search] duration={ms}ms, throughput={nq * 1000.0 / max(ms, 1e-9)}")
        return out_i, out_d

    # ── rows, ids, deletion ───────────────────────────────────────────
    def get_vector(self, stable_id: int) -> torch.Tensor:
        self._check_alive()
        if stable_id < 0:
            raise IndexError(f"stable_id must be non-negative, got {stable_id}")
        out = torch.empty(self._dim, dtype=self._torch_dtype, device="cuda")
        _lib.call("jb_graph_get_vector", self._handle, int(stable_id), _ptr(out))
        return out

    def reserve_ids(self, count: int) -> torch.Tensor:
        self._check_alive()
        if count <= 0:
            return torch.empty(0, dtype=torch.int32)
        out = torch.empty(count, dtype=torch.int32)
        _lib.call("jb_graph_reserve_ids", self._handle, int(count), _ptr(out))
        return out

    def mark_deleted(self, ids: torch.Tensor) -> None:
        self._check_alive()
        if ids.ndim != 1:
            raise ValueError(f"ids must be 1D, got {ids.ndim}D")
        ids = ids.detach().to(device="cpu", dtype=torch.int32).contiguous()
        if ids.numel() == 0:
            return
        _lib.call("jb_graph_mark_deleted", self._handle, _ptr(ids), ids.numel())

    def append(self, vectors: torch.Tensor, alpha: float = 1.2) -> torch.Tensor:
        """Append a batch of vectors to the live graph (python/jasper/
        __init__.py:673-697): the new rows are wired in with the
        construction's batched beam search + RobustPrune(alpha) and get
        fresh monotonic stable ids.  Returns the ids (int32, CPU) in input
        order."""
        self._check_alive()
        if not vectors.is_cuda:
            raise ValueError("vectors must be a CUDA tensor")
        if vectors.dtype != torch.float16:
            raise ValueError(f"vectors must be torch.float16, got {vectors.dtype}")
        if vectors.ndim != 2 or vectors.size(1) != self.dim:
            raise ValueError(f"vectors must be [n, {self.dim}]")
        vectors = vectors.contiguous()
        n = vectors.size(0)
        out_ids = torch.empty(n, dtype=torch.int32)
        _lib.call("jb_graph_append", self._handle, _ptr(vectors), n, vectors.size(1),
                  float(alpha), _ptr(out_ids), _stream_ptr(vectors.device))
        return out_ids

    def consolidate(self, alpha: float = 1.2) -> None:
        raise NotImplementedError("consolidate() is not part of this build")

    def compact(self) -> None:
        raise NotImplementedError("compact() is not part of this build")

    # ── lifetime ──────────────────────────────────────────────────────
    def free(self):
        if getattr(self, "_handle", None) is not None:
            try:
                _lib.call("jb_graph_free", self._handle)
            finally:
                self._handle = None

    def _check_alive(self):
        if self._handle is None:
            raise RuntimeError("Graph has been freed")

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass

    def __repr__(self) -> str:
        if self._handle is None:
            return "Graph(freed)"
        return (f"Graph(n_vectors={self.n_vectors}, dim={self.dim}, R={self._n_neighbors}, "
                f"dtype={self._data_type.value}, dist={self._distance.value})")


# ── Utils (python/jasper/__init__.py:770-946) ─────────────────────────────

def read_bin(path: str, dtype: str = "f32", max_vectors: int = 0) -> torch.Tensor:
    """Read a ``[u32 n][u32 dim][data]`` file (f32 or u8) as pinned float16."""
    if dtype == "f32":
        np_dtype = np.float32
    elif dtype == "u8":
        np_dtype = np.uint8
    elif dtype == "f16":
        np_dtype = np.float16
    else:
        raise ValueError(f"Unsupported dtype: {dtype!r}. Expected 'f32' or 'u8'.")
    with open(path, "rb") as f:
        n_vectors, dim = struct.unpack("II", f.read(8))
        if max_vectors > 0:
            n_vectors = min(n_vectors, max_vectors)
        nbytes = n_vectors * dim * np.dtype(np_dtype).itemsize
        data = np.frombuffer(f.read(nbytes), dtype=np_dtype).reshape(n_vectors, dim).copy()
    t = torch.from_numpy(data).to(torch.float16)
    return t.pin_memory() if torch.cuda.is_available() else t


def read_groundtruth(path: str, k: int = 10) -> tuple[torch.Tensor, torch.Tensor]:
    """Read ``[u32 nq][u32 k][u32 ids][f32 dists]`` ground truth."""
    with open(path, "rb") as f:
        n_queries, gt_k = struct.unpack("II", f.read(8))
        if gt_k < k:
            raise ValueError(f"Requested k={k} but ground truth only has k={gt_k}")
        ids = np.frombuffer(f.read(n_queries * gt_k * 4), dtype=np.uint32).reshape(n_queries, gt_k)
        dists = np.frombuffer(f.read(n_queries * gt_k * 4), dtype=np.float32).reshape(n_queries, gt_k)
    return (torch.from_numpy(ids[:, :k].copy()).to(dtype=torch.int32),
            torch.from_numpy(dists[:, :k].copy()))


def get_recall(gt, result_indices, k, n_queries, verbose: bool = True):
    """Set-intersection recall@k (python/jasper/__init__.py:819-826)."""
    count = sum(len(set(result_indices[i].tolist()) & set(gt[i].tolist())) for i in range(n_queries))
    recall = count / (n_queries * k)
    if verbose:
        print(f"Recall@{k}: {recall:.3f} ({count}/{(n_queries * k)})")
    return recall


def generate_groundtruth(vectors: torch.Tensor, queries: torch.Tensor, k: int = 100,
                         distance: str = "l2", query_batch_size: int = 1024,
                         vector_batch_size: int = 100_000, device: str = "cuda"):
    """Exact k-NN by streaming matmuls on the GPU (a utility, not the search path)."""
    n, dim = vectors.shape
    nq = queries.size(0)
    final_ids = torch.empty(nq, k, dtype=torch.int32)
    final_d = torch.empty(nq, k, dtype=torch.float32)
    for q0 in range(0, nq, query_batch_size):
        q = queries[q0:q0 + query_batch_size].to(device=device, dtype=torch.float32)
        qs = (q * q).sum(1, keepdim=True)
        top_d = torch.full((q.size(0), k), float("inf"), device=device)
        top_i = torch.zeros((q.size(0), k), dtype=torch.int64, device=device)
        for v0 in range(0, n, vector_batch_size):
            v = vectors[v0:v0 + vector_batch_size].to(device=device, dtype=torch.float32)
            if distance == "l2":
                d = (qs + (v * v).sum(1)[None, :] - 2.0 * (q @ v.T)).clamp_(min=0.0)
            elif distance == "ip":
                d = -(q @ v.T)
            else:
                raise ValueError(f"Unknown distance: {distance}")
            ids = torch.arange(v0, v0 + v.size(0), device=device)[None, :].expand(q.size(0), -1)
            md = torch.cat([top_d, d], 1)
            mi = torch.cat([top_i, ids], 1)
            top_d, sel = md.topk(k, dim=1, largest=False)
            top_i = mi.gather(1, sel)
        final_ids[q0:q0 + q.size(0)] = top_i.to(torch.int32).cpu()
        final_d[q0:q0 + q.size(0)] = top_d.cpu()
    return final_ids, final_d


def save_groundtruth(path: str, indices: torch.Tensor, distances: torch.Tensor):
    ids = indices.cpu().numpy().astype(np.uint32)
    dists = distances.cpu().numpy().astype(np.float32)
    nq, k = ids.shape
    with open(path, "wb") as f:
        f.write(struct.pack("II", nq, k))
        f.write(ids.tobytes())
        f.write(dists.tobytes())
