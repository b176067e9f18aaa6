"""ctypes binding of libjasper_b200.so (the C ABI declared in include/jasper_b200.h).

The library is built in-tree (``python -m jasper_b200.build``).  Loading fails
loudly when it is missing: there is no CPU fallback for any operation.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIB_PATH = Path(os.environ.get("JASPER_B200_LIB") or
                Path(__file__).resolve().parent / "lib" / "libjasper_b200.so")

JB_OK = 0
JB_ERR_INVALID_ARGUMENT = 1
JB_ERR_INVALID_HANDLE = 2
JB_ERR_IO = 3
JB_ERR_CUDA = 4
JB_ERR_RUNTIME = 5


class GraphInfo(C.Structure):
    _fields_ = [
        ("n_vectors", C.c_uint64),
        ("n_deleted", C.c_uint64),
        ("next_id", C.c_uint64),
        ("dim", C.c_uint32),
        ("n_neighbors", C.c_uint32),
        ("metric", C.c_int32),
        ("medoid", C.c_uint32),
        ("global_offset", C.c_uint32),
        ("on_host", C.c_int32),
        ("device", C.c_int32),
    ]


_P = C.c_void_p
_U32, _U64, _I32, _I64 = C.c_uint32, C.c_uint64, C.c_int32, C.c_int64

# name -> argument types (all return int status)
SIGNATURES: dict[str, list] = {
    "jb_abi_version": [],
    "jb_graph_construct": [_P, _U64, _U32, _U32, _U32, _I32, C.c_double, _U64, _I32, _P, C.POINTER(_I64)],
    "jb_graph_load": [C.c_char_p, _U32, _U32, _I32, _I32, C.POINTER(_I64)],
    "jb_graph_save": [_I64, C.c_char_p],
    "jb_graph_search": [_I64, _P, _U64, _U32, _P, _P, _U32, _U32, _U32, _P],
    "jb_graph_search_stats": [_I64, _P, _U64, _U32, _P, _P, _U32, _U32, _U32, _P, _P, _P],
    "jb_graph_search_host": [_I64, _P, _U64, _U32, _P, _P, _U32, _U32, _U32, _P],
    "jb_graph_search_noalloc": [_I64, _P, _U64, _U32, _P, _P, _U32, _U32, _U32, _P],
    "jb_graph_free": [_I64],
    "jb_graph_get_info": [_I64, C.POINTER(GraphInfo)],
    "jb_graph_get_vector": [_I64, _I64, _P],
    "jb_graph_reserve_ids": [_I64, _I64, _P],
    "jb_graph_mark_deleted": [_I64, _P, _U64],
    "jb_graph_create": [_P, _U64, _U32, _U32, _U32, _I32, _I32, C.POINTER(_I64)],
    "jb_graph_set_edges": [_I64, _P, _P, _P, _U32],
    "jb_graph_get_edges": [_I64, _P, _P, _P],
    "jb_graph_apply_global_offset": [_I64, _U32],
    "jb_rotation_matrix": [_U32, _U64, _P],
    "jb_graph_set_lsh": [_I64, _U32, _U32, _P, _P, _P, C.c_float],
    "jb_graph_set_pq": [_I64, _U32, _U32, _P, _P, _P],
    "jb_graph_get_directional_flags": [_I64, C.POINTER(_I32)],
    "jb_graph_directional_search": [_I64, _I32, _P, _U64, _U32, _P, _P, _U32, _U32, _U32, _P],
    "jb_merge_topk": [_P, _P, _U32, _U64, _U32, _P, _P, _P],
    "jb_search_set_warps_per_query": [_I32],
    "jb_graph_append": [_I64, _P, _U64, _U32, C.c_double, _P, _P],
    "jb_merge_topk_strided": [_P, _P, _U64, _U32, _U64, _U32, _P, _P, _P],
    "jb_graph_construct_directional": [_P, _U64, _U32, _U32, _U32, _I32, C.c_double, _U64, _I32,
                                       _I32, _U64, _P, C.POINTER(_I64)],
    "jb_graph_build_lsh": [_I64, _U32, _U64, _U64],
    "jb_graph_build_pq": [_I64, _U32, _U64, _U32, _U64],
    "jb_graph_save_directional": [_I64, C.c_char_p],
    "jb_graph_load_directional": [C.c_char_p, _U32, _U32, _I32, _U32, _I32, _I32, _U64,
                                  C.POINTER(_I64)],
    "jb_graph_get_lsh": [_I64, C.POINTER(_U32), C.POINTER(_U32), _P, _P, _P, C.POINTER(C.c_float)],
    "jb_graph_get_pq": [_I64, C.POINTER(_U32), C.POINTER(_U32), _P, _P, _P],
    "jb_rotate_rows": [_U32, _U64, _P, _P, _U64, _I32, _P],
    "jb_rabitq_quantize": [_P, _U64, _U32, _P, _P, _I32, _P, _P],
    "jb_graph_build_rabitq": [_I64],
    "jb_graph_set_rabitq": [_I64, _U32, _P, _P],
    "jb_graph_get_rabitq": [_I64, C.POINTER(_U32), _P, _P],
    "jb_graph_search_rabitq": [_I64, _P, _U64, _U32, _P, _P, _U32, _U32, _U32, C.c_float, _P, _P],
    "jb_graph_get_rabitq_err": [_I64, _P],
}


class JasperError(RuntimeError):
    """Raised when a libjasper_b200 call fails; `code` is the JB_ERR_* value."""

    def __init__(self, code: int, msg: str):
        super().__init__(msg)
        self.code = code


_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `python -m jasper_b200.build` "
                "(jasper_b200 has no CPU fallback)")
        L = C.CDLL(str(LIB_PATH))
        for name, argtypes in SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = argtypes
            fn.restype = C.c_int
        L.jb_last_error.argtypes = []
        L.jb_last_error.restype = C.c_char_p
        _lib = L
    return _lib


def call(name: str, *args) -> None:
    L = lib()
    rc = getattr(L, name)(*args)
    if rc != JB_OK:
        msg = L.jb_last_error().decode(errors="replace")
        if rc == JB_ERR_INVALID_ARGUMENT:
            raise ValueError(msg)
        if rc == JB_ERR_IO:
            raise OSError(msg)
        raise JasperError(rc, msg)
