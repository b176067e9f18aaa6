"""Graph file I/O through the C ABI: reference-written files load, saves are
byte-identical to the reference's layout, and a round trip preserves search."""
from pathlib import Path
import ctypes as C
import struct

import numpy as np
import pytest

from jasper_b200 import _lib, synthetic
from oracle import oracle as O
import jb_testlib as T

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


def load(path, dim, R, metric=0):
    h = C.c_int64(-1)
    _lib.call("jb_graph_load", str(path).encode(), dim, R, metric, 0, C.byref(h))
    return h.value


def test_reference_file_loads_and_resaves_identically(cuda, tmp_path):
    f = GOLDEN / "gauss_l2_r16_file.graph"
    if not f.exists():
        pytest.skip("golden graph file not generated yet")
    h = load(f, 32, 16)
    try:
        out = tmp_path / "re.graph"
        _lib.call("jb_graph_save", h, str(out).encode())
        a, b = f.read_bytes(), out.read_bytes()
        assert len(a) == len(b)
        # node records: compare all but the edge slots past each row's count
        n, _, bpn = struct.unpack_from("<QQQ", a, 8)[0], None, struct.unpack_from("<Q", a, 24)[0]
        assert a[:32] == b[:32]
        dim, R = 32, 16
        for i in range(n):
            ra = a[32 + i * bpn: 32 + (i + 1) * bpn]
            rb = b[32 + i * bpn: 32 + (i + 1) * bpn]
            cnt = ra[2 * dim]
            assert ra[:2 * dim + 1] == rb[:2 * dim + 1]
            o = 2 * dim + 1
            assert ra[o:o + 4 * cnt] == rb[o:o + 4 * cnt]
            assert ra[o + 4 * R:o + 4 * R + 2 * cnt] == rb[o + 4 * R:o + 4 * R + 2 * cnt]
            assert ra[-4:] == rb[-4:]
        assert a[32 + n * bpn:] == b[32 + n * bpn:]
    finally:
        T.free(h)


def test_round_trip_preserves_search(cuda, tmp_path):
    X = synthetic.gaussian(2000, 100, 41)   # dim % 8 != 0: padded rows on device
    Q = synthetic.gaussian(50, 100, 42)
    h = T.construct(X, 32, 0, 1.2)
    try:
        p = tmp_path / "g.graph"
        _lib.call("jb_graph_save", h, str(p).encode())
        raw = p.read_bytes()
        total, n, medoid, bpn = struct.unpack_from("<4Q", raw, 0)
        assert total == len(raw) and n == 2000 and medoid == 0
        assert bpn == 2 * 100 + 1 + 6 * 32 + 4
        h2 = load(p, 100, 32)
        try:
            a = T.search(h, Q, 10, 64)
            b = T.search(h2, Q, 10, 64)
            T.assert_same_results(a[0], a[1], b[0], b[1])
        finally:
            T.free(h2)
    finally:
        T.free(h)


def test_legacy_layout_loads(cuda, tmp_path):
    """bytes_per_node without id/deletion columns (graph.cuh:1460-1479)."""
    X = synthetic.gaussian(300, 16, 43)
    g = O.OracleGraph(X, 8)
    g.build(1.2, 6)
    n, dim, R = 300, 16, 8
    bpn = 2 * dim + 1 + 6 * R
    buf = bytearray(struct.pack("<4Q", 32 + n * bpn, n, 0, bpn))
    for i in range(n):
        buf += X[i].tobytes() + bytes([g.counts[i]]) + g.edges[i].tobytes() + g.edist[i].tobytes()
    p = tmp_path / "legacy.graph"
    p.write_bytes(bytes(buf))
    h = load(p, dim, R)
    try:
        e, d, c = T.get_edges(h, n, R)
        np.testing.assert_array_equal(c, g.counts)
        Q = synthetic.gaussian(20, 16, 44)
        oi, od, _, _ = g.search(Q, 10, 32, 64)
        ji, jd = T.search(h, Q, 10, 32)
        T.assert_same_results(ji, jd, oi, od)
    finally:
        T.free(h)


def test_bad_files_raise(cuda, tmp_path):
    with pytest.raises(OSError):
        load(tmp_path / "missing.graph", 32, 16)
    p = tmp_path / "short.graph"
    p.write_bytes(struct.pack("<4Q", 0, 10, 0, 2 * 32 + 1 + 6 * 16 + 4) + b"\0" * 10)
    with pytest.raises(OSError):
        load(p, 32, 16)
    p2 = tmp_path / "wrong.graph"
    p2.write_bytes(struct.pack("<4Q", 0, 10, 0, 12345))
    with pytest.raises(OSError):
        load(p2, 32, 16)


def test_corrupt_records_rejected_before_any_kernel(cuda, tmp_path):
    """A file whose medoid, edge count or neighbour ids point outside the
    file is rejected by the loader itself: every kernel walks the first
    count edges of a row and gathers the rows they name."""
    X = synthetic.gaussian(400, 32, 45)
    h = T.construct(X, 16, 0, 1.2)
    try:
        p = tmp_path / "g.graph"
        _lib.call("jb_graph_save", h, str(p).encode())
    finally:
        T.free(h)
    raw = bytearray(p.read_bytes())
    n, dim, R = 400, 32, 16
    bpn = 2 * dim + 1 + 6 * R + 4
    T.free(load(p, dim, R))                                # the intact file loads
    cases = {}
    bad = bytearray(raw)
    struct.pack_into("<Q", bad, 16, n)                     # medoid == n
    cases["medoid"] = bad
    bad = bytearray(raw)
    bad[32 + 5 * bpn + 2 * dim] = R + 1                    # count > R
    cases["count"] = bad
    bad = bytearray(raw)
    o = 32 + 7 * bpn + 2 * dim
    assert bad[o] > 0
    struct.pack_into("<I", bad, o + 1, n)                  # first edge id == n
    cases["edge"] = bad
    for name, data in cases.items():
        q = tmp_path / f"{name}.graph"
        q.write_bytes(bytes(data))
        with pytest.raises((OSError, RuntimeError), match="medoid|edge count|neighbour id"):
            load(q, dim, R)
