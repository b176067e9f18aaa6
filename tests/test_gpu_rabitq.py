"""RaBitQ on the GPU: the device quantizer against the reference's own
quantizer outputs and the CPU restatement (bit for bit), the codes of a
graph's rows, and the RaBitQ-estimated beam search against the restatement
of the same search (bit for bit; the search has no reference counterpart, so
its parity is unpinned), with a recall check against exact neighbours."""
import ctypes as C
from pathlib import Path

import numpy as np
import pytest

from jasper_b200 import _lib, synthetic
from oracle import oracle as O
import jb_testlib as T
from test_rabitq import golden_cases, regen, rotation, split

pytestmark = pytest.mark.gpu


@pytest.fixture(params=[1, 4], ids=["warp_per_query", "cta_per_query"], autouse=True)
def kernel_mode(request, cuda):
    """Every test runs on both query-search kernels (jb_search_set_warps_per_query:
    1 = a warp per query, 4 = a CTA per query)."""
    from jasper_b200 import _lib
    _lib.call("jb_search_set_warps_per_query", request.param)
    yield request.param
    _lib.call("jb_search_set_warps_per_query", 0)


def device_quantize(X, c, metric, rot=None):
    import torch
    x = torch.from_numpy(np.ascontiguousarray(X, np.float32)).cuda()
    cc = torch.from_numpy(np.ascontiguousarray(c, np.float32)).cuda()
    n, dim = X.shape
    out = torch.zeros(n * (O.rabitq_code_bytes(dim) + 8), dtype=torch.uint8, device="cuda")
    r = None
    if rot is not None:
        r = torch.from_numpy(np.ascontiguousarray(rot, np.float32).reshape(-1)).cuda()
    _lib.call("jb_rabitq_quantize", x.data_ptr(), n, dim, None if r is None else r.data_ptr(),
              cc.data_ptr(), metric, out.data_ptr(), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return out.cpu().numpy().reshape(n, -1)


@pytest.mark.parametrize("path", golden_cases(), ids=lambda p: p.stem)
def test_device_quantizer_matches_reference_golden(cuda, path):
    z = np.load(path)
    X, c = regen(z)
    n, dim, metric, rot = int(z["n"]), int(z["dim"]), int(z["metric"]), int(z["rotation_seed"])
    ref = z["store"].reshape(n, -1)
    if rot < 0:
        np.testing.assert_array_equal(device_quantize(X, c, metric), ref)
        return
    P = np.zeros(dim * dim, np.float32)
    _lib.call("jb_rotation_matrix", dim, rot, P.ctypes.data)
    got = device_quantize(X, c, metric, P)
    gc, ga, gr = split(got, dim)
    rc, ra, rr = split(ref, dim)
    bits_g = np.unpackbits(gc, axis=1, bitorder="little")[:, :dim]
    bits_r = np.unpackbits(rc, axis=1, bitorder="little")[:, :dim]
    assert (bits_g == bits_r).mean() > 0.999
    np.testing.assert_allclose(ga, ra, rtol=1e-3, atol=1e-3)
    np.testing.assert_allclose(gr, rr, rtol=1e-3)


@pytest.mark.parametrize("n,dim,metric", [(1000, 128, 0), (777, 97, 1), (300, 960, 1), (64, 8, 0)])
def test_device_quantizer_matches_oracle(cuda, n, dim, metric):
    rng = np.random.default_rng(dim)
    X = rng.standard_normal((n, dim)).astype(np.float32)
    c = (X.mean(0) + 0.1).astype(np.float32)
    np.testing.assert_array_equal(device_quantize(X, c, metric), O.rabitq_quantize(X, c, metric == 1))


CASES = [
    # data, n, dim, R, metric, prerotate
    ("relu_sphere", 3000, 960, 32, 1, True),
    ("relu_sphere", 3000, 128, 32, 1, False),
    ("gaussian", 2500, 128, 32, 0, True),
    ("gaussian", 2000, 200, 64, 0, False),
]


def search_rabitq(h, Q, k, bw, limit, margin, stats=False):
    import torch
    q = torch.from_numpy(O.pad_rows(Q)).cuda()
    nq = q.shape[0]
    oi = torch.empty(nq, k, dtype=torch.int32, device="cuda")
    od = torch.empty(nq, k, dtype=torch.float32, device="cuda")
    st = torch.zeros(nq, 5, dtype=torch.int32, device="cuda") if stats else None
    _lib.call("jb_graph_search_rabitq", h, q.data_ptr(), nq, q.shape[1], oi.data_ptr(),
              od.data_ptr(), k, bw, limit, float(margin), None if st is None else st.data_ptr(),
              torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    out = (oi.cpu().numpy(), od.cpu().numpy())
    return out + (st.cpu().numpy(),) if stats else out


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"{c[0]}-d{c[2]}-R{c[3]}-m{c[4]}-rot{int(c[5])}")
def test_rabitq_filtered_search_matches_oracle(cuda, case):
    kind, n, dim, R, metric, prerotate = case
    gen = getattr(synthetic, kind)
    X = gen(n, dim, 81)
    Q = gen(64, dim, 82) if kind == "gaussian" else gen(64, dim, 82, center_seed=81)
    alpha = 1.2 if metric == 0 else 1.0
    h = T.construct_directional(X, R, metric, alpha, prerotate, seed=4)
    try:
        _lib.call("jb_graph_build_rabitq", h)
        g = T.oracle_from_handle(h, n, dim, R, metric)
        nb = C.c_uint32(0)
        _lib.call("jb_graph_get_rabitq", h, C.byref(nb), None, None)
        store = np.zeros((n, nb.value), np.uint8)
        cent = np.zeros(dim, np.float32)
        err = np.zeros(n, np.float32)
        _lib.call("jb_graph_get_rabitq", h, None, store.ctypes.data, cent.ctypes.data)
        _lib.call("jb_graph_get_rabitq_err", h, err.ctypes.data)
        # codes and error scales of the stored rows around their column mean: bit-exact
        np.testing.assert_array_equal(cent.view(np.uint32), O.rabitq_centroid(g).view(np.uint32))
        rows = g.vec.view(np.float16)[:, :dim].astype(np.float32)
        ost, oerr = O.rabitq_quantize(rows, cent, metric == 1, with_err=True)
        np.testing.assert_array_equal(store, ost)
        np.testing.assert_array_equal(err.view(np.uint32), oerr.view(np.uint32))
        Qs = T.rotate_on_device(Q, dim, 4) if prerotate else Q   # the search's own query rotation
        try:
            for margin in (0.0, 1.0, 3.0):
                O.set_rabitq_filter(store, cent, err, margin)
                for k, bw, limit in [(10, 64, 128), (10, 128, 256), (20, 32, 64)]:
                    oi, od, _, oev = g.search(Qs, k, bw, limit)
                    ji, jd = search_rabitq(h, Q, k, bw, limit, margin)
                    T.assert_same_results(ji, jd, oi, od, msg=f"margin={margin} k={k} bw={bw}")
        finally:
            O.set_rabitq_filter(None)
        # the filter keeps the exact search's recall at margin 1 with fewer row reads
        gt, _ = O.bruteforce(g.vec.view(np.float16)[:, :dim], Qs, 10, metric)
        pi, pd = T.search(h, Qs, 10, 128)
        ri, rd, st = search_rabitq(h, Q, 10, 128, 256, 1.0, stats=True)
        _, _, pst = T.search(h, Qs, 10, 128, stats=True)
        rec = lambda ids: np.mean([len(set(a) & set(b)) / 10 for a, b in zip(ids, gt)])
        assert rec(ri) >= rec(pi) - 0.01, (rec(ri), rec(pi))
        assert st[:, 2].sum() < pst[:, 2].sum(), (st[:, 2].sum(), pst[:, 2].sum())
    finally:
        T.free(h)


def test_python_rabitq_surface(cuda):
    import torch
    import jasper_b200 as jasper
    X = torch.from_numpy(synthetic.relu_sphere(4000, 960, 83)).cuda()
    Q = torch.from_numpy(synthetic.relu_sphere(50, 960, 84, center_seed=83)).cuda()
    g = jasper.Graph.build(X, n_neighbors=64, distance="ip", alpha=1.0, build_rabitq=True)
    ids, d = g.rabitq_search(Q, k=10, beam_width=128)
    assert ids.shape == (50, 10) and ids.dtype == torch.int32
    from oracle import oracle as O2
    gt, _ = O2.bruteforce(X.cpu().numpy(), Q.cpu().numpy(), 10, 1)
    rec = np.mean([len(set(a) & set(b)) / 10 for a, b in zip(ids.cpu().numpy(), gt)])
    assert rec > 0.9, rec
    with pytest.raises(RuntimeError, match="build_lsh"):
        g.directional_search(Q)
    g.free()
