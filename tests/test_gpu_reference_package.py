"""Drop-in check with the reference's own, unmodified Python package.

The reference's `jasper` package (python/jasper/__init__.py, installed
unchanged into oracle/_ref/python by the build step) loads
`<package>/lib/libjasper_ffi.so` with tvm_ffi and looks its ops up by name
(python/jasper/__init__.py:12-14,117-149).  Here that `lib/` is this build's
library directory, so the reference's own Graph.build / search / save /
load / get_vector / directional_search / pq_search run on this build's
kernels.  Their results are compared with fixtures the reference itself
wrote (tests/golden/), bit for bit.
"""
from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

import numpy as np
import pytest

import jb_testlib as T
from jasper_b200 import _lib

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]
PKG_SRC = ROOT / "oracle" / "_ref" / "python" / "jasper" / "__init__.py"
OUR_LIB = ROOT / "jasper_b200" / "lib"
GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def refpkg(cuda, tmp_path_factory):
    pytest.importorskip("tvm_ffi")
    if not PKG_SRC.exists():
        pytest.skip("reference package not installed under oracle/_ref/python (build step)")
    if not (OUR_LIB / "libjasper_ffi.so").exists():
        pytest.fail("jasper_b200/lib/libjasper_ffi.so not built")
    pkg = tmp_path_factory.mktemp("refpkg") / "jasper"
    pkg.mkdir()
    (pkg / "__init__.py").write_bytes(PKG_SRC.read_bytes())
    (pkg / "lib").symlink_to(OUR_LIB, target_is_directory=True)
    name = "jasper_reference_package_under_test"
    spec = importlib.util.spec_from_file_location(name, pkg / "__init__.py",
                                                  submodule_search_locations=[str(pkg)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    try:
        spec.loader.exec_module(mod)
        yield mod
    finally:
        sys.modules.pop(name, None)


@pytest.mark.parametrize("case", ["gauss_l2_r32", "int_l2_r64", "gauss_ip_r32"])
def test_reference_package_plain_path(refpkg, case, tmp_path):
    import torch
    from test_oracle import regen
    z = np.load(GOLDEN / f"{case}.npz")
    X, Q = regen(z)
    R, metric = int(z["R"]), str(z["metric"])
    Xd = torch.from_numpy(X).cuda()
    Qd = torch.from_numpy(Q).cuda()
    g = refpkg.Graph.build(Xd, n_neighbors=R, distance=metric, alpha=float(z["alpha"]))
    try:
        for bw in z["bws"]:
            bw = int(bw)
            ids, dist = g.search(Qd, k=10, beam_width=bw)
            T.assert_same_results(ids.cpu().numpy(), dist.cpu().numpy(), z[f"idx_bw{bw}"],
                                  z[f"dist_bw{bw}"], msg=f"{case} bw={bw}")
        p = tmp_path / "g.graph"
        g.save(str(p))
        v = g.get_vector(5)
        np.testing.assert_array_equal(v.cpu().numpy().view(np.uint16), X[5].view(np.uint16))
    finally:
        g.free()
    # the reference package's append (python/jasper/__init__.py:673-697) on a
    # graph of the first 80 % of the rows: ids continue the sequence and the
    # appended rows find themselves
    n0 = X.shape[0] * 4 // 5
    ga = refpkg.Graph.build(Xd[:n0], n_neighbors=R, distance=metric, alpha=float(z["alpha"]))
    try:
        ids = ga.append(Xd[n0:], alpha=float(z["alpha"]))
        assert ids.tolist() == list(range(n0, X.shape[0]))
        if metric == "l2":
            found, _ = ga.search(Xd[n0:], k=1, beam_width=64)
            base, _ = ga.search(Xd[:300], k=1, beam_width=64)
            own = (base[:, 0].cpu() == torch.arange(300)).float().mean().item()
            assert (found[:, 0].cpu() == ids).float().mean().item() >= own - 0.03
    finally:
        ga.free()
    g2 = refpkg.Graph.load(str(p), dim=X.shape[1], n_neighbors=R, distance=metric)
    try:
        bw = int(z["bws"][-1])
        ids, dist = g2.search(Qd, k=10, beam_width=bw)
        T.assert_same_results(ids.cpu().numpy(), dist.cpu().numpy(), z[f"idx_bw{bw}"],
                              z[f"dist_bw{bw}"], msg=f"{case} reloaded bw={bw}")
    finally:
        g2.free()


@pytest.mark.parametrize("path", sorted((GOLDEN / "directional").glob("*.npz")),
                         ids=lambda p: p.stem)
def test_reference_package_directional_path(refpkg, path, tmp_path):
    """A directional file (golden graph + golden payloads, written by this
    build) loaded by the reference package; its directional_search and
    pq_search equal the reference's own outputs on those payloads."""
    import torch
    from test_oracle import regen, oracle_from_golden
    z = np.load(path)
    X, Q = regen(z)
    kr, R, metric = int(z["k_ranks"]), int(z["R"]), str(z["metric"])
    h = T.create_graph(oracle_from_golden(z, X))
    p = tmp_path / "d.graph"
    try:
        T.set_artifacts(h, z, kr)
        _lib.call("jb_graph_save_directional", h, str(p).encode())
    finally:
        T.free(h)
    g = refpkg.Graph.load(str(p), dim=X.shape[1], n_neighbors=R, distance=metric, k_ranks=kr,
                          prerotate=False)
    try:
        Qd = torch.from_numpy(Q).cuda()
        for name in ("directional_search", "pq_search"):
            for bw in z["bws"]:
                bw = int(bw)
                ids, dist = getattr(g, name)(Qd, k=10, beam_width=bw)
                T.assert_same_results(ids.cpu().numpy(), dist.cpu().numpy(),
                                      z[f"{name}_idx_bw{bw}"], z[f"{name}_dist_bw{bw}"],
                                      msg=f"{path.stem} {name} bw={bw}")
    finally:
        g.free()
