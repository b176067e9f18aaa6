"""The tvm_ffi module (jasper_b200/lib/libjasper_ffi.so) exports every op the
reference's Python package looks up by name (python/jasper/__init__.py:
117-149) and behaves like the reference's module when driven the same way."""
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
MOD = ROOT / "jasper_b200" / "lib" / "libjasper_ffi.so"
PLAIN_OPS = ["load", "construct", "search", "save", "get_vector", "mark_deleted",
             "consolidate", "compact", "append"]
CONFIGS = [f"f16_r{r}_{m}" for m in ("l2", "ip") for r in (8, 16, 32, 64)]
DIR_OPS = ["construct_directional", "build_lsh", "build_pq", "directional_search", "pq_search",
           "save_directional", "load_directional", "get_vector_directional",
           "get_directional_flags"]
DIR_CONFIGS = [f"f16_r{r}_{m}_k{kr}_{d}" for m in ("l2", "ip") for kr in (4, 16) for r in (32, 64)
               for d in ("d128", "d32678")]
AGNOSTIC = ["jasper_free_graph", "jasper_get_n_vectors", "jasper_get_n_tombstoned",
            "jasper_get_n_live", "jasper_reserve_ids", "jasper_get_dim"]


def module():
    tvm_ffi = pytest.importorskip("tvm_ffi")
    if not MOD.exists():
        pytest.fail(f"{MOD} not built (python -m jasper_b200.build)")
    return tvm_ffi.load_module(str(MOD))


def test_exports_reference_op_names():
    m = module()
    for cfg in CONFIGS:
        for op in PLAIN_OPS:
            assert getattr(m, f"jasper_{op}_{cfg}") is not None
    for cfg in DIR_CONFIGS:
        for op in DIR_OPS:
            assert getattr(m, f"jasper_{op}_{cfg}") is not None
    for name in AGNOSTIC:
        assert getattr(m, name) is not None


def test_invalid_handle_raises():
    m = module()
    with pytest.raises(Exception, match="Invalid handle"):
        m.jasper_get_dim(123456)


@pytest.mark.gpu
def test_reference_calling_convention_matches_golden(cuda):
    import torch
    from test_oracle import regen
    m = module()
    z = np.load(ROOT / "tests" / "golden" / "gauss_l2_r32.npz")
    X, Q = regen(z)
    cfg = "f16_r32_l2"
    h = getattr(m, f"jasper_construct_{cfg}")(torch.from_numpy(X).cuda(), 128, 1.2, 10**10, False)
    try:
        assert m.jasper_get_n_vectors(h) == 3000 and m.jasper_get_dim(h) == 128
        q = torch.from_numpy(Q).cuda()
        for bw in z["bws"]:
            bw = int(bw)
            oi = torch.empty(Q.shape[0], 10, dtype=torch.int32, device="cuda")
            od = torch.empty(Q.shape[0], 10, dtype=torch.float32, device="cuda")
            getattr(m, f"jasper_search_{cfg}")(h, q, oi, od, 10, bw, 2 * bw, False)
            torch.cuda.synchronize()
            np.testing.assert_array_equal(oi.cpu().numpy(), z[f"idx_bw{bw}"])
            np.testing.assert_array_equal(od.cpu().numpy().view(np.uint32),
                                          z[f"dist_bw{bw}"].view(np.uint32))
    finally:
        m.jasper_free_graph(h)


@pytest.mark.gpu
def test_reference_directional_calling_convention(cuda, tmp_path):
    """Directional ops driven as python/jasper/__init__.py:323-429 drives them."""
    import torch
    from jasper_b200 import synthetic
    m = module()
    cfg = "f16_r32_l2_k4_d128"
    X = torch.from_numpy(synthetic.gaussian(2000, 128, 81)).cuda()
    Q = torch.from_numpy(synthetic.gaussian(32, 128, 82)).cuda()
    h = getattr(m, f"jasper_construct_directional_{cfg}")(X, 128, 1.2, 10**10, False, True, 42)
    path = str(tmp_path / "d.graph")
    try:
        getattr(m, f"jasper_build_lsh_{cfg}")(h, 4096, 42)
        getattr(m, f"jasper_build_pq_{cfg}")(h, 2000, 3, 123)
        assert getattr(m, f"jasper_get_directional_flags_{cfg}")(h) == 3
        outs = []
        for op in ("directional_search", "pq_search"):
            oi = torch.empty(32, 10, dtype=torch.int32, device="cuda")
            od = torch.empty(32, 10, dtype=torch.float32, device="cuda")
            getattr(m, f"jasper_{op}_{cfg}")(h, Q, oi, od, 10, 64, 128, False)
            outs.append((oi, od))
        getattr(m, f"jasper_save_directional_{cfg}")(h, path)
        h2 = getattr(m, f"jasper_load_directional_{cfg}")(path, 128, False, True, 42)
        try:
            assert getattr(m, f"jasper_get_directional_flags_{cfg}")(h2) == 3
            for op, (ri, rd) in zip(("directional_search", "pq_search"), outs):
                oi = torch.empty(32, 10, dtype=torch.int32, device="cuda")
                od = torch.empty(32, 10, dtype=torch.float32, device="cuda")
                getattr(m, f"jasper_{op}_{cfg}")(h2, Q, oi, od, 10, 64, 128, False)
                torch.cuda.synchronize()
                assert torch.equal(oi, ri) and torch.equal(od, rd), op
            v = torch.empty(128, dtype=torch.float16, device="cuda")
            getattr(m, f"jasper_get_vector_directional_{cfg}")(h2, 5, v)
        finally:
            m.jasper_free_graph(h2)
    finally:
        m.jasper_free_graph(h)
