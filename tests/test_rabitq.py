"""RaBitQ 1-bit quantizer: the CPU restatement (oracle/jasper_oracle.c)
against the reference's own quantizer outputs (tests/golden/rabitq/, written
by make_golden_rabitq.py with oracle/_ref/bin/ref_rabitq), and the
properties the reference's tests/test_rabitq.cu checks (layout sizes, 1-bit
codes, negative L2 rescale, identical rows quantize identically, L2 and IP
factors differ).  CPU only."""
import hashlib
import sys
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O

GOLDEN = Path(__file__).resolve().parent / "golden" / "rabitq"
sys.path.insert(0, str(GOLDEN.parent))


def golden_cases():
    return sorted(GOLDEN.glob("*.npz"))


def regen(z):
    from make_golden_rabitq import case_inputs
    X, c = case_inputs(int(z["n"]), int(z["dim"]), str(z["centroid"]), str(z["rows"]), int(z["seed"]))
    assert hashlib.sha256(X.tobytes()).hexdigest() == str(z["x_sha"]), "rows differ"
    return X, c


def rotation(dim, seed):
    from jasper_b200 import _lib
    P = np.zeros(dim * dim, np.float32)
    _lib.call("jb_rotation_matrix", dim, seed, P.ctypes.data)
    return P.reshape(dim, dim)   # row i = column i of P


def split(store, dim):
    cb = O.rabitq_code_bytes(dim)
    codes = store[:, :cb]
    f = np.ascontiguousarray(store[:, cb:cb + 8]).view(np.float32)
    return codes, f[:, 0], f[:, 1]


@pytest.mark.parametrize("dim,bits,code,node", [(128, 1, 16, 24), (97, 1, 16, 24), (960, 1, 120, 128),
                                                (32, 1, 4, 12)])
def test_node_layout(dim, bits, code, node):
    """layout.cuh code_bytes / node_bytes (test_rabitq.cu:98-141)."""
    assert O.rabitq_code_bytes(dim) == code
    assert O.rabitq_code_bytes(dim) + 8 == node


@pytest.mark.parametrize("path", golden_cases(), ids=lambda p: p.stem)
def test_oracle_matches_reference_golden(path):
    z = np.load(path)
    X, c = regen(z)
    n, dim, metric = int(z["n"]), int(z["dim"]), int(z["metric"])
    ref = z["store"].reshape(n, -1)
    rot = int(z["rotation_seed"])
    if rot < 0:
        got = O.rabitq_quantize(X, c, metric == 1)
        np.testing.assert_array_equal(got, ref)      # bit-exact
        return
    # the reference rotates rows by P^T and the centroid by P with cuBLAS; the
    # restatement gets float64-rotated inputs rounded to f32, so compare codes
    # (signs flip only for near-zero residuals) and factors with a tolerance
    M = rotation(dim, rot).astype(np.float64)          # M[i] = column i of P
    Xr = (X.astype(np.float64) @ M.T).astype(np.float32)
    cr = (M.T @ c.astype(np.float64)).astype(np.float32)
    got = O.rabitq_quantize(Xr, cr, metric == 1)
    gc, ga, gr = split(got, dim)
    rc, ra, rr = split(ref, dim)
    bits_g = np.unpackbits(gc, axis=1, bitorder="little")[:, :dim]
    bits_r = np.unpackbits(rc, axis=1, bitorder="little")[:, :dim]
    assert (bits_g == bits_r).mean() > 0.999
    np.testing.assert_allclose(ga, ra, rtol=1e-3, atol=1e-3)
    np.testing.assert_allclose(gr, rr, rtol=1e-3)


def test_reference_properties():
    rng = np.random.default_rng(42)
    X = rng.standard_normal((8, 32)).astype(np.float32)
    c = np.zeros(32, np.float32)
    st_l2 = O.rabitq_quantize(X, c, False)
    codes, f_add, f_rescale = split(st_l2, 32)
    assert np.isfinite(f_add).all() and np.isfinite(f_rescale).all()
    assert (f_rescale < 0).all()                                       # Rescale_IsNegative_L2
    bits = np.unpackbits(codes, axis=1, bitorder="little")[:, :32]
    np.testing.assert_array_equal(bits, (X >= 0).astype(np.uint8))     # code = sign of the residual
    st_ip = O.rabitq_quantize(X, c, True)
    assert np.abs(split(st_ip, 32)[1] - f_add).max() > 1e-6             # InnerProduct_DifferentFactors
    same = np.tile(np.arange(1, 17, dtype=np.float32), (4, 1))
    st = O.rabitq_quantize(same, np.zeros(16, np.float32), False)
    assert (st == st[0]).all()                                         # IdenticalVectors_SameQuantization


def test_estimator_tracks_distance():
    """<code - 1/2, q> scaled by the factors estimates |o - q|^2 (L2) and
    1 - <o, q> (IP) with small relative error on 960-d unit rows."""
    rng = np.random.default_rng(5)
    X = rng.standard_normal((400, 960)).astype(np.float32)
    X /= np.linalg.norm(X, axis=1, keepdims=True)
    Q = rng.standard_normal((20, 960)).astype(np.float32)
    Q /= np.linalg.norm(Q, axis=1, keepdims=True)
    c = X.mean(0).astype(np.float32)
    for ip in (False, True):
        st = O.rabitq_quantize(X, c, ip)
        codes, f_add, f_rescale = split(st, 960)
        xu = np.unpackbits(codes, axis=1, bitorder="little")[:, :960].astype(np.float64) - 0.5
        for q in Q[:5]:
            g = -(c @ q) if ip else ((q - c) ** 2).sum()
            est = f_add + f_rescale * (xu @ q) + g
            true = 1.0 - X @ q if ip else ((X - q) ** 2).sum(1)
            err = np.abs(est - true) / np.abs(true).mean()
            assert np.median(err) < 0.05, (ip, np.median(err))
