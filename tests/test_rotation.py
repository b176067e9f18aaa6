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


@pytest.mark.gpu
@pytest.mark.parametrize("dim,n", [(128, 20000), (96, 3000), (200, 5000), (960, 2000), (40, 700),
                                   (256, 40000), (960, 12000), (128, 300000)])
def test_tensor_core_rotation_matches_reference_gemm(cuda, dim, n):
    """tcgen05 rotation GEMM vs the SIMT fp32-accumulate GEMM and a float64
    product of the same fp16 operands.  Tolerance per output: 1 fp16 ulp of
    the exact value (final rounding) plus the fp32 summation bound
    dim * 2^-24 * sum_k |x_k a_k| (the two GEMMs only sum in different
    orders)."""
    import torch
    from jasper_b200 import _lib
    rng = np.random.default_rng(dim)
    dpad = (dim + 7) // 8 * 8
    X = np.zeros((n, dpad), np.float16)
    X[:, :dim] = rng.standard_normal((n, dim)).astype(np.float16)
    x = torch.from_numpy(X.view(np.uint16)).cuda()
    outs = []
    for tc in (1, 0):
        y = torch.full((n, dpad), 0x7E00, dtype=torch.int16, device="cuda")
        _lib.call("jb_rotate_rows", dim, 7, x.data_ptr(), y.data_ptr(), n, tc,
                  torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        outs.append(y.cpu().numpy().view(np.float16).astype(np.float64))
    Yt, Ys = outs
    P = np.zeros((dim, dim), np.float32)
    _lib.call("jb_rotation_matrix", dim, 7, P.ctypes.data)
    A = P.astype(np.float16).astype(np.float64)      # row i = weights of output i
    Xd = X[:, :dim].astype(np.float64)
    exact = Xd @ A.T
    tol = (np.spacing(np.abs(exact).astype(np.float16)).astype(np.float64)
           + dim * 2.0 ** -24 * (np.abs(Xd) @ np.abs(A).T))
    for name, Y in (("tensor cores", Yt), ("simt", Ys)):
        err = np.abs(Y[:, :dim] - exact)
        bad = err > tol
        r, c = np.nonzero(bad)
        assert not bad.any(), (name, int(bad.sum()), r[:5], c[:5], err[bad][:5], tol[bad][:5])
    assert np.all(Yt[:, dim:] == 0)                    # pad lanes stay zero
    assert (Yt == Ys).mean() > 0.98
