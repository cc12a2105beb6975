"""The training-side ops on the GPU against the oracle: gemm_tn (tensor.rs:
156-198), the depthwise-conv backward (autograd.rs:1050-1097) and the fused
AdamW step (optim.rs:33-72)."""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _sum_tol(terms_abs_sum, rel=1e-5):
    # Two summation orders of the same f32 terms differ by at most a few
    # ulps of the sum of |terms| per addition; 1e-5 of that sum bounds it
    # for the lengths used here.
    return rel * terms_abs_sum + 1e-6


@pytest.mark.parametrize("p,m,n", [(37, 50, 70), (1, 1, 1), (64, 64, 64), (1000, 129, 257), (4096, 512, 768)])
def test_gemm_tn_matches_the_oracle(gpu, orc, p, m, n):
    rng = np.random.default_rng(p + m + n)
    a = rng.standard_normal((p, m)).astype(np.float32)
    b = rng.standard_normal((p, n)).astype(np.float32)
    got = gpu.gemm_tn(a, b, p, m, n)
    ref = orc.gemm_tn(a, b, p, m, n)
    bound = _sum_tol(np.abs(a).T.astype(np.float64) @ np.abs(b).astype(np.float64))
    assert (np.abs(got - ref) <= bound).all()
    # selftest.rs:35-75 bound against the exact product.
    assert np.abs(got - a.T.astype(np.float64) @ b.astype(np.float64)).max() < 2e-3 * max(1.0, np.sqrt(p / 64))


def test_gemm_tn_edge_cases(gpu, orc):
    # p = 0 gives zeros; a zero A element skips its row of B even where that
    # row holds inf / NaN (tensor.rs:188-190).
    assert not gpu.gemm_tn(np.zeros(0), np.zeros(0), 0, 3, 5).any()
    a = np.array([[0.0, 1.0, 2.0], [3.0, 0.0, 1.0]], np.float32)
    b = np.array([[np.inf, 1.0], [np.nan, 2.0]], np.float32)
    got = gpu.gemm_tn(a, b, 2, 3, 2)
    ref = orc.gemm_tn(a, b, 2, 3, 2)
    assert np.array_equal(np.isnan(got), np.isnan(ref)) and np.array_equal(np.isinf(got), np.isinf(ref))
    fin = np.isfinite(ref)
    assert np.allclose(got[fin], ref[fin], atol=1e-6)


@pytest.mark.parametrize("batch,t,d,k", [(2, 3, 2, 6), (3, 17, 5, 4), (1, 1, 1, 1), (4, 300, 96, 7),
                                         (2, 2500, 33, 16)])
def test_dwconv_backward_matches_the_oracle(gpu, orc, batch, t, d, k):
    rng = np.random.default_rng(batch * 1000 + t + d + k)
    n = batch * t * d
    x = rng.standard_normal(n).astype(np.float32)
    w = rng.standard_normal(k * d).astype(np.float32)
    go = rng.standard_normal(n).astype(np.float32)
    gx0 = rng.standard_normal(n).astype(np.float32)
    gw0 = rng.standard_normal(k * d).astype(np.float32)
    gb0 = rng.standard_normal(d).astype(np.float32)
    gx, gw, gb = gpu.dwconv_backward(x, w, go, batch, t, d, k, gx=gx0, gw=gw0, gb=gb0)
    rx, rw, rb = orc.dwconv_backward(x, w, go, batch, t, d, k, gx=gx0, gw=gw0, gb=gb0)
    # gx: the reference's order, bit for bit.
    assert np.array_equal(gx, rx)
    # gw, gb: sums over batch * t rows in another fixed order.
    xs, gos = x.reshape(batch, t, d).astype(np.float64), go.reshape(batch, t, d).astype(np.float64)
    absw = np.zeros((k, d))
    for q in range(k):
        if q < t:
            absw[q] = np.abs(gos[:, q:] * xs[:, : t - q]).sum(axis=(0, 1))
    assert (np.abs(gw - rw).reshape(k, d) <= _sum_tol(absw + np.abs(gw0).reshape(k, d))).all()
    assert (np.abs(gb - rb) <= _sum_tol(np.abs(gos).sum(axis=(0, 1)) + np.abs(gb0))).all()
    # Deterministic: a second run gives the same bits.
    gx2, gw2, gb2 = gpu.dwconv_backward(x, w, go, batch, t, d, k, gx=gx0, gw=gw0, gb=gb0)
    assert np.array_equal(gx2, gx) and np.array_equal(gw2, gw) and np.array_equal(gb2, gb)


def test_dwconv_backward_partial_gradients(gpu, orc):
    # Any subset of the three gradients (Graph::backward's req flags).
    batch, t, d, k = 2, 9, 8, 3
    rng = np.random.default_rng(3)
    x, go = rng.standard_normal((2, batch * t * d)).astype(np.float32)
    w = rng.standard_normal(k * d).astype(np.float32)
    rx, rw, rb = orc.dwconv_backward(x, w, go, batch, t, d, k)
    gw = np.zeros(k * d, np.float32)
    gpu._check(gpu.lib().nk_dwconv_backward(gpu._ptr(x), None, gpu._ptr(go), None, gpu._ptr(gw), None,
                                            batch, t, d, k, 0))
    assert np.allclose(gw, rw, atol=1e-5)
    gx = np.zeros(batch * t * d, np.float32)
    gpu._check(gpu.lib().nk_dwconv_backward(None, gpu._ptr(w), gpu._ptr(go), gpu._ptr(gx), None, None,
                                            batch, t, d, k, 0))
    assert np.array_equal(gx, rx)


def test_adamw_matches_the_oracle_bit_for_bit(gpu, orc):
    rng = np.random.default_rng(5)
    n = 100_003  # not a multiple of the block size
    val = rng.standard_normal(n).astype(np.float32)
    m = np.zeros(n, np.float32)
    v = np.zeros(n, np.float32)
    ov, om, ovv = val.copy(), m.copy(), v.copy()
    for t in range(1, 7):
        g = (rng.standard_normal(n) * 10 ** rng.uniform(-6, 2, n)).astype(np.float32)
        decay, wd = t % 3 != 0, (0.0 if t == 5 else 0.05)
        val, m, v = gpu.adamw_step(val, g, m, v, lr=3e-3, t=t, decay=decay, wd=wd)
        ov, om, ovv = orc.adamw_step(ov, g, om, ovv, lr=3e-3, t=t, decay=decay, wd=wd)
        assert np.array_equal(val, ov) and np.array_equal(m, om) and np.array_equal(v, ovv), t


def test_adamw_converges(gpu):
    # selftest.rs:787 (test_optimizer): AdamW drives a least-squares fit down.
    rng = np.random.default_rng(9)
    A = rng.standard_normal((64, 16)).astype(np.float32)
    x_true = rng.standard_normal(16).astype(np.float32)
    y = A @ x_true
    x = np.zeros(16, np.float32)
    m = np.zeros(16, np.float32)
    v = np.zeros(16, np.float32)
    first = None
    for t in range(1, 401):
        r = A @ x - y
        mse = float((r * r).mean())
        first = mse if first is None else first
        g = (2.0 / len(y)) * (A.T @ r)
        x, m, v = gpu.adamw_step(x, g.astype(np.float32), m, v, lr=0.05, t=t, decay=False)
    assert mse < 1e-2 * first, (first, mse)


def test_adamw_non_finite_gradient_is_refused(gpu):
    z = np.zeros(5, np.float32)
    g = np.array([0.1, np.nan, 0.2, np.inf, -0.3], np.float32)
    with pytest.raises(gpu.NoeticError) as e:
        gpu.adamw_step(np.ones(5), g, z, z, lr=0.1, t=1)
    assert e.value.status == gpu.NK_ERR_INVALID
    with pytest.raises(gpu.NoeticError):
        gpu.adamw_step(np.array([1.0, np.nan]), np.zeros(2), np.zeros(2), np.zeros(2), lr=0.1, t=1)


def test_gemm_tn_tensor_core_path_with_non_finite_operands(gpu, orc):
    # Shapes the tcgen05 path takes (m, n >= 128); a non-finite element in B
    # (or A) sends the product to the exact kernel, which keeps kern_tn's
    # zero-skip semantics; p not a multiple of 4 exercises the K padding.
    rng = np.random.default_rng(21)
    p, m, n = 258, 130, 200
    a = rng.standard_normal((p, m)).astype(np.float32)
    b = rng.standard_normal((p, n)).astype(np.float32)
    a[5, :] = 0.0
    a[5, 3] = 2.0
    b[5, 7] = np.inf
    b[9, 11] = np.nan
    a[9, :] = 0.0
    got = gpu.gemm_tn(a, b, p, m, n)
    ref = orc.gemm_tn(a, b, p, m, n)
    assert np.array_equal(np.isnan(got), np.isnan(ref)) and np.array_equal(np.isinf(got), np.isinf(ref))
    fin = np.isfinite(ref)
    bound = 1e-5 * (np.abs(a).T.astype(np.float64) @ np.where(np.isfinite(b), np.abs(b), 0).astype(np.float64))
    assert (np.abs(got[fin] - ref[fin]) <= bound[fin] + 1e-6).all()
    # All finite at the same shape: the tensor-core result within the sum bound.
    b[5, 7], b[9, 11] = 1.0, -1.0
    got = gpu.gemm_tn(a, b, p, m, n)
    ref = orc.gemm_tn(a, b, p, m, n)
    bound = 1e-5 * (np.abs(a).T.astype(np.float64) @ np.abs(b).astype(np.float64)) + 1e-6
    assert (np.abs(got - ref) <= bound).all()
