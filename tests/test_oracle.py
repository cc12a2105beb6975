"""The CPU oracle against the reference's own known-answer and property tests
(transcribed in tests/golden/reference_kats.json) and its frozen regression
vectors.  No GPU needed."""

import json
import math
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _f(x):
    return float(x) if not isinstance(x, str) else float(x.replace("inf", "inf"))


@pytest.fixture(scope="module")
def kats():
    with open(os.path.join(GOLDEN, "reference_kats.json")) as f:
        return json.load(f)


@pytest.fixture(scope="module")
def regress():
    with open(os.path.join(GOLDEN, "oracle_regression.json")) as f:
        return json.load(f)


def test_zero_nucleus_keeps_exactly_the_best_token(orc, kats):
    k = kats["zero_nucleus"]
    logits = np.array([_f(v) for v in k["logits"]], dtype=np.float32)
    assert orc.sample_token(logits, orc.SampleCfg(**k["cfg"]), [], orc.Rng(k["rng_seed"])) == k["expected"]


def test_softmax_non_finite_inputs(orc, kats):
    k = kats["softmax_tied_infinities"]
    x = np.array([_f(v) for v in k["input"]], dtype=np.float32)
    orc.softmax_inplace(x)
    assert x.tolist() == k["expected"]
    k = kats["softmax_all_invalid"]
    x = np.array([_f(v) for v in k["input"]], dtype=np.float32)
    orc.softmax_inplace(x)
    assert np.all(np.abs(x - np.array(k["expected"])) < k["tol"])


def test_worker_count_thresholds(orc, kats):
    for req, jobs, work, want in kats["worker_count"]["cases"]:
        assert orc.worker_count(req, jobs, work) == want


def test_chunked_scan_matches_sequential_awkward_shapes(orc, kats):
    k = kats["scan_awkward_shapes"]
    rng = orc.Rng(k["rng_seed"])
    for batch, t, d, threads in k["shapes"]:
        n = batch * t * d
        a = np.array([rng.f32_unit() * np.float32(0.98) + np.float32(0.01) for _ in range(n)], dtype=np.float32)
        b = np.array([rng.normal() for _ in range(n)], dtype=np.float32)
        seq = orc.scan_sequential(a, b, batch, t, d, threads)
        chk = orc.scan_chunked(a, b, batch, t, d, threads)
        assert np.abs(seq - chk).max() < k["tol"], (batch, t, d, threads)


def test_scan_equivalence_selftest(orc, kats):
    k = kats["scan_equivalence"]
    batch, t, d = k["shape"]
    rng = orc.Rng(20250816)
    n = batch * t * d
    a = np.empty(n, np.float32)
    b = np.empty(n, np.float32)
    for i in range(n):
        a[i] = rng.f32_unit() * np.float32(0.98) + np.float32(0.01)
        b[i] = rng.normal()
    seq = orc.scan_sequential(a, b, batch, t, d, 2)
    par = orc.scan_chunked(a, b, batch, t, d, 2)
    assert np.abs(seq - par).max() < k["tol_chunked"]
    acc = np.float32(0.0)
    worst = 0.0
    for i in range(t):
        idx = i * d + k["channel"]
        acc = np.float32(a[idx] * acc + b[idx])
        worst = max(worst, abs(float(acc) - float(seq[idx])))
    assert worst < k["tol_scalar"]


def test_streaming_matches_batched(orc, kats):
    k = kats["stream_matches_batch"]
    m = orc.Model(orc.LmConfig(**k["cfg"]), seed=20250816)
    rng = orc.Rng(5)
    ids = np.array([rng.below(k["cfg"]["vocab"]) for _ in range(k["t"])], dtype=np.uint32)
    batched = m.logits(ids, 1, k["t"])
    dec = orc.Decoder(m)
    err = max(float(np.abs(dec.step(t) - batched[i]).max()) for i, t in enumerate(ids))
    # Same accumulation order on both paths: far inside the 1e-5 hard limit.
    assert err <= k["hard_limit"]


def test_streaming_matches_batched_awkward_configs(orc, kats):
    k = kats["stream_matches_batch_awkward"]
    for conv_k, n_layer, t in k["cases_conv_k_layers_t"]:
        r = orc.Rng(k["seed"])
        cfg = orc.LmConfig(vocab=k["vocab"], d_model=16, n_layer=n_layer, expand=2, conv_k=conv_k, mlp_mult=2,
                           eps=1e-5, tau_max=8.0)
        m = orc.Model(cfg, rng=r)
        ids = np.array([r.below(cfg.vocab) for _ in range(t)], dtype=np.uint32)
        batched = m.logits(ids, 1, t)
        dec = orc.Decoder(m)
        err = max(float(np.abs(dec.step(tok) - batched[i]).max()) for i, tok in enumerate(ids))
        assert err < k["tol"], (conv_k, n_layer, t, err)


def test_batched_prefill_state_equals_streaming_state(orc):
    cfg = orc.LmConfig(vocab=23, d_model=16, n_layer=2, expand=2, conv_k=3, mlp_mult=2, eps=1e-5, tau_max=8.0)
    m = orc.Model(cfg, seed=3)
    for t in [1, 2, 3, 7]:
        ids = np.arange(t, dtype=np.uint32) % 23
        st, heads, last = m.prefill_state(ids, 1, t)
        dec = orc.Decoder(m)
        for tok in ids:
            lg = dec.step(tok).copy()
        s2, h2 = dec.get_state()
        assert heads[0] == h2
        assert np.array_equal(st[0], s2)
        assert np.array_equal(last[0], lg)


def test_decoder_reset_matches_fresh(orc, kats):
    k = kats["decoder_reset"]
    m = orc.Model(orc.LmConfig(**k["cfg"]), seed=k["rng_seed"])
    dec = orc.Decoder(m)
    base = [dec.step(t).copy() for t in k["prompt"]]
    for t in k["junk"]:
        dec.step(t)
    dec.reset()
    for i, t in enumerate(k["prompt"]):
        assert np.abs(dec.step(t) - base[i]).max() < k["tol"]


def test_sampling_controls_stay_in_range(orc, kats):
    k = kats["sampling_controls"]
    rng = orc.Rng(k["rng_seed"])
    base = np.array([(i % 7) - 3 for i in range(k["vocab"])], dtype=np.float32)
    g = orc.SampleCfg(**k["greedy_cfg"])
    assert orc.sample_token(base.copy(), g, [], rng) == orc.sample_token(base.copy(), g, [], rng)
    s = orc.SampleCfg(**k["stochastic_cfg"])
    for _ in range(k["draws"]):
        assert 0 <= orc.sample_token(base.copy(), s, k["history"], rng) < k["vocab"]


def test_checkpoint_round_trip(orc, tmp_path):
    cfg = orc.LmConfig(vocab=40, d_model=24, n_layer=2, expand=2, conv_k=3, mlp_mult=2, eps=1e-5, tau_max=16.0)
    m = orc.Model(cfg, seed=3)
    p = str(tmp_path / "m.ckpt")
    m.save(p)
    m2 = orc.Model.load(p, orc.Rng(9999))
    for (n1, a1), (n2, a2) in zip(m.tensors(), m2.tensors()):
        assert n1 == n2 and np.array_equal(a1, a2)
    raw = bytearray(open(p, "rb").read())
    raw[40] ^= 0xFF
    bad = str(tmp_path / "bad.ckpt")
    open(bad, "wb").write(bytes(raw))
    with pytest.raises(IOError, match="CRC"):
        orc.Model.load(bad)


def test_crc32_matches_zlib(orc):
    import zlib

    for data in [b"", b"a", b"NOETIC\x00\x01", bytes(range(256)) * 3]:
        assert orc.crc32(data) == zlib.crc32(data)


# ---------------------------------------------------------------- RNG
# An independent restatement of rng.rs in pure Python: two implementations of
# the same text must agree bit-for-bit.
M64 = (1 << 64) - 1


def _splitmix(z):
    z = (z + 0x9E3779B97F4A7C15) & M64
    r = z
    r = ((r ^ (r >> 30)) * 0xBF58476D1CE4E5B9) & M64
    r = ((r ^ (r >> 27)) * 0x94D049BB133111EB) & M64
    return z, r ^ (r >> 31)


class PyRng:
    def __init__(self, seed):
        z = seed ^ 0xA0761D6478BD642F
        self.s = []
        for _ in range(4):
            z, v = _splitmix(z)
            self.s.append(v)
        if not any(self.s):
            self.s[0] = 0x9E3779B97F4A7C15

    def next_u64(self):
        s = self.s
        rotl = lambda x, k: ((x << k) | (x >> (64 - k))) & M64  # noqa: E731
        r = (rotl((s[0] + s[3]) & M64, 23) + s[0]) & M64
        t = (s[1] << 17) & M64
        s[2] ^= s[0]
        s[3] ^= s[1]
        s[1] ^= s[2]
        s[0] ^= s[3]
        s[2] ^= t
        s[3] = rotl(s[3], 45)
        return r

    def f32_unit(self):
        return float(np.float32(self.next_u64() >> 40) * np.float32(1.0 / 16777216.0))

    def below(self, n):
        if n == 1:
            return 0
        thr = ((1 << 64) - n) % n
        while True:
            r = self.next_u64()
            if r >= thr:
                return r % n


@pytest.mark.parametrize("seed", [0, 1, 7, 99, 20250816, 2**63 + 5, 2**64 - 1])
def test_rng_restatements_agree(orc, seed):
    a, b = orc.Rng(seed), PyRng(seed)
    assert a.s == b.s
    for _ in range(64):
        assert a.next_u64() == b.next_u64()
    for _ in range(64):
        assert a.f32_unit() == b.f32_unit()
    for n in [1, 2, 3, 7, 1000, 2**40 + 3, 2**63 + 1]:
        assert a.below(n) == b.below(n)


def test_oracle_regression_vectors(orc, regress):
    for seed, v in regress["rng"].items():
        r = orc.Rng(int(seed))
        assert [str(x) for x in r.s] == v["state"]
        assert [str(r.next_u64()) for _ in range(4)] == v["next_u64"]
        assert [r.f32_unit() for _ in range(4)] == v["f32_unit"]
        assert [r.below(1000) for _ in range(4)] == v["below_1000"]
        assert [r.normal() for _ in range(4)] == v["normal"]
    t = regress["tiny_model"]
    m = orc.Model(orc.LmConfig(**t["cfg"]), seed=t["seed"])
    for name, a in m.tensors():
        ref = t["tensors"][name]
        assert list(a.shape) == ref["shape"]
        assert float(np.asarray(a, np.float64).sum()) == ref["sum"]
    dec = orc.Decoder(m)
    for tok, row in zip(t["prompt"], t["stream_logits"]):
        assert dec.step(tok).tolist() == row


def test_normal_moments(orc):
    # selftest.rs:433-457 style sanity: N(0,1) mean/variance.
    r = orc.Rng(20250816)
    x = np.array([r.normal() for _ in range(20000)])
    assert abs(x.mean()) < 0.03 and abs(x.var() - 1.0) < 0.05
    u = np.array([r.f32_unit() for _ in range(20000)])
    assert u.min() >= 0.0 and u.max() < 1.0 and abs(u.mean() - 0.5) < 0.01
    assert math.isfinite(float(x.sum()))


def test_softmax_ce_restatement(orc):
    # Graph::softmax_ce forward (autograd.rs:579-624) against an f64 numpy
    # statement of the same sums: ignored targets, an all-ignored batch, the
    # 1e-20 probability floor and the non-finite / out-of-range rejections.
    rng = np.random.default_rng(7)
    lg = rng.normal(size=(9, 13)).astype(np.float32) * 3
    lg[4, 5] = 90.0  # one row whose other probabilities underflow the floor
    tg = rng.integers(0, 13, size=9).astype(np.uint32)
    tg[2] = 0xFFFFFFFF
    tg[4] = 0
    x = lg.astype(np.float64)
    p = np.exp(x - x.max(1, keepdims=True))
    p /= p.sum(1, keepdims=True)
    keep = tg != 0xFFFFFFFF
    ref = -np.log(np.maximum(p[np.arange(9)[keep], tg[keep]], 1e-20)).mean()
    assert abs(orc.softmax_ce(lg, tg) - ref) < 1e-5
    assert orc.softmax_ce(lg, np.full(9, 0xFFFFFFFF, np.uint32)) == 0.0
    bad = lg.copy()
    bad[0, 0] = np.inf
    with pytest.raises(ValueError, match="finite"):
        orc.softmax_ce(bad, tg)
    with pytest.raises(ValueError, match="range"):
        orc.softmax_ce(lg, np.full(9, 13, np.uint32))


def test_lm_loss_is_softmax_ce_of_lm_logits(orc):
    cfg = orc.LmConfig(vocab=31, d_model=16, n_layer=2, expand=2, conv_k=3, mlp_mult=2, eps=1e-5, tau_max=8.0)
    m = orc.Model(cfg, seed=11)
    r = orc.Rng(4)
    ids = np.array([r.below(31) for _ in range(3 * 7)], dtype=np.uint32)
    tg = np.roll(ids, -1)
    loss, lg = m.loss(ids, tg, 3, 7, want_logits=True)
    assert np.array_equal(lg, m.logits(ids, 3, 7))
    assert loss == orc.softmax_ce(lg, tg)


def test_scan_adjoint_closed_form(orc):
    # scan.rs:291-315: c_t = sum_{s >= t} g_s prod_{r=t+1..s} a_r, with the
    # reference's draws (Rng::new(5): a = f32_unit, then g = normal).
    batch, t, d = 2, 6, 2
    n = batch * t * d
    rng = orc.Rng(5)
    a = np.array([rng.f32_unit() for _ in range(n)], dtype=np.float32)
    g = np.array([rng.normal() for _ in range(n)], dtype=np.float32)
    c = orc.scan_adjoint(a, g, batch, t, d)
    for bi in range(batch):
        for j in range(d):
            for ti in range(t):
                exp, prod = np.float32(0.0), np.float32(1.0)
                for s in range(ti, t):
                    if s > ti:
                        prod = np.float32(prod * a[(bi * t + s) * d + j])
                    exp = np.float32(exp + g[(bi * t + s) * d + j] * prod)
                assert abs(exp - c[(bi * t + ti) * d + j]) < 1e-4


def _dwconv_forward64(x, w, b, batch, t, d, k):
    """autograd.rs:550-575 in float64: y = bias + sum_{q < min(t+1, k)} w[q] x[t-q]."""
    x = x.reshape(batch, t, d).astype(np.float64)
    w = w.reshape(k, d).astype(np.float64)
    y = np.broadcast_to(b.astype(np.float64), (batch, t, d)).copy()
    for ti in range(t):
        for q in range(min(ti + 1, k)):
            y[:, ti] += w[q] * x[:, ti - q]
    return y


def test_gemm_tn_restatement(orc):
    # selftest.rs:35-75: gemm_tn of the transposed A against a naive product, 2e-3.
    rng = np.random.default_rng(7)
    for p, m, n in [(33, 17, 29), (1, 5, 3), (64, 64, 64)]:
        a = rng.standard_normal((p, m)).astype(np.float32)
        b = rng.standard_normal((p, n)).astype(np.float32)
        c = orc.gemm_tn(a, b, p, m, n)
        assert np.abs(c - a.T.astype(np.float64) @ b.astype(np.float64)).max() < 2e-3
    # p = 0: C = 0; a zero A element skips its (non-finite) row of B (tensor.rs:188-190).
    assert not orc.gemm_tn(np.zeros(0), np.zeros(0), 0, 3, 4).any()
    a = np.array([[0.0, 1.0]], np.float32)
    b = np.array([[np.inf, 2.0]], np.float32)
    assert np.array_equal(orc.gemm_tn(a, b, 1, 2, 2), np.array([[0.0, 0.0], [np.inf, 2.0]], np.float32))


def test_dwconv_backward_restatement(orc):
    # selftest.rs:722-784: the three gradients of sum(dwconv(x, w, b) * m)
    # against central differences, with a kernel longer than the sequence.
    for batch, t, d, k in [(2, 3, 2, 6), (3, 7, 4, 3)]:
        rng = np.random.default_rng(batch * 100 + k)
        x = rng.standard_normal(batch * t * d).astype(np.float32)
        w = (rng.standard_normal(k * d) * 0.5).astype(np.float32)
        b = (rng.standard_normal(d) * 0.1).astype(np.float32)
        m = rng.standard_normal(batch * t * d).astype(np.float32)
        gx, gw, gb = orc.dwconv_backward(x, w, m, batch, t, d, k)

        def loss(xs, ws, bs):
            return float((_dwconv_forward64(xs, ws, bs, batch, t, d, k).reshape(-1) * m).sum())

        eps = 1e-3
        for arr, grad, which in [(x, gx, 0), (w, gw, 1), (b, gb, 2)]:
            for i in range(arr.size):
                plus, minus = arr.astype(np.float64).copy(), arr.astype(np.float64).copy()
                plus[i] += eps
                minus[i] -= eps
                args_p = [x.astype(np.float64), w.astype(np.float64), b.astype(np.float64)]
                args_m = list(args_p)
                args_p[which], args_m[which] = plus, minus
                fd = (loss(*args_p) - loss(*args_m)) / (2 * eps)
                assert abs(fd - grad[i]) / (1 + abs(fd)) < 5e-3, (batch, t, d, k, which, i)
    # The gradients add into what the buffers held (Graph::backward accumulates).
    gx0 = np.full(batch * t * d, 0.5, np.float32)
    gx2, gw2, gb2 = orc.dwconv_backward(x, w, m, batch, t, d, k, gx=gx0, gw=np.ones(k * d), gb=np.ones(d))
    assert np.allclose(gx2, gx + 0.5, atol=1e-6) and np.allclose(gw2, gw + 1, atol=1e-5)
    assert np.allclose(gb2, gb + 1, atol=1e-6)


def _powf(x, y):
    """The C library's powf, which Rust's f32::powf calls (numpy's float32
    power rounds differently in the last place for some arguments)."""
    import ctypes

    libm = ctypes.CDLL("libm.so.6")
    libm.powf.restype = ctypes.c_float
    libm.powf.argtypes = [ctypes.c_float, ctypes.c_float]
    return np.float32(libm.powf(float(x), float(y)))


def _adamw_numpy(val, grad, m, v, lr, t, decay, b1=0.9, b2=0.95, eps=1e-8, wd=0.0):
    """optim.rs:43-71 in numpy float32 (every operation rounded to f32)."""
    f = np.float32
    b1, b2, eps, wd, lr = f(b1), f(b2), f(eps), f(wd), f(lr)
    inv_bc1 = f(1) / (f(1) - _powf(b1, t))
    inv_bc2 = f(1) / (f(1) - _powf(b2, t))
    mi = b1 * m + (f(1) - b1) * grad
    vi = b2 * v + (f(1) - b2) * grad * grad
    upd = (mi * inv_bc1) / (np.sqrt(vi * inv_bc2) + eps)
    if decay and wd != 0:
        upd = upd + wd * val
    return val - lr * upd, mi, vi


def test_adamw_restatement(orc):
    rng = np.random.default_rng(11)
    n = 1000
    val = rng.standard_normal(n).astype(np.float32)
    m = np.zeros(n, np.float32)
    v = np.zeros(n, np.float32)
    ev, em, ev2 = val.copy(), m.copy(), v.copy()
    for t in range(1, 8):
        g = rng.standard_normal(n).astype(np.float32)
        decay = t % 2 == 0
        val, m, v = orc.adamw_step(val, g, m, v, lr=1e-2, t=t, decay=decay, wd=0.1)
        ev, em, ev2 = _adamw_numpy(ev, g, em, ev2, 1e-2, t, decay, wd=0.1)
        assert np.array_equal(val, ev) and np.array_equal(m, em) and np.array_equal(v, ev2), t
    # The first step moves every weight by lr * sign(g) (m_hat / sqrt(v_hat) = +-1).
    v1, _, _ = orc.adamw_step(np.zeros(3), np.array([2.0, -0.5, 0.0]), np.zeros(3), np.zeros(3), lr=0.1, t=1)
    assert np.allclose(v1, [-0.1, 0.1, 0.0], atol=1e-6)
    # The reference's assertions (optim.rs:34-38, 55-56).
    for kw in [dict(lr=-1.0), dict(lr=0.1, b1=1.0), dict(lr=0.1, b2=-0.1), dict(lr=0.1, eps=0.0),
               dict(lr=0.1, wd=float("nan"))]:
        with pytest.raises(ValueError):
            orc.adamw_step(np.zeros(2), np.zeros(2), np.zeros(2), np.zeros(2), t=1, **kw)
    with pytest.raises(ValueError):
        orc.adamw_step(np.zeros(2), np.array([0.0, np.nan]), np.zeros(2), np.zeros(2), lr=0.1, t=1)
