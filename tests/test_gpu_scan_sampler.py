"""GPU prefix scans (scan.rs) and the device sampler (infer.rs:228-305)
against the CPU oracle."""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


# ---------------------------------------------------------------- scans
def _scan_inputs(orc, rng, n):
    a = np.array([rng.f32_unit() * np.float32(0.98) + np.float32(0.01) for _ in range(n)], dtype=np.float32)
    b = np.array([rng.normal() for _ in range(n)], dtype=np.float32)
    return a, b


def test_scans_match_oracle_on_awkward_shapes(gpu, orc):
    # scan.rs:269-288 shape table, seed 99, tolerance 1e-4.
    rng = orc.Rng(99)
    for batch, t, d, threads in [(1, 1, 1, 1), (3, 7, 5, 3), (2, 129, 3, 4), (5, 64, 1, 8), (1, 1024, 9, 4),
                                 (2, 1000, 4, 3)]:
        a, b = _scan_inputs(orc, rng, batch * t * d)
        ref = orc.scan_sequential(a, b, batch, t, d, 1)
        assert np.abs(gpu.scan_sequential(a, b, batch, t, d) - ref).max() < 1e-4
        assert np.abs(gpu.scan_chunked(a, b, batch, t, d) - ref).max() < 1e-4


def test_chunked_scan_long_sequences(gpu, orc):
    rs = np.random.default_rng(5)
    for batch, t, d in [(1, 8192, 256), (2, 5000, 33), (4, 777, 1)]:
        a = rs.uniform(0.01, 0.99, batch * t * d).astype(np.float32)
        b = rs.standard_normal(batch * t * d).astype(np.float32)
        ref = orc.scan_sequential(a, b, batch, t, d, 1)
        assert np.abs(gpu.scan_chunked(a, b, batch, t, d) - ref).max() < 1e-4
        assert np.abs(gpu.scan_sequential(a, b, batch, t, d) - ref).max() < 1e-5


def test_scan_linearity(gpu):
    # h is linear in b for fixed a: scan(a, b1 + b2) == scan(a, b1) + scan(a, b2).
    rs = np.random.default_rng(9)
    batch, t, d = 3, 3000, 17
    a = rs.uniform(0.5, 0.999, batch * t * d).astype(np.float32)
    b1 = rs.standard_normal(batch * t * d).astype(np.float32)
    b2 = rs.standard_normal(batch * t * d).astype(np.float32)
    for fn in (gpu.scan_sequential, gpu.scan_chunked):
        lhs = fn(a, b1 + b2, batch, t, d)
        rhs = fn(a, b1, batch, t, d) + fn(a, b2, batch, t, d)
        assert np.abs(lhs - rhs).max() < 1e-4


def test_scan_empty_is_a_no_op(gpu):
    assert gpu.scan_chunked(np.zeros(0, np.float32), np.zeros(0, np.float32), 0, 5, 3).size == 0


# ---------------------------------------------------------------- sampler
def test_zero_nucleus_known_answer(gpu, orc):
    cfg = gpu.SampleCfg(temperature=1.0, top_k=0, top_p=0.0, rep_penalty=1.0, rep_window=0, greedy=False)
    logits = np.array([np.nan, np.inf, np.inf, -2.0], dtype=np.float32)
    rng = gpu.rng_state(7)
    assert gpu.sample_token(logits, cfg, [], rng) == 1
    # The mutated row is the softmax of the tied infinities (tensor.rs:373-375).
    assert logits.tolist() == [0.0, 0.5, 0.5, 0.0]
    # One f32_unit draw consumed, exactly as the reference's Rng.
    r = orc.Rng(7)
    r.f32_unit()
    assert [int(v) for v in rng] == r.s


def test_greedy_is_deterministic_and_in_range(gpu):
    # tests/engine.rs:153-173
    base = np.array([(i % 7) - 3 for i in range(64)], dtype=np.float32)
    rng = gpu.rng_state(21)
    g = gpu.SampleCfg(temperature=1.0, top_k=0, top_p=1.0, rep_penalty=1.0, rep_window=0, greedy=True)
    assert gpu.sample_token(base.copy(), g, [], rng) == gpu.sample_token(base.copy(), g, [], rng) == 6
    s = gpu.SampleCfg(temperature=0.8, top_k=5, top_p=0.9, rep_penalty=1.2, rep_window=8, greedy=False)
    for _ in range(50):
        assert 0 <= gpu.sample_token(base.copy(), s, [1, 1, 2, 3], rng) < 64


CFGS = [
    dict(temperature=0.8, top_k=0, top_p=0.95, rep_penalty=1.0, rep_window=0, greedy=False),
    dict(temperature=0.9, top_k=40, top_p=0.95, rep_penalty=1.1, rep_window=64, greedy=False),
    dict(temperature=1e-6, top_k=0, top_p=1.0, rep_penalty=1.0, rep_window=0, greedy=False),
    dict(temperature=2.0, top_k=3, top_p=0.5, rep_penalty=1.3, rep_window=4, greedy=False),
    dict(temperature=0.9, top_k=40, top_p=0.95, rep_penalty=1.1, rep_window=64, greedy=True),
]


@pytest.mark.parametrize("ci", range(len(CFGS)))
def test_teacher_forced_sampling_matches_oracle(gpu, orc, ci):
    """Token equality except where the oracle's draw lands within 1e-5 of a
    CDF edge or the nucleus cut is within 1e-6 of a rank boundary; the rng
    state must be bit-identical after every draw."""
    cfgd = CFGS[ci]
    V = 1024
    rs = np.random.default_rng(100 + ci)
    seed = 3000 + ci
    grng = gpu.rng_state(seed)
    orng = orc.Rng(seed)
    mismatches = 0
    for it in range(60):
        logits = (rs.standard_normal(V) * rs.uniform(0.1, 3.0)).astype(np.float32)
        hist = rs.integers(0, V, size=rs.integers(0, 80)).astype(np.uint32)
        hist[: len(hist) // 3] = hist[-1] if len(hist) else 0  # repeats
        a, b = logits.copy(), logits.copy()
        tok_g = gpu.sample_token(a, gpu.SampleCfg(**cfgd), hist, grng)
        tok_o, info = orc.sample_token(b, orc.SampleCfg(**cfgd), hist, orng, info=True)
        assert [int(v) for v in grng] == orng.s, it
        if tok_g != tok_o:
            mismatches += 1
            assert info.cdf_margin < 1e-5 or info.cut_margin < 1e-6 or info.top2_margin < 1e-6, it
        if not cfgd["greedy"]:
            assert np.abs(a - b).max() < 1e-6  # probabilities after softmax
    assert mismatches <= 2


def test_decoder_sample_batched_rows(gpu, orc):
    kw = dict(vocab=1024, d_model=32, n_layer=1, expand=1, conv_k=4, mlp_mult=3, eps=1e-5, tau_max=128.0)
    om = orc.Model(orc.LmConfig(**kw), seed=0)
    gm = gpu.Model.new(gpu.LmConfig(**kw), 0)
    S = 16
    dec = gpu.Decoder(gm, S)
    toks = np.arange(S, dtype=np.uint32) * 7
    lg = dec.step(toks).copy()
    cfg = dict(temperature=0.8, top_k=0, top_p=0.95, rep_penalty=1.0, rep_window=0, greedy=False)
    rng = np.stack([gpu.rng_state(3000 + s) for s in range(S)])
    out = dec.sample(gpu.SampleCfg(**cfg), rng)
    for s in range(S):
        r = orc.Rng(3000 + s)
        tok, info = orc.sample_token(lg[s].copy(), orc.SampleCfg(**cfg), [], r, info=True)
        assert [int(v) for v in rng[s]] == r.s
        assert out[s] == tok or info.cdf_margin < 1e-5 or info.cut_margin < 1e-6


@pytest.mark.parametrize("chunked", [False, True])
def test_scan_adjoint_matches_oracle(gpu, orc, chunked):
    # The awkward-shape table of scan.rs:269-288 plus blocks crossing 256.
    for batch, t, d in [(1, 1, 1), (3, 7, 5), (2, 129, 3), (5, 64, 1), (1, 1024, 9), (2, 1000, 4), (1, 777, 33)]:
        n = batch * t * d
        rng = orc.Rng(batch * 1000 + t)
        a = np.array([rng.f32_unit() * np.float32(0.98) + np.float32(0.01) for _ in range(n)], dtype=np.float32)
        g = np.array([rng.normal() for _ in range(n)], dtype=np.float32)
        ref = orc.scan_adjoint(a, g, batch, t, d)
        got = gpu.scan_adjoint(a, g, batch, t, d, chunked=chunked)
        assert np.abs(got - ref).max() < 1e-4, (batch, t, d, chunked)


def test_scan_adjoint_linearity_at_size(gpu):
    # c is linear in g: c(g1 + g2) = c(g1) + c(g2) (to f32 rounding), and the
    # two forms agree, on a C5-sized channel count over a long sequence.
    batch, t, d = 2, 4096, 768
    r = np.random.default_rng(3)
    a = (r.random(batch * t * d, dtype=np.float32) * 0.98 + 0.01).astype(np.float32)
    g1 = r.standard_normal(batch * t * d, dtype=np.float32)
    g2 = r.standard_normal(batch * t * d, dtype=np.float32)
    c1 = gpu.scan_adjoint(a, g1, batch, t, d, chunked=True)
    c2 = gpu.scan_adjoint(a, g2, batch, t, d, chunked=True)
    c12 = gpu.scan_adjoint(a, g1 + g2, batch, t, d, chunked=True)
    scale = np.abs(c12).max()
    assert np.abs(c12 - (c1 + c2)).max() <= 1e-5 * scale
    cs = gpu.scan_adjoint(a, g1, batch, t, d, chunked=False)
    assert np.abs(cs - c1).max() <= 1e-4 * np.abs(cs).max()


@pytest.mark.parametrize("adjoint", [False, True])
def test_one_pass_scan_block_edges(gpu, orc, adjoint):
    """The one-pass chunked scan (time blocks of 128 steps of 32 channels,
    carries by look-back) on shapes that cross every edge it has: lengths
    around a block (127, 128, 129), many blocks (4097), channel counts that
    leave a partial lane group (16, 33, 100), against the oracle's sequential
    scan (tolerance 1e-4, scan.rs:286) and against the three-pass form of the
    no-allocation entry point."""
    rs = np.random.default_rng(17 + int(adjoint))
    for batch, t, d in [(1, 1, 16), (2, 127, 33), (3, 128, 32), (1, 129, 100), (2, 4097, 48), (1, 300, 768)]:
        n = batch * t * d
        a = rs.uniform(0.01, 0.99, n).astype(np.float32)
        b = rs.standard_normal(n).astype(np.float32)
        if adjoint:
            ref = orc.scan_adjoint(a, b, batch, t, d)
            got = gpu.scan_adjoint(a, b, batch, t, d, chunked=True)
        else:
            ref = orc.scan_sequential(a, b, batch, t, d, 1)
            got = gpu.scan_chunked(a, b, batch, t, d)
        assert np.abs(got - ref).max() < 1e-4, (batch, t, d)


def test_one_pass_scan_slow_decay_long_rows(gpu, orc):
    # Decays near 1 carry the state across every block of a 20000-step row,
    # so each block's entering state depends on all its predecessors.
    rs = np.random.default_rng(29)
    batch, t, d = 2, 20000, 32
    n = batch * t * d
    a = rs.uniform(0.995, 0.9999, n).astype(np.float32)
    b = (rs.standard_normal(n) * 0.01).astype(np.float32)
    ref = orc.scan_sequential(a, b, batch, t, d, 1)
    got = gpu.scan_chunked(a, b, batch, t, d)
    assert np.abs(got - ref).max() < 1e-4 * max(1.0, float(np.abs(ref).max()))
