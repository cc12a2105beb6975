"""The tcgen05 3xTF32 projection engine against the f32 CUDA-core engine and
the oracle.  3xTF32 keeps ~22 mantissa bits per product, so the two engines
agree to f32 rounding (logits 1e-4, state 1e-5 relative) and both stay within
the oracle tolerances (logits 1e-3, state 1e-4)."""

import numpy as np
import pytest

from conftest import same_model, state_rel_err

pytestmark = pytest.mark.gpu

# Every projection of this model is tensor-core eligible at >= 128 streams:
# N in {768, 256, 1536, 256, 512}, K in {256, 768}.
WIDE = dict(vocab=512, d_model=256, n_layer=2, expand=1, conv_k=4, mlp_mult=3, eps=1e-5, tau_max=128.0)


def _ids(S, T, V, base):
    from noetic_b200.prompts import uniform_prompts

    return uniform_prompts(S, T, V, base)


# tensor-core tiles 128 / 256 columns wide on one SM; 256 x 256 on a CTA pair
@pytest.mark.parametrize("tile_bits", [16, 32, 128])
def test_tensor_core_engine_matches_f32_engine(gpu, orc, tile_bits):
    om, gm = same_model(orc, gpu, WIDE, seed=1)
    S, T = 384, 4
    ids = _ids(S, T, WIDE["vocab"], 10)
    tc, f32 = gpu.Decoder(gm, S), gpu.Decoder(gm, S)
    tc.set_engine(tile_bits)
    f32.set_engine(1)
    tc.profile_begin()
    for t in range(T):
        a = tc.step(ids[:, t]).copy()
        b = f32.step(ids[:, t])
        assert np.abs(a - b).max() <= 1e-4, t
    prof = tc.profile_end()
    assert prof["tensor_core"], "the tensor-core engine did not run"
    sa, ha = tc.get_state()
    sb, hb = f32.get_state()
    assert np.array_equal(ha, hb)
    assert state_rel_err(sa, sb) <= 1e-5
    for s in [0, 191, 383]:
        od = orc.Decoder(om)
        for t in range(T):
            ref = od.step(ids[s, t])
        assert np.abs(a[s] - ref).max() <= 1e-3


def test_tensor_core_prefill_matches_stepping(gpu, orc):
    om, gm = same_model(orc, gpu, WIDE, seed=3)
    S, T = 64, 40  # 2560 prompt rows per projection
    ids = _ids(S, T, WIDE["vocab"], 77)
    lens = np.full(S, T, np.uint32)
    lens[5] = 17
    dec = gpu.Decoder(gm, S)
    dec.profile_begin()
    last = dec.prefill(ids, lens).copy()
    assert dec.profile_end()["tensor_core"]
    st, heads = dec.get_state()
    k, E = WIDE["conv_k"], WIDE["d_model"]
    for s in [0, 5, 63]:
        od = orc.Decoder(om)
        for t in ids[s, : lens[s]]:
            ref = od.step(t)
        ost, oh = od.get_state()
        assert heads[s] == oh
        assert state_rel_err(st[s][:, k * E:], ost[:, k * E:]) <= 1e-4
        assert np.abs(last[s] - ref).max() <= 1e-3


def test_headline_model_stream_subset(gpu, orc):
    """The d=1024 / 24-layer / vocab-32768 model (seed 2) at 512 streams:
    scan prefill of 8 prompt tokens, then 2 greedy steps; 3 streams checked
    against the oracle."""
    kw = dict(vocab=32768, d_model=1024, n_layer=24, expand=1, conv_k=4, mlp_mult=3, eps=1e-5, tau_max=128.0)
    om, gm = same_model(orc, gpu, kw, seed=2)
    om.set_threads(8)
    S, T = 512, 8
    ids = _ids(S, T, kw["vocab"], 5000)
    dec = gpu.Decoder(gm, S)
    dec.profile_begin()
    last = dec.prefill(ids).copy()
    tok = np.argmax(last, axis=1).astype(np.uint32)
    lg = dec.step(tok).copy()
    assert dec.profile_end()["tensor_core"]
    st, _ = dec.get_state()
    k, E = 4, 1024
    for s in [0, 300, 511]:
        od = orc.Decoder(om)
        for t in ids[s]:
            ref = od.step(t).copy()
        assert np.abs(last[s] - ref).max() <= 1e-3, s
        ref2 = od.step(int(tok[s]))
        assert np.abs(lg[s] - ref2).max() <= 1e-3, s
        ost, _ = od.get_state()
        for layer in [0, 11, 23]:
            assert state_rel_err(st[s, layer, k * E:], ost[layer, k * E:]) <= 1e-4, (s, layer)


@pytest.mark.parametrize("engine", [0, 128])  # default tiles / the CTA-pair kernel
def test_fused_argmax_epilogue_matches_materialised_logits(gpu, orc, engine):
    """Greedy steps through the logits projection's argmax epilogue (no
    logits stored) pick the same tokens as argmax over stored logits, except
    where the two best logits are within 1e-4."""
    _, gm = same_model(orc, gpu, WIDE, seed=5)
    S = 256
    ids = _ids(S, 3, WIDE["vocab"], 31)
    fused, plain = gpu.Decoder(gm, S), gpu.Decoder(gm, S)
    fused.set_engine(engine)
    plain.set_engine(engine)
    for t in range(3):
        tok = fused.step_greedy(ids[:, t])
        lg = plain.step(ids[:, t])
        ref = np.argmax(lg, axis=1)
        top2 = np.sort(lg, axis=1)[:, -2:]
        clear = (top2[:, 1] - top2[:, 0]) > 1e-4
        assert np.array_equal(tok[clear], ref[clear]), t
        assert clear.mean() > 0.9
    st_a, _ = fused.get_state()
    st_b, _ = plain.get_state()
    assert state_rel_err(st_a, st_b) <= 1e-6


def test_hidden_width_off_the_interleave_grid(gpu, orc):
    """H = 600 is not a multiple of 32: the up projection keeps its row order
    and SwiGLU runs as a row kernel instead of in the projection epilogue."""
    kw = dict(vocab=512, d_model=200, n_layer=2, expand=1, conv_k=4, mlp_mult=3, eps=1e-5, tau_max=128.0)
    om, gm = same_model(orc, gpu, kw, seed=6)
    S, T = 256, 3
    ids = _ids(S, T, kw["vocab"], 31)
    tc, f32 = gpu.Decoder(gm, S), gpu.Decoder(gm, S)
    f32.set_engine(1)
    tc.profile_begin()
    for t in range(T):
        a = tc.step(ids[:, t]).copy()
        b = f32.step(ids[:, t])
        assert np.abs(a - b).max() <= 1e-4, t
    assert tc.profile_end()["tensor_core"]
    sa, _ = tc.get_state()
    sb, _ = f32.get_state()
    assert state_rel_err(sa, sb) <= 1e-5
    od = orc.Decoder(om)
    for t in range(T):
        ref = od.step(ids[7, t])
    assert np.abs(a[7] - ref).max() <= 1e-3


@pytest.mark.parametrize("engine", [0, 128])
def test_large_batch_tilings(gpu, orc, engine):
    """16384 streams of a d=1024 model.  Engine 0: stream-K over 148 SMs
    (out_proj: 512 tiles x 64 K-blocks, 222 K-blocks per CTA, so most CTAs
    finish one tile cut at a range boundary).  Engine 128: every projection
    runs on the CTA-pair kernel (256 x 256 tiles).  Every stream, the last
    rows and columns included, equals the f32 engine."""
    kw = dict(vocab=2048, d_model=1024, n_layer=1, expand=1, conv_k=4, mlp_mult=3, eps=1e-5, tau_max=128.0)
    om, gm = same_model(orc, gpu, kw, seed=8)
    S = 16384
    ids = _ids(S, 2, kw["vocab"], 900)
    tc, f32 = gpu.Decoder(gm, S), gpu.Decoder(gm, S)
    tc.set_engine(engine)
    f32.set_engine(1)
    for t in range(2):
        a = tc.step(ids[:, t]).copy()
        b = f32.step(ids[:, t])
        assert np.abs(a - b).max() <= 1e-4, t
    sa, _ = tc.get_state()
    sb, _ = f32.get_state()
    assert state_rel_err(sa, sb) <= 1e-5
    for s in [0, 16383]:
        od = orc.Decoder(om)
        for t in range(2):
            ref = od.step(ids[s, t])
        assert np.abs(a[s] - ref).max() <= 1e-3, s


def test_stream_k_small_grids(gpu, orc):
    """2048 streams (one GPU's share of 16384 on eight): out_proj has 64
    tiles x 64 K-blocks for 148 SMs, 28 K-blocks per CTA, so a tile spans up
    to three CTAs and its first CTA adds the others' partial sums in a fixed
    order; the result equals the f32 engine's, and two runs are
    bit-identical."""
    kw = dict(vocab=2048, d_model=1024, n_layer=2, expand=1, conv_k=4, mlp_mult=3, eps=1e-5, tau_max=128.0)
    om, gm = same_model(orc, gpu, kw, seed=9)
    S = 2048
    ids = _ids(S, 3, kw["vocab"], 4100)
    tc, tc2, f32 = gpu.Decoder(gm, S), gpu.Decoder(gm, S), gpu.Decoder(gm, S)
    f32.set_engine(1)
    tc.profile_begin()
    for t in range(3):
        a = tc.step(ids[:, t]).copy()
        a2 = tc2.step(ids[:, t]).copy()
        b = f32.step(ids[:, t])
        assert np.array_equal(a, a2), t
        assert np.abs(a - b).max() <= 1e-4, t
    assert tc.profile_end()["tensor_core"]
    sa, _ = tc.get_state()
    sb, _ = f32.get_state()
    assert state_rel_err(sa, sb) <= 1e-5
    for s in [0, 2047]:
        od = orc.Decoder(om)
        for t in range(3):
            ref = od.step(ids[s, t])
        assert np.abs(a[s] - ref).max() <= 1e-3, s


@pytest.mark.parametrize("S", [9, 64, 127])
def test_fewer_streams_than_a_tile(gpu, orc, S):
    # 9..127 streams: one 128-row tile whose rows past S read zeros from the
    # tensor map and are masked in every epilogue (store, SwiGLU, argmax).
    om, gm = same_model(orc, gpu, WIDE, seed=2)
    T = 3
    ids = _ids(S, T, WIDE["vocab"], 40)
    tc, f32 = gpu.Decoder(gm, S), gpu.Decoder(gm, S)
    f32.set_engine(1)
    tc.profile_begin()
    for t in range(T):
        a = tc.step(ids[:, t]).copy()
        b = f32.step(ids[:, t])
        assert np.abs(a - b).max() <= 1e-4, t
    assert tc.profile_end()["tensor_core"]
    sa, ha = tc.get_state()
    sb, hb = f32.get_state()
    assert np.array_equal(ha, hb) and state_rel_err(sa, sb) <= 1e-5
    od = orc.Decoder(om)
    for t in range(T):
        ref = od.step(ids[S - 1, t])
    assert np.abs(a[S - 1] - ref).max() <= 1e-3
    # Greedy steps (the argmax epilogue) agree with the f32 engine's choice.
    toks = ids[:, -1].copy()
    ga, gb = tc.step_greedy(toks).copy(), f32.step_greedy(toks).copy()
    assert (ga == gb).mean() > 0.95


C5_WIDTHS = dict(vocab=16384, d_model=768, n_layer=2, expand=1, conv_k=4, mlp_mult=3, eps=1e-5, tau_max=128.0)


@pytest.mark.parametrize("S", [64, 127, 512])
def test_long_prompt_model_widths_at_serving_batches(gpu, orc, S):
    """The long-prompt model's widths (d 768, H 2304, V 16384) at 64 / 127 /
    512 streams.  Up to 128 streams every projection has one row of tiles and
    is split along K over the SMs (pieces summed in a fixed order by a
    reduction kernel); the result matches the f32 engine and the oracle, and
    two decoders agree bit for bit."""
    om, gm = same_model(orc, gpu, C5_WIDTHS, seed=3)
    T = 3
    ids = _ids(S, T, C5_WIDTHS["vocab"], 6000)
    tc, tc2, f32 = gpu.Decoder(gm, S), gpu.Decoder(gm, S), gpu.Decoder(gm, S)
    f32.set_engine(1)
    tc.profile_begin()
    for t in range(T):
        a = tc.step(ids[:, t]).copy()
        a2 = tc2.step(ids[:, t]).copy()
        b = f32.step(ids[:, t])
        assert np.array_equal(a, a2), t
        assert np.abs(a - b).max() <= 1e-4, t
    assert tc.profile_end()["tensor_core"]
    sa, ha = tc.get_state()
    sb, hb = f32.get_state()
    assert np.array_equal(ha, hb) and state_rel_err(sa, sb) <= 1e-5
    for s in [0, S - 1]:
        od = orc.Decoder(om)
        for t in range(T):
            ref = od.step(ids[s, t])
        assert np.abs(a[s] - ref).max() <= 1e-3, s
    toks = ids[:, -1].copy()
    ga, gb = tc.step_greedy(toks).copy(), f32.step_greedy(toks).copy()
    assert (ga == gb).mean() > 0.95


@pytest.mark.parametrize("S", [64, 384, 2048])
def test_folded_rmsnorm_matches_standalone_norms(gpu, orc, S):
    """RMSNorm folded into the projections (engine bit 14; the default below
    384 streams at widths >= 512) against the stand-alone RMSNorm kernels
    (engine bit 18 below 384 streams, the default above) and the oracle, at
    split-K (64, 384, 2048 streams) tilings, greedy steps included."""
    kw = dict(vocab=2048, d_model=512, n_layer=3, expand=1, conv_k=4, mlp_mult=3, eps=1e-5, tau_max=128.0)
    om, gm = same_model(orc, gpu, kw, seed=21)
    T = 3
    ids = _ids(S, T, kw["vocab"], 900)
    fold, plain = gpu.Decoder(gm, S), gpu.Decoder(gm, S)
    fold.set_engine(16384)
    plain.set_engine(262144)  # below 384 streams the default folds too
    for t in range(T):
        a = fold.step(ids[:, t]).copy()
        b = plain.step(ids[:, t])
        assert np.abs(a - b).max() <= 1e-4, t
    sa, _ = fold.get_state()
    sb, _ = plain.get_state()
    assert state_rel_err(sa, sb) <= 1e-5
    for s in [0, S - 1]:
        od = orc.Decoder(om)
        for t in range(T):
            ref = od.step(ids[s, t])
        assert np.abs(a[s] - ref).max() <= 1e-3, s
    toks = ids[:, -1].copy()
    ga, gb = fold.step_greedy(toks).copy(), plain.step_greedy(toks).copy()
    assert (ga == gb).mean() > 0.95


@pytest.mark.parametrize("S", [16, 64, 512])
def test_split_k_reductions_take_over_norm_and_recurrence(gpu, orc, S):
    """When the projections are split along K (up to 512 streams here), the
    input projection's reduction also runs the recurrent branch and, from 384
    streams on, the residual projections' reductions the next RMSNorm.  Both repeat the
    separate kernels' operations (ssm_decode, rmsnorm_rows), so the steps
    equal those with the separate kernels (engine bits 16, 17) -- logits, greedy
    tokens and every layer's state -- and the oracle within tolerance."""
    kw = dict(vocab=4096, d_model=768, n_layer=3, expand=1, conv_k=4, mlp_mult=3, eps=1e-5, tau_max=128.0)
    om, gm = same_model(orc, gpu, kw, seed=23)
    T = 3
    ids = _ids(S, T, kw["vocab"], 910)
    fused, plain = gpu.Decoder(gm, S), gpu.Decoder(gm, S)
    # stand-alone norms (below 384 streams the default folds them instead)
    fused.set_engine(262144)
    plain.set_engine(262144 | 65536 | 131072)
    n0, p0 = fused.launch_count(), plain.launch_count()
    for t in range(T):
        a = fused.step(ids[:, t]).copy()
        b = plain.step(ids[:, t])
        assert np.abs(a - b).max() <= 1e-6 * max(1.0, float(np.abs(b).max())), t
    # Per layer and step the ssm step's launch is saved, from 384 streams on
    # also the two RMSNorms' (below that the separate norms are faster).
    saved = 3 * (3 if S >= 384 else 1) * T
    assert (fused.launch_count() - n0) + saved == plain.launch_count() - p0
    sa, ha = fused.get_state()
    sb, hb = plain.get_state()
    assert np.array_equal(ha, hb) and state_rel_err(sa, sb) <= 1e-6
    for s in [0, S - 1]:
        od = orc.Decoder(om)
        for t in range(T):
            ref = od.step(ids[s, t])
        assert np.abs(a[s] - ref).max() <= 1e-3, s
    toks = ids[:, -1].copy()
    assert np.array_equal(fused.step_greedy(toks), plain.step_greedy(toks))
