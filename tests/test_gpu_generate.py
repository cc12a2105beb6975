"""cli.rs:generate (cli.rs:470-518) for many streams on the GPU, checked
step by step against the oracle under teacher forcing: the oracle follows the
GPU's tokens and at every step makes its own decision; decisions must agree
except at flagged near-ties, and every stream's rng state must be
bit-identical at the end."""

import numpy as np
import pytest

from conftest import c1_cfg, same_model

pytestmark = pytest.mark.gpu


def _teacher_forced(orc, om, prompt, gpu_tokens, cfgd, seed):
    """Replays generate() on the oracle along gpu_tokens; returns
    (#undecidable mismatches, #hard mismatches, final rng)."""
    cfg = orc.SampleCfg(**cfgd)
    rng = orc.Rng(seed)
    dec = orc.Decoder(om)
    ids = list(prompt) if len(prompt) else [10]
    for t in ids:
        lg = dec.step(t).copy()
    W = cfgd["rep_window"]
    hist = ids[max(0, len(ids) - W):] if W > 0 else []
    soft = hard = 0
    n = len(gpu_tokens)
    for g, gt in enumerate(gpu_tokens):
        tok, info = orc.sample_token(lg, cfg, hist, rng, info=True)
        if tok != gt:
            near = (info.cdf_margin < 1e-5 or info.cut_margin < 1e-6 or info.order_margin < 2e-4
                    or (cfgd["greedy"] and info.top2_margin < 2e-3))
            soft += near
            hard += not near
        if W > 0:
            hist = (hist + [int(gt)])[-W:]
        if g + 1 < n:
            lg = dec.step(int(gt)).copy()
    return soft, hard, rng


@pytest.mark.parametrize("cfgd", [
    dict(temperature=0.8, top_k=0, top_p=0.95, rep_penalty=1.0, rep_window=0, greedy=False),
    dict(temperature=0.9, top_k=40, top_p=0.95, rep_penalty=1.1, rep_window=64, greedy=False),
    dict(temperature=1.0, top_k=0, top_p=1.0, rep_penalty=1.1, rep_window=64, greedy=True),
])
def test_generate_matches_oracle_teacher_forced(gpu, orc, cfgd):
    kw = c1_cfg(dict)
    om, gm = same_model(orc, gpu, kw, seed=0)
    S, T, N = 6, 32, 24
    lens = np.array([32, 32, 5, 1, 0, 17], dtype=np.uint32)
    ids = np.zeros((S, T), dtype=np.uint32)
    for s in range(S):
        r = orc.Rng(2000 + s)
        ids[s, : lens[s]] = [r.below(1024) for _ in range(lens[s])]
    rng = np.stack([gpu.rng_state(3000 + s) for s in range(S)])
    dec = gpu.Decoder(gm, S)
    out = dec.generate(ids, lens, N, gpu.SampleCfg(**cfgd), rng)
    assert out.shape == (S, N) and out.max() < 1024
    total_soft = 0
    for s in range(S):
        soft, hard, r = _teacher_forced(orc, om, ids[s, : lens[s]], out[s], cfgd, 3000 + s)
        assert hard == 0, s
        total_soft += soft
        if not cfgd["greedy"]:
            assert [int(v) for v in rng[s]] == r.s, s
    assert total_soft <= 2


def test_greedy_generate_is_reproducible(gpu, orc):
    kw = c1_cfg(dict)
    _, gm = same_model(orc, gpu, kw, seed=0)
    cfg = gpu.SampleCfg(temperature=1.0, top_k=0, top_p=1.0, rep_penalty=1.0, rep_window=0, greedy=True)
    ids = (np.arange(64, dtype=np.uint32) * 13 % 1024).reshape(4, 16)
    lens = np.full(4, 16, np.uint32)
    a = gpu.Decoder(gm, 4).generate(ids, lens, 20, cfg, np.zeros((4, 4), np.uint64))
    b = gpu.Decoder(gm, 4).generate(ids, lens, 20, cfg, np.zeros((4, 4), np.uint64))
    assert np.array_equal(a, b)


def test_checkpoint_reload_reproduces_logits(gpu, orc, tmp_path):
    # tests/engine.rs:29-85 (the reload half): an oracle-written checkpoint
    # loads on the GPU and streams the oracle's logits; a GPU-written copy
    # reloads to identical logits.
    kw = dict(vocab=40, d_model=24, n_layer=2, expand=2, conv_k=3, mlp_mult=2, eps=1e-5, tau_max=16.0)
    om = orc.Model(orc.LmConfig(**kw), seed=4)
    p = str(tmp_path / "m.ckpt")
    om.save(p)
    gm = gpu.Model.load(p, device=0)
    ids = [(i * 5 + 1) % 40 for i in range(6)]
    d1, od = gpu.Decoder(gm, 1), orc.Decoder(om)
    first = []
    for t in ids:
        row = d1.step([t])[0].copy()
        first.append(row)
        assert np.abs(row - od.step(t)).max() <= 1e-3
    q = str(tmp_path / "g.ckpt")
    gm.save(q)
    gm2 = gpu.Model.load(q, device=0)
    d2 = gpu.Decoder(gm2, 1)
    for i, t in enumerate(ids):
        assert np.abs(d2.step([t])[0] - first[i]).max() < 1e-6


@pytest.mark.parametrize("cfgd", [
    dict(temperature=0.9, top_k=40, top_p=0.95, rep_penalty=1.1, rep_window=64, greedy=False),  # SampleCfg::default_cfg
    dict(temperature=0.8, top_k=0, top_p=0.95, rep_penalty=1.0, rep_window=0, greedy=False),
])
def test_generate_samples_at_the_headline_vocabulary(gpu, orc, cfgd):
    """noetic gen's default (sampled) path at V = 32768, teacher-forced
    against the oracle with the rng state bit-exact per stream."""
    kw = dict(vocab=32768, d_model=64, n_layer=2, expand=1, conv_k=4, mlp_mult=3, eps=1e-5, tau_max=128.0)
    om, gm = same_model(orc, gpu, kw, seed=2)
    S, T, N = 5, 12, 16
    lens = np.array([12, 3, 0, 12, 7], dtype=np.uint32)
    ids = np.zeros((S, T), dtype=np.uint32)
    for s in range(S):
        r = orc.Rng(5000 + s)
        ids[s, : lens[s]] = [r.below(32768) for _ in range(lens[s])]
    rng = np.stack([gpu.rng_state(3000 + s) for s in range(S)])
    out = gpu.Decoder(gm, S).generate(ids, lens, N, gpu.SampleCfg(**cfgd), rng)
    assert out.shape == (S, N) and out.max() < 32768
    total_soft = 0
    for s in range(S):
        soft, hard, r = _teacher_forced(orc, om, ids[s, : lens[s]], out[s], cfgd, 3000 + s)
        assert hard == 0, s
        total_soft += soft
        assert [int(v) for v in rng[s]] == r.s, s
    assert total_soft <= 1


@pytest.mark.parametrize("cfgd", [
    dict(temperature=0.9, top_k=40, top_p=0.95, rep_penalty=1.1, rep_window=64, greedy=False),
    dict(temperature=0.8, top_k=0, top_p=0.95, rep_penalty=1.0, rep_window=0, greedy=False),
    dict(temperature=1.0, top_k=0, top_p=1.0, rep_penalty=1.0, rep_window=0, greedy=True),
])
def test_fused_logits_sampling_equals_the_plain_step_and_sampler(gpu, orc, cfgd):
    """The logits projection's sampling epilogue (penalty bitmap, temperature,
    row maxima) and the greedy argmax epilogue give bit-identical tokens and
    rng states to storing the logits and running the stand-alone sampler
    (engine bit 11), on the same whole-tile projections (engine bit 8)."""
    kw = dict(vocab=32768, d_model=64, n_layer=2, expand=1, conv_k=4, mlp_mult=3, eps=1e-5, tau_max=128.0)
    _, gm = same_model(orc, gpu, kw, seed=3)
    S, T, N = 24, 9, 20
    lens = np.full(S, T, np.uint32)
    lens[3] = 2
    ids = (np.arange(S * T, dtype=np.uint32).reshape(S, T) * 2654435761 % 32768).astype(np.uint32)
    outs, rngs = [], []
    for engine in (256, 256 | 2048):
        dec = gpu.Decoder(gm, S)
        dec.set_engine(engine)
        rng = np.stack([gpu.rng_state(700 + s) for s in range(S)])
        outs.append(dec.generate(ids, lens, N, gpu.SampleCfg(**cfgd), rng))
        rngs.append(rng)
    assert np.array_equal(outs[0], outs[1])
    assert np.array_equal(rngs[0], rngs[1])
