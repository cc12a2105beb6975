"""The fused small-batch decode step (<= 8 streams: four kernels per layer,
L2 weight prefetch ahead of programmatic dependent launch, CUDA-graph replay
of greedy steps) against the oracle and against the unfused kernels."""

import numpy as np
import pytest

from conftest import c1_cfg, same_model, state_rel_err, tiny_cfg

pytestmark = pytest.mark.gpu

UNFUSED = 8  # engine bit: no fused small-batch step
SMALL = 1024  # engine bit: no persistent step kernel (the fused small-batch kernels)


@pytest.mark.parametrize("S", [1, 3, 8])
def test_small_batch_step_matches_oracle_and_unfused(gpu, orc, S):
    kw = c1_cfg(dict)
    om, gm = same_model(orc, gpu, kw, seed=0)
    from noetic_b200.prompts import uniform_prompts

    ids = uniform_prompts(S, 6, kw["vocab"], 40)
    fused, plain = gpu.Decoder(gm, S), gpu.Decoder(gm, S)
    fused.set_engine(SMALL)
    plain.set_engine(UNFUSED)
    ods = [orc.Decoder(om) for _ in range(S)]
    for t in range(6):
        a = fused.step(ids[:, t]).copy()
        b = plain.step(ids[:, t])
        assert np.abs(a - b).max() <= 1e-5
        for s in range(S):
            assert np.abs(a[s] - ods[s].step(ids[s, t])).max() <= 1e-3
    sa, ha = fused.get_state()
    sb, hb = plain.get_state()
    assert np.array_equal(ha, hb) and state_rel_err(sa, sb) <= 1e-5


def test_graph_replayed_greedy_steps_follow_the_oracle(gpu, orc):
    """Greedy steps replayed from the captured graph, teacher-forced with the
    oracle's tokens: identical choices wherever the top-2 margin > 1e-3."""
    kw = c1_cfg(dict)
    om, gm = same_model(orc, gpu, kw, seed=0)
    S = 2
    dec = gpu.Decoder(gm, S)
    dec.set_engine(SMALL)
    ods = [orc.Decoder(om) for _ in range(S)]
    toks = np.array([17, 900], dtype=np.uint32)
    checked = 0
    for step in range(24):
        nxt = dec.step_greedy(toks)
        for s in range(S):
            lg = ods[s].step(int(toks[s])).copy()
            top2 = np.sort(lg)[-2:]
            if top2[1] - top2[0] > 1e-3:
                assert int(nxt[s]) == orc.argmax(lg), (step, s)
                checked += 1
        toks = np.array([orc.argmax(ods[s].logits) for s in range(S)], dtype=np.uint32)
    assert checked >= 40
    assert dec.launch_count() > 0


def test_small_batch_awkward_shapes(gpu, orc):
    # Odd widths take the scalar loads; conv widths 1 and 7.
    for kw in [dict(vocab=29, d_model=5, n_layer=2, expand=3, conv_k=2, mlp_mult=1, eps=1e-5, tau_max=4.0),
               tiny_cfg(dict, 17, conv_k=1, n_layer=1), tiny_cfg(dict, 17, conv_k=7, n_layer=2)]:
        om, gm = same_model(orc, gpu, kw, seed=3)
        S = 3
        dec = gpu.Decoder(gm, S)
        dec.set_engine(SMALL)
        ods = [orc.Decoder(om) for _ in range(S)]
        for t in range(5):
            tok = np.array([(t * 7 + s) % kw["vocab"] for s in range(S)], dtype=np.uint32)
            lg = dec.step(tok)
            for s in range(S):
                assert np.abs(lg[s] - ods[s].step(int(tok[s]))).max() <= 1e-3
        st, hd = dec.get_state()
        for s in range(S):
            ost, oh = ods[s].get_state()
            assert hd[s] == oh and state_rel_err(st[s], ost) <= 1e-4
