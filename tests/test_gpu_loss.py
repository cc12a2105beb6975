"""Lm::loss on the GPU (nk_model_loss: the batched forward of model.rs:209-226
through the prefill kernels, final norm and tied logits for every position,
softmax_ce of autograd.rs:579-624) against the oracle."""

import numpy as np
import pytest

from conftest import c1_cfg, same_model, tiny_cfg

pytestmark = pytest.mark.gpu


def _seq(orc, n, vocab, seed):
    r = orc.Rng(seed)
    return np.array([r.below(vocab) for _ in range(n)], dtype=np.uint32)


@pytest.mark.parametrize("batch,t", [(1, 1), (1, 9), (3, 17), (5, 40)])
def test_loss_and_logits_match_oracle(gpu, orc, batch, t):
    kw = c1_cfg(dict)
    om, gm = same_model(orc, gpu, kw, seed=0)
    ids = _seq(orc, batch * t, kw["vocab"], 100 + t)
    tg = np.roll(ids, -1)
    tg[::7] = 0xFFFFFFFF  # ignored positions
    ref_loss, ref_lg = om.loss(ids, tg, batch, t, want_logits=True)
    loss, lg = gm.loss(ids, tg, batch, t, want_logits=True)
    assert np.abs(lg - ref_lg).max() <= 1e-3
    assert abs(loss - ref_loss) <= 1e-4 * max(1.0, abs(ref_loss))


def test_loss_tensor_core_rows(gpu, orc):
    # 8 sequences x 64 positions = 512 rows: every projection and the logits
    # run on the tcgen05 engine.
    kw = dict(vocab=512, d_model=256, n_layer=2, expand=1, conv_k=4, mlp_mult=3, eps=1e-5, tau_max=128.0)
    om, gm = same_model(orc, gpu, kw, seed=4)
    batch, t = 8, 64
    ids = _seq(orc, batch * t, kw["vocab"], 5)
    tg = _seq(orc, batch * t, kw["vocab"], 6)
    ref = om.loss(ids, tg, batch, t)
    got = gm.loss(ids, tg, batch, t)
    assert abs(got - ref) <= 1e-4 * max(1.0, abs(ref))


def test_loss_edge_cases(gpu, orc):
    kw = tiny_cfg(dict, 19)
    om, gm = same_model(orc, gpu, kw, seed=2)
    ids = _seq(orc, 12, 19, 3)
    # every target ignored: the mean over no rows is 0 (denominator 1)
    assert gm.loss(ids, np.full(12, 0xFFFFFFFF, np.uint32), 2, 6) == 0.0
    with pytest.raises(gpu.NoeticError) as e:
        gm.loss(ids, np.full(12, 19, np.uint32), 2, 6)
    assert e.value.status == gpu.NK_ERR_INVALID
    bad = ids.copy()
    bad[5] = 19
    with pytest.raises(gpu.NoeticError):
        gm.loss(bad, ids, 2, 6)
    # the loss leaves decoders alone: a decoder mid-stream continues unchanged
    dec = gpu.Decoder(gm, 2)
    dec.step([1, 2])
    before = dec.get_state()
    gm.loss(ids, ids, 2, 6)
    after = dec.get_state()
    assert np.array_equal(before[0], after[0]) and np.array_equal(before[1], after[1])
