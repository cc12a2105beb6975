"""Scan prefill on the GPU vs stepping the oracle through the prompt.

The reference's gen path prefills with one Decoder::step per prompt token
(cli.rs:478-480); the batched forward with the scan (model.rs:148-165) is
pinned equal to it by selftest.rs:273-299.  The GPU prefill must leave the
same LmState (conv ring, head, h) and the same last-position logits."""

import numpy as np
import pytest

from conftest import c1_cfg, same_model, state_rel_err, tiny_cfg

pytestmark = pytest.mark.gpu

LOGIT_TOL = 1e-3
STATE_TOL = 1e-4
SEQ, CHUNKED = 4, 2  # engine bits forcing the prefill scan variant


def _ragged(S, T, V, lens, seed):
    import oracle as O

    ids = np.zeros((S, T), dtype=np.uint32)
    for s in range(S):
        r = O.Rng(seed + s)
        ids[s, : lens[s]] = [r.below(V) for _ in range(lens[s])]
    return ids


def _check(dec, od_list, last, lens, kw, live_logits):
    k, E = kw["conv_k"], kw["d_model"] * kw["expand"]
    st, heads = dec.get_state()
    for s, od in enumerate(od_list):
        ost, oh = od.get_state()
        assert heads[s] == oh, s
        for layer in range(ost.shape[0]):
            assert state_rel_err(st[s, layer, k * E:], ost[layer, k * E:]) <= STATE_TOL, (s, layer)
            assert state_rel_err(st[s, layer, : k * E], ost[layer, : k * E]) <= STATE_TOL, (s, layer)
        if lens[s] > 0:
            assert np.abs(last[s] - live_logits[s]).max() <= LOGIT_TOL, s


@pytest.mark.parametrize("engine", [SEQ, CHUNKED])
def test_ragged_prefill_matches_stepping(gpu, orc, engine):
    kw = c1_cfg(dict)
    om, gm = same_model(orc, gpu, kw, seed=0)
    lens = [0, 1, 3, 17, 70, 200]
    S, T = len(lens), max(lens)
    ids = _ragged(S, T, kw["vocab"], lens, 1000)
    dec = gpu.Decoder(gm, S)
    dec.set_engine(engine)
    last = dec.prefill(ids, lens).copy()
    ods, live = [], []
    for s in range(S):
        od = orc.Decoder(om)
        lg = None
        for t in ids[s, : lens[s]]:
            lg = od.step(t).copy()
        ods.append(od)
        live.append(lg)
    _check(dec, ods, last, lens, kw, live)


@pytest.mark.parametrize("engine", [SEQ, CHUNKED])
def test_prefill_continues_from_a_stepped_state(gpu, orc, engine):
    kw = tiny_cfg(dict, 31, conv_k=4, n_layer=3)
    om, gm = same_model(orc, gpu, kw, seed=9)
    S = 3
    dec = gpu.Decoder(gm, S)
    dec.set_engine(engine)
    ods = [orc.Decoder(om) for _ in range(S)]
    for t in [4, 5]:
        dec.step([t] * S)
        for od in ods:
            od.step(t)
    lens = [1, 2, 130]
    ids = _ragged(S, 130, 31, lens, 40)
    last = dec.prefill(ids, lens).copy()
    live = []
    for s, od in enumerate(ods):
        lg = None
        for t in ids[s, : lens[s]]:
            lg = od.step(t).copy()
        live.append(lg)
    _check(dec, ods, last, lens, kw, live)
    # And decoding continues identically afterwards.
    nxt = dec.step([7, 8, 9])
    for s, od in enumerate(ods):
        assert np.abs(nxt[s] - od.step([7, 8, 9][s])).max() <= LOGIT_TOL


@pytest.mark.parametrize("conv_k", [1, 2, 7])
def test_prefill_awkward_conv_widths(gpu, orc, conv_k):
    kw = tiny_cfg(dict, 17, conv_k=conv_k, n_layer=2)
    om, gm = same_model(orc, gpu, kw, seed=20250816)
    lens = [1, conv_k, conv_k + 1, 9]
    S = len(lens)
    ids = _ragged(S, 9, 17, lens, 5)
    for engine in [SEQ, CHUNKED]:
        dec = gpu.Decoder(gm, S)
        dec.set_engine(engine)
        last = dec.prefill(ids, lens).copy()
        ods, live = [], []
        for s in range(S):
            od = orc.Decoder(om)
            lg = None
            for t in ids[s, : lens[s]]:
                lg = od.step(t).copy()
            ods.append(od)
            live.append(lg)
        _check(dec, ods, last, lens, kw, live)


def test_long_prompt_chunked_scan_matches_batched_oracle(gpu, orc):
    # A prompt much longer than the scan's time block, two streams: the
    # time-parallel scan path, checked against the oracle's batched forward.
    kw = tiny_cfg(dict, 23, conv_k=4, n_layer=2)
    om, gm = same_model(orc, gpu, kw, seed=6)
    S, T = 2, 1500
    ids = _ragged(S, T, 23, [T, T - 37], 900)
    lens = [T, T - 37]
    dec = gpu.Decoder(gm, S)
    dec.set_engine(CHUNKED)
    last = dec.prefill(ids, lens).copy()
    st, heads = dec.get_state()
    k, E = kw["conv_k"], kw["d_model"] * kw["expand"]
    for s in range(S):
        ost, oh, olast = om.prefill_state(ids[s, : lens[s]], 1, lens[s])
        assert heads[s] == oh[0]
        assert state_rel_err(st[s][:, k * E:], ost[0][:, k * E:]) <= STATE_TOL
        assert np.abs(last[s] - olast[0]).max() <= LOGIT_TOL


def test_prefill_rejects_bad_input(gpu, orc):
    kw = tiny_cfg(dict, 19)
    _, gm = same_model(orc, gpu, kw, seed=1)
    dec = gpu.Decoder(gm, 2)
    with pytest.raises(gpu.NoeticError):
        dec.prefill(np.array([[1, 2], [3, 19]], dtype=np.uint32))
    with pytest.raises(gpu.NoeticError):
        dec.prefill(np.array([[1, 2], [3, 4]], dtype=np.uint32), lens=[3, 1])


def test_long_prompt_prefill_at_full_length(gpu):
    """The long-prompt prefill shape (d768, 12 layers, vocab 16384, 32768-token
    prompts, stream s from Rng::new(6000 + s)): the time-chunked scan prefill
    leaves the state the sequential scan prefill leaves (scan.rs:286, 1e-4)
    and the state that stepping every token through the decoder leaves (the
    decoder is pinned to the oracle by the streaming tests), with the same
    last-position logits.  Size-independent checks at the full length, where
    the oracle would take hours."""
    import torch

    from noetic_b200.prompts import uniform_prompts

    kw = dict(vocab=16384, d_model=768, n_layer=12, expand=1, conv_k=4, mlp_mult=3, eps=1e-5, tau_max=128.0)
    gm = gpu.Model.new(gpu.LmConfig(**kw), 3)
    S, T = 2, 32768
    ids = uniform_prompts(S, T, kw["vocab"], 6000)
    a, b = gpu.Decoder(gm, S), gpu.Decoder(gm, S)
    a.set_engine(CHUNKED)
    b.set_engine(SEQ)
    la, lb = a.prefill(ids).copy(), b.prefill(ids).copy()
    # Stepping: the prompt columns already on the device, one step per token.
    c = gpu.Decoder(gm, S)
    cols = torch.from_numpy(np.ascontiguousarray(ids.T).astype(np.int32)).cuda()
    out = torch.empty(S, dtype=torch.int32, device="cuda")
    for t in range(T - 1):
        c.step_greedy_device(cols[t].data_ptr(), out.data_ptr())
    torch.cuda.synchronize()
    lc = c.step(ids[:, T - 1]).copy()
    sa, ha = a.get_state()
    sb, hb = b.get_state()
    sc, hc = c.get_state()
    assert np.array_equal(ha, hb) and np.array_equal(ha, hc)
    assert state_rel_err(sa, sb) <= STATE_TOL
    assert state_rel_err(sa, sc) <= STATE_TOL
    assert np.abs(la - lb).max() <= LOGIT_TOL and np.abs(la - lc).max() <= LOGIT_TOL


def test_prefill_then_decode_at_the_4096_stream_shape(gpu, orc):
    """d512 L8 V8192 (seed 1), 4096 streams x 512-token prompts (stream s from
    Rng::new(4000 + s)), the scan prefill then greedy steps: streams spread
    over the batch against the oracle's batched forward and its decoder,
    teacher-forced with the oracle's tokens."""
    from noetic_b200.prompts import uniform_prompts

    kw = dict(vocab=8192, d_model=512, n_layer=8, expand=1, conv_k=4, mlp_mult=3, eps=1e-5, tau_max=128.0)
    om, gm = same_model(orc, gpu, kw, seed=1)
    S, T = 4096, 512
    ids = uniform_prompts(S, T, kw["vocab"], 4000)
    dec = gpu.Decoder(gm, S)
    last = dec.prefill(ids).copy()
    st, heads = dec.get_state()
    probe = [0, 1365, 2730, 4095]
    ods = []
    for s in probe:
        ost, oh, olast = om.prefill_state(ids[s], 1, T)
        assert heads[s] == oh[0], s
        assert state_rel_err(st[s], ost[0]) <= STATE_TOL, s
        assert np.abs(last[s] - olast[0]).max() <= LOGIT_TOL, s
        od = orc.Decoder(om)
        od.set_state(ost[0], int(oh[0]))
        ods.append((od, olast[0].copy()))
    # Greedy steps, the probed streams fed the oracle's own tokens.
    toks = np.array([orc.argmax(row) for row in last], dtype=np.uint32)
    checked = 0
    for step in range(4):
        for i, s in enumerate(probe):
            toks[s] = orc.argmax(ods[i][1])
        nxt = dec.step_greedy(toks).copy()
        for i, s in enumerate(probe):
            lg = ods[i][0].step(int(toks[s])).copy()
            top2 = np.sort(lg)[-2:]
            if top2[1] - top2[0] > LOGIT_TOL:
                assert int(nxt[s]) == orc.argmax(lg), (step, s)
                checked += 1
            ods[i] = (ods[i][0], lg)
        toks = nxt
    assert checked >= 12
