"""The failure path of the bounded device waits, exercised without a fault.

Every cross-CTA wait in the decode kernels is bounded; on expiry the kernel
records an error code, finishes its work in bounds and exits, and the host
reports NK_ERR_DEVICE with the code.  The reference has no counterpart: it
aborts (release builds use panic = "abort").  Test controls (decoder engine
bits 12 and 13) make one hand-off never happen, so the waits run out (after
2 ms): the tensor-core projections publish no stream-K partial tile (code
121), or the persistent step's first CTA skips its first grid-barrier arrival
(code 113).  The decoder must then be usable: after restoring the state the
failed step left undefined, the next steps equal those of a decoder that
never failed, bit for bit (both engines are deterministic)."""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

WITHHOLD_PUBLISH = 4096
WITHHOLD_ARRIVAL = 8192
MODEL = dict(vocab=4096, d_model=1024, n_layer=2, expand=1, conv_k=4, mlp_mult=3, eps=1e-5, tau_max=128.0)


def _run(gpu, gm, S, ids, control, code):
    ref = gpu.Decoder(gm, S)
    dec = gpu.Decoder(gm, S)
    t_ref = t = None
    for d in (ref, dec):
        last = d.prefill(ids)
        tok = np.argmax(last, axis=1).astype(np.uint32)
        tok = d.step_greedy(tok).copy()
        if d is ref:
            t_ref = tok
        else:
            t = tok
    assert np.array_equal(t, t_ref)
    state, heads = dec.get_state()
    dec.set_engine(control)
    with pytest.raises(gpu.NoeticError) as e:
        dec.step_greedy(t)
    assert e.value.status == gpu.NK_ERR_DEVICE
    assert f"code {code}" in str(e.value), str(e.value)
    dec.set_engine(0)
    dec.set_state(state, heads)
    for _ in range(3):
        t = dec.step_greedy(t).copy()
        t_ref = ref.step_greedy(t_ref).copy()
        assert np.array_equal(t, t_ref)
    s1, h1 = dec.get_state()
    s2, h2 = ref.get_state()
    assert np.array_equal(h1, h2)
    assert np.array_equal(s1.view(np.uint32), s2.view(np.uint32))


def test_expired_stream_k_handoff_is_reported_and_recovered(gpu):
    # 2048 streams: the A operand fits L2, so every 256-wide store and SwiGLU
    # projection is spread by stream-K and has partial tiles to hand off.
    gm = gpu.Model.new(gpu.LmConfig(**MODEL), 11, device=0)
    S = 2048
    ids = (np.arange(S * 4, dtype=np.uint32).reshape(S, 4) * 40503 % MODEL["vocab"]).astype(np.uint32)
    _run(gpu, gm, S, ids, WITHHOLD_PUBLISH, 121)


@pytest.mark.parametrize("S", [1, 3])
def test_expired_persistent_grid_barrier_is_reported_and_recovered(gpu, S):
    gm = gpu.Model.new(gpu.LmConfig(**MODEL), 12, device=0)
    ids = (np.arange(S * 5, dtype=np.uint32).reshape(S, 5) * 977 % MODEL["vocab"]).astype(np.uint32)
    _run(gpu, gm, S, ids, WITHHOLD_ARRIVAL, 113)
