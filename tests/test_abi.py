"""The product library's C ABI on CPU: it loads, exports every symbol that
include/noetic_gpu.h declares, and its host-side parts (seeded initialiser,
checkpoint reader/writer, validation) agree with the oracle.  Nothing here
launches a kernel."""

import os
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_symbols():
    names = set()
    for fn in os.listdir(os.path.join(ROOT, "include")):
        if fn.endswith(".h"):
            text = open(os.path.join(ROOT, "include", fn)).read()
            text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
            names |= set(re.findall(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b(nk_\w+)\s*\(", text, flags=re.M))
    return sorted(names)


def test_library_exports_every_declared_symbol(nb):
    import ctypes

    L = ctypes.CDLL(nb.LIB_PATH)
    syms = header_symbols()
    assert len(syms) >= 30
    missing = [s for s in syms if not hasattr(L, s)]
    assert not missing, missing
    # The Python mirror binds exactly the declared surface.
    assert set(syms) == set(nb.SIGNATURES)


def test_config_check_mirrors_lmconfig_check(nb):
    nb.LmConfig(vocab=10, d_model=8, n_layer=1).check()
    for bad in [dict(vocab=0), dict(d_model=0), dict(n_layer=0), dict(expand=0), dict(conv_k=0),
                dict(mlp_mult=0), dict(eps=0.0), dict(eps=float("nan")), dict(tau_max=0.5)]:
        kw = dict(vocab=10, d_model=8, n_layer=1)
        kw.update(bad)
        with pytest.raises(nb.NoeticError) as e:
            nb.LmConfig(**kw).check()
        assert e.value.status == nb.NK_ERR_INVALID


CFGS = [
    dict(vocab=19, d_model=16, n_layer=2, expand=2, conv_k=3, mlp_mult=2, eps=1e-5, tau_max=8.0),
    dict(vocab=1024, d_model=192, n_layer=3, expand=1, conv_k=4, mlp_mult=3, eps=1e-5, tau_max=128.0),
    dict(vocab=17, d_model=5, n_layer=1, expand=3, conv_k=1, mlp_mult=1, eps=1e-5, tau_max=1.0),
]


@pytest.mark.parametrize("cfg", CFGS)
def test_seeded_init_is_bit_exact_with_the_oracle(nb, orc, cfg):
    seed = 20250816
    gm = nb.Model(nb.LmConfig(**cfg), device=-1)
    import ctypes

    after = np.zeros(4, dtype=np.uint64)
    nb._check(nb.lib().nk_model_init_random(gm.h, seed, after.ctypes.data_as(ctypes.c_void_p)))
    r = orc.Rng(seed)
    om = orc.Model(orc.LmConfig(**cfg), rng=r)
    names = [n for n, _ in gm.tensor_names()]
    assert names == [n for n, _ in om.tensors()]
    for name, a in om.tensors():
        assert np.array_equal(gm.get_tensor(name), a), name
    assert [int(v) for v in after] == r.s


def test_checkpoint_interop_with_the_oracle(nb, orc, tmp_path):
    cfg = CFGS[0]
    om = orc.Model(orc.LmConfig(**cfg), seed=11)
    p = str(tmp_path / "o.ckpt")
    om.save(p)
    gm = nb.Model.load(p, device=-1)
    assert gm.cfg.vocab == cfg["vocab"] and gm.cfg.n_layer == cfg["n_layer"]
    for name, a in om.tensors():
        assert np.array_equal(gm.get_tensor(name), a)
    q = str(tmp_path / "g.ckpt")
    gm.save(q)
    om2 = orc.Model.load(q)
    for (n1, a1), (n2, a2) in zip(om.tensors(), om2.tensors()):
        assert n1 == n2 and np.array_equal(a1, a2)


def test_corrupt_truncated_and_mismatched_checkpoints_are_rejected(nb, orc, tmp_path):
    om = orc.Model(orc.LmConfig(**CFGS[0]), seed=11)
    p = str(tmp_path / "o.ckpt")
    om.save(p)
    raw = open(p, "rb").read()
    cases = {
        "flip": raw[:50] + bytes([raw[50] ^ 1]) + raw[51:],
        "truncated": raw[: len(raw) // 2],
        "tiny": raw[:10],
        "empty": b"",
    }
    for name, data in cases.items():
        f = str(tmp_path / f"{name}.ckpt")
        open(f, "wb").write(data)
        with pytest.raises(nb.NoeticError) as e:
            nb.Model.load(f, device=-1)
        assert e.value.status == nb.NK_ERR_IO, name
    with pytest.raises(nb.NoeticError):
        nb.Model.load(str(tmp_path / "missing.ckpt"), device=-1)


def test_missing_metadata_is_rejected(nb, orc, tmp_path):
    om = orc.Model(orc.LmConfig(**CFGS[0]), seed=11)
    meta = om.default_meta()
    del meta["tau_max"]
    p = str(tmp_path / "nometa.ckpt")
    om.save(p, meta)
    with pytest.raises(nb.NoeticError) as e:
        nb.Model.load(p, device=-1)
    assert "tau_max" in str(e.value)


def test_set_tensor_validates_name_shape_and_values(nb):
    gm = nb.Model(nb.LmConfig(**CFGS[0]), device=-1)
    with pytest.raises(nb.NoeticError):
        gm.set_tensor("no.such.tensor", np.zeros(3, np.float32))
    with pytest.raises(nb.NoeticError):
        gm.set_tensor("emb", np.zeros((19, 17), np.float32))
    bad = np.zeros((19, 16), np.float32)
    bad[3, 4] = np.nan
    with pytest.raises(nb.NoeticError):
        gm.set_tensor("emb", bad)
    ok = np.arange(19 * 16, dtype=np.float32).reshape(19, 16)
    gm.set_tensor("emb", ok)
    assert np.array_equal(gm.get_tensor("emb"), ok)


def test_host_only_model_cannot_run_a_decoder(nb):
    gm = nb.Model(nb.LmConfig(**CFGS[0]), device=-1)
    with pytest.raises(nb.NoeticError) as e:
        nb.Decoder(gm, 2)
    assert e.value.status == nb.NK_ERR_INVALID


def test_rng_state_helper_matches_oracle(nb, orc):
    for seed in [0, 3000, 2**64 - 1]:
        assert [int(v) for v in nb.rng_state(seed)] == orc.Rng(seed).s


def test_training_ops_refuse_bad_arguments_before_any_device_work(nb):
    # AdamW's assertions (optim.rs:34-38) and the shape limits are checked on
    # the host, so these refusals need no GPU.
    z = np.zeros(4, np.float32)
    for kw in [dict(lr=-1.0), dict(lr=float("inf")), dict(lr=0.1, b1=1.0), dict(lr=0.1, b2=-0.5),
               dict(lr=0.1, eps=0.0), dict(lr=0.1, wd=-1.0), dict(lr=0.1, t=0)]:
        args = dict(t=1)
        args.update(kw)
        with pytest.raises(nb.NoeticError) as e:
            nb.adamw_step(z, z, z, z, **args)
        assert e.value.status == nb.NK_ERR_INVALID
    with pytest.raises(nb.NoeticError) as e:  # kernel width above the weight-gradient kernel's 16
        nb.dwconv_backward(np.zeros(34), np.zeros(17 * 2), np.zeros(34), 1, 17, 2, 17)
    assert e.value.status == nb.NK_ERR_INVALID
    with pytest.raises(nb.NoeticError) as e:
        nb.dwconv_backward(np.zeros(0), np.zeros(0), np.zeros(0), 1, 0, 0, 4)
    assert e.value.status == nb.NK_ERR_INVALID
    # Empty products need no device either.
    assert nb.gemm_tn(np.zeros(0), np.zeros(0), 0, 0, 5).shape == (0, 5)


def test_crc32_pieces_combine_to_the_reference_crc(nb):
    # ckpt::crc32 (ckpt.rs:35-54) is zlib's CRC-32; the library computes it in
    # 16 MiB pieces combined by polynomial arithmetic, as the loader does.
    import ctypes
    import zlib

    rng = np.random.default_rng(4)
    for n in [0, 1, 7, 8, 9, 1000, (16 << 20) - 1, 16 << 20, (16 << 20) + 1, (40 << 20) + 12345]:
        data = rng.integers(0, 256, n, dtype=np.uint8)
        out = ctypes.c_uint32(0)
        nb._check(nb.lib().nk_crc32(data.ctypes.data_as(ctypes.c_void_p), n, ctypes.byref(out)))
        assert out.value == zlib.crc32(data.tobytes()), n
