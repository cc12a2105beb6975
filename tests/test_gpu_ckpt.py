"""The direct checkpoint -> device loader (nk_model_load_ckpt on a device):
headers scanned, payloads streamed through pinned buffers into the device
arena, CRC (ckpt.rs:35-54) and finiteness checked -- against the host reader
and the oracle."""

import struct
import zlib

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

# 34 MB of weights: three 16 MiB streaming chunks, tensors across both boundaries.
BIG = dict(vocab=20000, d_model=256, n_layer=4, expand=1, conv_k=4, mlp_mult=3, eps=1e-5, tau_max=64.0)


def _parse(raw: bytes):
    """(meta items, [(name, shape, f32 array)]) of a checkpoint (ckpt.rs:299-383)."""
    off = 12

    def u32():
        nonlocal off
        v = struct.unpack_from("<I", raw, off)[0]
        off += 4
        return v

    def s():
        nonlocal off
        n = u32()
        v = raw[off:off + n].decode()
        off += n
        return v

    meta = [(s(), s()) for _ in range(u32())]
    tensors = []
    for _ in range(u32()):
        name = s()
        shape = [u32() for _ in range(u32())]
        n = u32()
        tensors.append((name, shape, np.frombuffer(raw, np.float32, n, off).copy()))
        off += 4 * n
    return meta, tensors


def _write(meta, tensors) -> bytes:
    """A checkpoint in the reference's format (ckpt.rs:125-200)."""
    b = bytearray(b"NOETIC\x00\x01") + struct.pack("<I", 1) + struct.pack("<I", len(meta))
    for k, v in meta:
        for x in (k.encode(), v.encode()):
            b += struct.pack("<I", len(x)) + x
    b += struct.pack("<I", len(tensors))
    for name, shape, data in tensors:
        nb_ = name.encode()
        b += struct.pack("<I", len(nb_)) + nb_ + struct.pack("<I", len(shape))
        b += b"".join(struct.pack("<I", d) for d in shape) + struct.pack("<I", data.size)
        b += np.ascontiguousarray(data, np.float32).tobytes()
    return bytes(b + struct.pack("<I", zlib.crc32(bytes(b))))


@pytest.fixture(scope="module")
def big_ckpt(orc, tmp_path_factory):
    om = orc.Model(orc.LmConfig(**BIG), seed=6)
    p = str(tmp_path_factory.mktemp("ck") / "big.ckpt")
    om.save(p)
    return om, p


def test_direct_load_equals_the_host_reader_and_the_oracle(gpu, orc, big_ckpt):
    om, p = big_ckpt
    raw = open(p, "rb").read()
    assert len(raw) > 2 * (16 << 20)
    gm = gpu.Model.load(p, device=0)
    hm = gpu.Model.load(p, device=-1)
    _, tensors = _parse(raw)
    for name, shape, data in tensors:
        got = gm.get_tensor(name)
        assert np.array_equal(got.reshape(-1), data), name
        assert np.array_equal(hm.get_tensor(name).reshape(-1), data), name
    # The loaded weights run: streaming logits follow the oracle.
    dec, od = gpu.Decoder(gm, 1), orc.Decoder(om)
    for t in [5, 19999, 123, 7]:
        assert np.abs(dec.step([t])[0] - od.step(t)).max() <= 1e-3


def test_direct_load_rejects_corruption(gpu, big_ckpt, tmp_path):
    _, p = big_ckpt
    raw = open(p, "rb").read()
    meta, tensors = _parse(raw)
    nan_in_payload = [(n, s, d.copy()) for n, s, d in tensors]
    nan_in_payload[3][2][17] = np.nan
    inf_in_aux = tensors + [("aux.adamw.m.emb", [4], np.array([0, 1, np.inf, 3], np.float32))]
    cases = {
        "flip_in_payload": raw[: 20 << 20] + bytes([raw[20 << 20] ^ 4]) + raw[(20 << 20) + 1:],
        "flip_in_crc": raw[:-1] + bytes([raw[-1] ^ 1]),
        "truncated": raw[: len(raw) // 2],
        "tiny": raw[:10],
        "empty": b"",
        "trailing": raw[:-4] + b"\x00\x00\x00\x00" + raw[-4:],
        "nan_in_tensor": _write(meta, nan_in_payload),
        "inf_in_aux": _write(meta, inf_in_aux),
        "missing_tensor": _write(meta, tensors[:-1]),
        "wrong_shape": _write(meta, [(n, ([s[0] + 1] + s[1:]) if i == 0 else s,
                                      np.zeros(int(np.prod([s[0] + 1] + s[1:])), np.float32) if i == 0 else d)
                                     for i, (n, s, d) in enumerate(tensors)]),
    }
    for name, data in cases.items():
        f = str(tmp_path / f"{name}.ckpt")
        open(f, "wb").write(data)
        with pytest.raises(gpu.NoeticError) as e:
            gpu.Model.load(f, device=0)
        assert e.value.status == gpu.NK_ERR_IO, name


def test_aux_tensors_are_checked_but_not_kept(gpu, orc, tmp_path):
    # apply_exact (ckpt.rs:410-436) ignores the aux.* namespace.
    kw = dict(vocab=40, d_model=24, n_layer=2, expand=2, conv_k=3, mlp_mult=2, eps=1e-5, tau_max=16.0)
    om = orc.Model(orc.LmConfig(**kw), seed=4)
    p = str(tmp_path / "m.ckpt")
    om.save(p)
    meta, tensors = _parse(open(p, "rb").read())
    aux = [("aux.adamw.m.emb", [40 * 24], np.ones(40 * 24, np.float32)), ("aux.steps", [0], np.zeros(0, np.float32))]
    q = str(tmp_path / "aux.ckpt")
    open(q, "wb").write(_write(meta, aux[:1] + tensors + aux[1:]))
    gm = gpu.Model.load(q, device=0)
    for name, _, data in tensors:
        assert np.array_equal(gm.get_tensor(name).reshape(-1), data)


def test_a_directly_loaded_model_can_be_edited_and_saved(gpu, orc, big_ckpt, tmp_path):
    om, p = big_ckpt
    gm = gpu.Model.load(p, device=0)
    d1 = gpu.Decoder(gm, 1)
    before = d1.step([11])[0].copy()
    # set_tensor on a model whose host copies start empty: every other tensor
    # must come back from the device before the next upload.
    g = gm.get_tensor("norm_f.gain")
    gm.set_tensor("norm_f.gain", (g * 2).astype(np.float32))
    d2 = gpu.Decoder(gm, 1)
    after = d2.step([11])[0]
    assert not np.allclose(before, after)
    q = str(tmp_path / "edited.ckpt")
    gm.save(q)
    gm2 = gpu.Model.load(q, device=0)
    assert np.array_equal(gm2.get_tensor("norm_f.gain"), (g * 2).astype(np.float32))
    assert np.array_equal(gm2.get_tensor("emb"), gm.get_tensor("emb"))
    d3 = gpu.Decoder(gm2, 1)
    assert np.abs(d3.step([11])[0] - after).max() < 1e-6
