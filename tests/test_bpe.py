"""Byte-level BPE text I/O (bpe.rs) in the product library (nk_bpe_*, host
code) against the pure-Python restatement in oracle/bpe.py."""

import os
import subprocess

import numpy as np
import pytest

from oracle import bpe as ob

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CSRC = os.path.join(ROOT, "noetic_b200", "csrc")

SAMPLES = [  # selftest.rs:324-329
    "the quiet engine folds the dense lattice .",
    "memo alpha = 512 ; query alpha = 512 .",
    "unicode: héllo αβγ 漢字 \U0001f680 done",
    "12 + 34 = 46 .",
]


def _train_merges(text: str, n_merges: int) -> ob.Bpe:
    """A merge table for the tests: repeatedly merge the most frequent
    adjacent pair inside pre-token chunks (ties: smallest pair)."""
    bpe = ob.Bpe()
    words = [list(c.encode("utf-8")) for c in ob.pretokenize(text)]
    for _ in range(n_merges):
        counts = {}
        for w in words:
            for p in zip(w, w[1:]):
                counts[p] = counts.get(p, 0) + 1
        if not counts:
            break
        best = min(counts, key=lambda p: (-counts[p], p))
        new = bpe.vocab_size()
        bpe.push_merge(*best)
        for w in words:
            i = 0
            while i + 1 < len(w):
                if (w[i], w[i + 1]) == best:
                    w[i:i + 2] = [new]
                i += 1
    return bpe


def _random_text(rng, n_words: int) -> str:
    pieces = ["the", "a", "engine", "lattice", "héllo", "αβγ", "漢字", "\U0001f680",
              "12", "3456", ",", ".", ";", "  ", "\t", "x1y2", "مرحبا", "कि",
              "ª", "ͅ", "Ⅳ", "_", "'s", "あい"]
    return " ".join(pieces[i] for i in rng.integers(0, len(pieces), n_words))


@pytest.fixture(scope="module")
def trained():
    rng = np.random.default_rng(0)
    corpus = " ".join(SAMPLES) + " " + _random_text(rng, 400)
    return _train_merges(corpus, 120)


def _load(nb, tmp_path, text: str, name="tok.bpe"):
    path = tmp_path / name
    path.write_bytes(text.encode("utf-8") if isinstance(text, str) else text)
    return nb.Bpe.load(str(path))


def test_alphabetic_table_is_the_generated_one():
    # The committed table regenerates from the Unicode database byte for byte.
    gen = subprocess.run(["perl", os.path.join(CSRC, "gen_unicode_alpha.pl")], capture_output=True, text=True,
                         check=True).stdout
    with open(os.path.join(CSRC, "unicode_alpha.inc")) as f:
        assert f.read() == gen
    # Known members and non-members of the Alphabetic property.
    for ch, alpha in [("a", True), ("é", True), ("ª", True), ("ͅ", True), ("Ⅳ", True),
                      ("漢", True), ("0", False), ("١", False), ("_", False), ("\U0001f680", False)]:
        assert ob.is_alphabetic(ch) == alpha, ch


def test_encode_matches_the_restatement(nb, tmp_path, trained):
    gpu_bpe = _load(nb, tmp_path, trained.save_text())
    assert gpu_bpe.merges() == trained.merges and gpu_bpe.vocab_size() == trained.vocab_size()
    rng = np.random.default_rng(1)
    texts = SAMPLES + [_random_text(rng, int(k)) for k in rng.integers(1, 60, 40)] + ["", " ", "  x", "x  ", "é"]
    for t in texts:
        ids = gpu_bpe.encode(t)
        assert list(ids) == trained.encode(t), t
        assert gpu_bpe.decode(ids) == t  # selftest.rs:332-334
        assert gpu_bpe.decode_bytes(ids) == t.encode("utf-8")


def test_byte_path_round_trips_and_matches(nb, tmp_path, trained):
    # selftest.rs:338-344: arbitrary bytes encode / decode exactly; an id past
    # the vocabulary decodes to nothing (an error here).
    gpu_bpe = _load(nb, tmp_path, trained.save_text())
    rng = np.random.default_rng(2)
    for n in [0, 1, 2, 512, 3000]:
        data = rng.integers(0, 256, n, dtype=np.uint8).tobytes()
        ids = gpu_bpe.encode_bytes(data)
        assert list(ids) == trained.encode_bytes(data)
        assert gpu_bpe.decode_bytes(ids) == data
    # Repetitive input: ties between equal-rank pairs resolve leftmost first.
    for data in [b"aaaaaaa", b"abababab", b"the the the", b"    "]:
        assert list(gpu_bpe.encode_bytes(data)) == trained.encode_bytes(data)
    with pytest.raises(nb.NoeticError) as e:
        gpu_bpe.decode_bytes([gpu_bpe.vocab_size()])
    assert e.value.status == nb.NK_ERR_INVALID
    assert gpu_bpe.decode([gpu_bpe.vocab_size()]) == ""


def test_chained_merges(nb, tmp_path):
    # Merges that build on merges (256 + i used by later merges), as training makes.
    o = ob.Bpe()
    for a, b in [(97, 98), (256, 99), (257, 257), (100, 100), (259, 259), (258, 260)]:
        o.push_merge(a, b)
    g = _load(nb, tmp_path, o.save_text())
    for data in [b"abcabc", b"abcabcdddd", b"abcabcabcabcdddddddd", b"aabbcc", b"dddddd"]:
        assert list(g.encode_bytes(data)) == o.encode_bytes(data), data


def test_save_load_round_trip(nb, tmp_path, trained):
    g = _load(nb, tmp_path, trained.save_text())
    out = tmp_path / "saved.bpe"
    g.save(str(out))
    assert out.read_text() == trained.save_text()
    assert nb.Bpe.load(str(out)).merges() == trained.merges
    assert not [p for p in os.listdir(tmp_path) if ".tmp." in p]
    empty = nb.Bpe.bytes_only()
    empty.save(str(out))
    assert out.read_text() == "noetic-bpe 1\n0\n"


BAD_FILES = [
    "",  # no header
    "noetic-bpe 2\n0\n",
    "noetic-bpe 1\n",  # count missing
    "noetic-bpe 1\n-1\n",
    "noetic-bpe 1\n1 \n97 98\n",
    "noetic-bpe 1\n2\n97 98\n",  # truncated
    "noetic-bpe 1\n1\n97\n",
    "noetic-bpe 1\n1\n97 x\n",
    "noetic-bpe 1\n1\n97 98 99\n",
    "noetic-bpe 1\n1\n256 97\n",  # unknown token
    "noetic-bpe 1\n2\n97 98\n97 98\n",  # duplicate
    "noetic-bpe 1\n1\n97 98\nextra\n",
    "noetic-bpe 1\n1000001\n",
    "noetic-bpe 1\n1\n97 4294967296\n",
]
GOOD_FILES = [
    "noetic-bpe 1\n0\n",
    "noetic-bpe 1\r\n1\r\n97 98\r\n",  # CRLF line endings
    "noetic-bpe 1\n+1\n+97\t98\n",  # u32 FromStr takes a '+'; any Unicode whitespace separates
    "noetic-bpe 1\n1\n97 98\n",
    "noetic-bpe 1\n1\n97 98\n\n  \t\n",  # blank trailing lines
    "noetic-bpe 1\n1\n97 98",  # no final newline
]


@pytest.mark.parametrize("text", BAD_FILES + GOOD_FILES)
def test_loader_accepts_and_rejects_like_the_reference(nb, tmp_path, text):
    try:
        ref = ob.load_text(text.encode("utf-8"))
    except ValueError:
        ref = None
    assert (text in GOOD_FILES) == (ref is not None)
    if ref is None:
        with pytest.raises(nb.NoeticError) as e:
            _load(nb, tmp_path, text)
        assert e.value.status == nb.NK_ERR_IO
    else:
        assert _load(nb, tmp_path, text).merges() == ref.merges


def test_loader_rejects_exponential_token_expansion(nb, tmp_path):
    # bpe.rs:383-395: 22 self-merges of one token would expand to 4 MiB.
    text = "noetic-bpe 1\n22\n" + "".join(f"{97 if m == 0 else 255 + m} {97 if m == 0 else 255 + m}\n"
                                          for m in range(22))
    with pytest.raises(ValueError):
        ob.load_text(text.encode())
    with pytest.raises(nb.NoeticError) as e:
        _load(nb, tmp_path, text)
    assert e.value.status == nb.NK_ERR_IO


def test_loader_rejects_invalid_utf8_and_bad_text(nb, tmp_path):
    with pytest.raises(nb.NoeticError):
        _load(nb, tmp_path, b"noetic-bpe 1\n0\n\xff\n")
    b = nb.Bpe.bytes_only()
    with pytest.raises(nb.NoeticError) as e:  # encode takes &str: UTF-8 only
        b._ids(nb.lib().nk_bpe_encode, b"\xc3\x28")
    assert e.value.status == nb.NK_ERR_INVALID
    with pytest.raises(nb.NoeticError):
        nb.Bpe.load(str(tmp_path / "missing.bpe"))
