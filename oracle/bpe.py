"""Pure-Python restatement of the reference's byte-level BPE (bpe.rs), test
infrastructure only: the oracle the product's BPE (nk_bpe_*) is checked
against, for small inputs (encode_raw is the reference's O(n^2) rescan).

char::is_alphabetic is the Unicode Alphabetic property.  Its code points come
from the Unicode database that ships with Perl, listed once per process by
``perl -e`` (no table is shared with the product library).
"""

from __future__ import annotations

import functools
import subprocess

MAX_TOKENIZER_FILE_BYTES = 64 * 1024 * 1024  # bpe.rs:15-18
MAX_SERIALIZED_MERGES = 1_000_000
MAX_EXPANDED_TOKEN_BYTES = 1024 * 1024
MAX_TOTAL_EXPANDED_BYTES = 128 * 1024 * 1024

# char::is_whitespace (the White_Space property), used by str::trim and
# str::split_whitespace.
_WHITE_SPACE = set(range(0x09, 0x0E)) | {0x20, 0x85, 0xA0, 0x1680, 0x2028, 0x2029, 0x202F, 0x205F, 0x3000} | set(
    range(0x2000, 0x200B))


@functools.lru_cache(maxsize=1)
def _alphabetic() -> frozenset:
    script = ('for my $c (0..0x10FFFF) { next if $c >= 0xD800 && $c <= 0xDFFF; '
              'print "$c\\n" if chr($c) =~ /\\p{Alphabetic}/ }')
    out = subprocess.run(["perl", "-e", script], capture_output=True, text=True, check=True).stdout
    return frozenset(int(x) for x in out.split())


def is_alphabetic(ch: str) -> bool:
    return ord(ch) in _alphabetic()


def pretokenize(text: str) -> list[str]:
    """Bpe::pretokenize (bpe.rs:77-115)."""
    out: list[str] = []
    cur = ""
    cur_kind = 0  # 0 none, 1 alpha, 2 digit, 3 other
    for ch in text:
        kind = 1 if is_alphabetic(ch) else 2 if "0" <= ch <= "9" else 3
        if ch == " ":
            if cur:
                out.append(cur)
            cur = ch
            cur_kind = 0
            continue
        if cur_kind == 0 and cur == " ":
            cur += ch
            cur_kind = kind
            continue
        if kind != cur_kind or kind == 3:
            if cur:
                out.append(cur)
                cur = ""
            cur_kind = kind
        cur += ch
    if cur:
        out.append(cur)
    return out


class Bpe:
    """Bpe (bpe.rs:21-27): merge i makes token 256 + i."""

    def __init__(self):
        self.merges: list[tuple[int, int]] = []
        self.rank: dict[tuple[int, int], int] = {}
        self.token_bytes: list[bytes] = [bytes([b]) for b in range(256)]

    def vocab_size(self) -> int:
        return len(self.token_bytes)

    def push_merge(self, a: int, b: int):
        """Bpe::push_merge (bpe.rs:59-75)."""
        assert a < len(self.token_bytes) and b < len(self.token_bytes)
        assert (a, b) not in self.rank
        self.rank[(a, b)] = len(self.merges)
        self.merges.append((a, b))
        self.token_bytes.append(self.token_bytes[a] + self.token_bytes[b])

    def encode_raw(self, data: bytes) -> list[int]:
        """Bpe::encode_raw (bpe.rs:222-246): rescan, merge the lowest-rank
        (leftmost) pair, repeat."""
        symbols = list(data)
        while len(symbols) >= 2:
            best_rank, best_index = None, None
            for i in range(len(symbols) - 1):
                r = self.rank.get((symbols[i], symbols[i + 1]))
                if r is not None and (best_rank is None or r < best_rank):
                    best_rank, best_index = r, i
            if best_index is None:
                break
            symbols[best_index] = 256 + best_rank
            del symbols[best_index + 1]
        return symbols

    def encode(self, text: str) -> list[int]:
        """Bpe::encode (bpe.rs:252-258)."""
        out: list[int] = []
        for chunk in pretokenize(text):
            out.extend(self.encode_raw(chunk.encode("utf-8")))
        return out

    def encode_bytes(self, data: bytes) -> list[int]:
        return self.encode_raw(data)

    def decode_bytes(self, ids) -> bytes | None:
        """Bpe::decode_bytes (bpe.rs:268-279): None on an out-of-range id."""
        if any(i >= len(self.token_bytes) for i in ids):
            return None
        return b"".join(self.token_bytes[i] for i in ids)

    def save_text(self) -> str:
        """The text Bpe::save (bpe.rs:288-307) writes."""
        return "noetic-bpe 1\n" + f"{len(self.merges)}\n" + "".join(f"{a} {b}\n" for a, b in self.merges)


def _parse_uint(s: str, limit: int) -> int | None:
    """u32 / usize FromStr: an optional '+', then ASCII digits."""
    body = s[1:] if s.startswith("+") else s
    if not body or not all("0" <= c <= "9" for c in body):
        return None
    v = int(body)
    return v if v <= limit else None


def _split_ws(line: str) -> list[str]:
    out, cur = [], ""
    for ch in line:
        if ord(ch) in _WHITE_SPACE:
            if cur:
                out.append(cur)
            cur = ""
        else:
            cur += ch
    if cur:
        out.append(cur)
    return out


def load_text(raw: bytes) -> Bpe:
    """Bpe::load (bpe.rs:309-380) on the file's bytes; raises ValueError
    where the reference returns an InvalidData error."""
    if len(raw) > MAX_TOKENIZER_FILE_BYTES:
        raise ValueError("tokenizer file exceeds the supported size limit")
    try:
        text = raw.decode("utf-8")
    except UnicodeDecodeError as e:
        raise ValueError("stream did not contain valid UTF-8") from e
    # str::lines: split on "\n", a "\r" before the "\n" dropped.
    parts = text.split("\n")
    lines = [ln[:-1] if ln.endswith("\r") else ln for ln in parts[:-1]]
    if parts[-1] != "":
        lines.append(parts[-1])
    it = iter(lines)
    if next(it, None) != "noetic-bpe 1":
        raise ValueError("unsupported tokenizer header or version")
    cnt_line = next(it, None)
    if cnt_line is None:
        raise ValueError("tokenizer merge count is missing")
    count = _parse_uint(cnt_line, 2**64 - 1)
    if count is None:
        raise ValueError("tokenizer merge count is invalid")
    if count > MAX_SERIALIZED_MERGES or count > 0xFFFFFFFF - 256:
        raise ValueError("tokenizer declares too many merges")
    bpe = Bpe()
    total = 256
    for _ in range(count):
        line = next(it, None)
        if line is None:
            raise ValueError("tokenizer merge list is truncated")
        fields = _split_ws(line)
        if len(fields) < 1:
            raise ValueError("tokenizer merge is missing its first token")
        a = _parse_uint(fields[0], 0xFFFFFFFF)
        if a is None:
            raise ValueError("tokenizer merge token is invalid")
        if len(fields) < 2:
            raise ValueError("tokenizer merge is missing its second token")
        b = _parse_uint(fields[1], 0xFFFFFFFF)
        if b is None:
            raise ValueError("tokenizer merge token is invalid")
        if len(fields) > 2:
            raise ValueError("tokenizer merge has extra fields")
        nxt = bpe.vocab_size()
        if a >= nxt or b >= nxt:
            raise ValueError("tokenizer merge references an unknown token")
        if (a, b) in bpe.rank:
            raise ValueError("tokenizer contains a duplicate merge pair")
        expanded = len(bpe.token_bytes[a]) + len(bpe.token_bytes[b])
        if expanded > MAX_EXPANDED_TOKEN_BYTES:
            raise ValueError("tokenizer contains an excessively large expanded token")
        total += expanded
        if total > MAX_TOTAL_EXPANDED_BYTES:
            raise ValueError("tokenizer expanded vocabulary exceeds the supported size limit")
        bpe.push_merge(a, b)
    for line in it:
        if _split_ws(line):
            raise ValueError("tokenizer has trailing data")
    return bpe
