"""Client-compatible output: the `RTL_TOKENS:` / `DECODED:` lines that
`bfp_client tokens` prints (rtl/vc707/host/bfp_client.cpp:1503-1524), from a
token stream decoded on the GPU, so demo flows built around the client's
output work unchanged.

The vocabulary is the client's `BFPV` blob (written by
rtl/vc707/host/gen_bfp_vocab_bin.py:1-79): magic "BFPV", u32 version = 1,
u32 n_tokens, u32 blob_size, n_tokens x (u32 offset, u32 length), blob; all
little-endian.  Each entry holds the raw UTF-8 bytes of one token.

Decoding concatenates the token bytes and repairs "mojibake" the way the
client does (bfp_client.cpp:904-1027): the byte string is read as UTF-8
code points (an invalid lead byte stands for itself), every maximal run of
code points that map back to single Windows-1252 bytes >= 0x80 is turned
into those bytes, and if the bytes decode as UTF-8 without an invalid lead
byte and produce a code point above 0xFF, the decoded text replaces the run.

Usage as a program (needs a B200 for the decode):
    python -m bfp200.client --image lbfp_full_DDR3.bin --roms <dir> \
        --vocab bfp_vocab.bin --n-gen 15 [--feed rtl]
"""
from __future__ import annotations

import struct

MAGIC = b"BFPV"

# code points of Windows-1252's 0x80-0x9F specials -> their byte
# (bfp_client.cpp:947-971)
_WIN1252_SPECIAL = {
    0x20AC: 0x80, 0x201A: 0x82, 0x0192: 0x83, 0x201E: 0x84, 0x2026: 0x85, 0x2020: 0x86, 0x2021: 0x87,
    0x02C6: 0x88, 0x2030: 0x89, 0x0160: 0x8A, 0x2039: 0x8B, 0x0152: 0x8C, 0x017D: 0x8E, 0x2018: 0x91,
    0x2019: 0x92, 0x201C: 0x93, 0x201D: 0x94, 0x2022: 0x95, 0x2013: 0x96, 0x2014: 0x97, 0x02DC: 0x98,
    0x2122: 0x99, 0x0161: 0x9A, 0x203A: 0x9B, 0x0153: 0x9C, 0x017E: 0x9E, 0x0178: 0x9F,
}


class VocabError(ValueError):
    pass


class Vocab:
    """The client's token -> bytes table (Vocab::load, bfp_client.cpp:876-903)."""

    def __init__(self, entries, blob):
        self.entries = list(entries)
        self.blob = bytes(blob)

    @classmethod
    def from_bytes(cls, data: bytes) -> "Vocab":
        if len(data) < 4 or data[:4] != MAGIC:
            raise VocabError("bad vocab magic")
        if len(data) < 16:
            raise VocabError("vocab truncated")
        version, n, blob_size = struct.unpack_from("<III", data, 4)
        if version != 1:
            raise VocabError(f"unsupported vocab version {version}")
        off = 16
        if len(data) < off + 8 * n + blob_size:
            raise VocabError("vocab truncated")
        entries = [struct.unpack_from("<II", data, off + 8 * i) for i in range(n)]
        off += 8 * n
        return cls(entries, data[off:off + blob_size])

    @classmethod
    def load(cls, path) -> "Vocab":
        with open(path, "rb") as f:
            return cls.from_bytes(f.read())

    def to_bytes(self) -> bytes:
        out = bytearray(MAGIC)
        out += struct.pack("<III", 1, len(self.entries), len(self.blob))
        for o, n in self.entries:
            out += struct.pack("<II", o, n)
        return bytes(out + self.blob)

    @classmethod
    def from_tokens(cls, token_bytes) -> "Vocab":
        """Builds a table from per-id byte strings (id = list index)."""
        entries, blob = [], bytearray()
        for b in token_bytes:
            entries.append((len(blob), len(b)))
            blob += b
        return cls(entries, blob)

    def bytes_for(self, tok: int) -> bytes:
        """Raw bytes of one id; empty for an unknown id or a bad entry."""
        if tok < 0 or tok >= len(self.entries):
            return b""
        o, n = self.entries[tok]
        if o + n > len(self.blob):
            return b""
        return self.blob[o:o + n]


def _next_cp(s: bytes, i: int):
    """One UTF-8 code point at s[i]: (code point, next index); an invalid or
    truncated sequence yields its lead byte as the code point."""
    b = s[i]
    if b < 0x80:
        return b, i + 1
    if (b & 0xE0) == 0xC0:
        n, cp = 2, b & 0x1F
    elif (b & 0xF0) == 0xE0:
        n, cp = 3, b & 0x0F
    elif (b & 0xF8) == 0xF0:
        n, cp = 4, b & 0x07
    else:
        return b, i + 1
    if i + n > len(s):
        return b, i + 1
    for k in range(1, n):
        c = s[i + k]
        if (c & 0xC0) != 0x80:
            return b, i + 1
        cp = (cp << 6) | (c & 0x3F)
    return cp, i + n


def _cp_bytes(cp: int) -> bytes:
    """UTF-8 encoding of any code point below 2^21 (surrogates included)."""
    if cp < 0x80:
        return bytes([cp])
    if cp < 0x800:
        return bytes([0xC0 | (cp >> 6), 0x80 | (cp & 0x3F)])
    if cp < 0x10000:
        return bytes([0xE0 | (cp >> 12), 0x80 | ((cp >> 6) & 0x3F), 0x80 | (cp & 0x3F)])
    return bytes([0xF0 | (cp >> 18), 0x80 | ((cp >> 12) & 0x3F), 0x80 | ((cp >> 6) & 0x3F), 0x80 | (cp & 0x3F)])


def _win1252_byte(cp: int) -> int:
    if cp < 0x80 or 0xA0 <= cp <= 0xFF:
        return cp
    return _WIN1252_SPECIAL.get(cp, -1)


def fix_mojibake(raw: bytes) -> bytes:
    """The client's greedy repair of UTF-8 text that was decoded as
    Windows-1252 and re-encoded (bfp_client.cpp:977-1018)."""
    cps, i = [], 0
    while i < len(raw):
        cp, i = _next_cp(raw, i)
        cps.append(cp)
    out = bytearray()
    i = 0
    while i < len(cps):
        if _win1252_byte(cps[i]) < 0x80:
            out += _cp_bytes(cps[i])
            i += 1
            continue
        j = i
        run = bytearray()
        while j < len(cps):
            b = _win1252_byte(cps[j])
            if b < 0x80:
                break
            run.append(b)
            j += 1
        decoded = bytearray()
        ok, gained, k = len(run) > 0, False, 0
        while k < len(run):
            prev = k
            cp, k = _next_cp(run, k)
            if k == prev + 1 and run[prev] >= 0x80:
                ok = False
                break
            if cp > 0xFF:
                gained = True
            decoded += _cp_bytes(cp)
        if ok and gained:
            out += decoded
        else:
            for c in cps[i:j]:
                out += _cp_bytes(c)
        i = j
    return bytes(out)


def decode_tokens(vocab: Vocab, tokens) -> bytes:
    """Token ids -> UTF-8 text bytes (decode_tokens, bfp_client.cpp:1020-1027)."""
    return fix_mojibake(b"".join(vocab.bytes_for(int(t)) for t in tokens))


def format_tokens(tokens, vocab: Vocab | None = None) -> bytes:
    """The client's printout (print_tokens, bfp_client.cpp:1503-1523):
    `RTL_TOKENS: t0 t1 ...` and, with a vocabulary, `DECODED:` + the text."""
    out = b"RTL_TOKENS:" + b"".join(b" %d" % int(t) for t in tokens) + b"\n"
    if vocab is not None:
        text = decode_tokens(vocab, tokens).split(b"\0", 1)[0]      # printf("%s") stops at a NUL
        out += b"DECODED:\n" + text + b"\n"
    return out


def main(argv=None):
    import argparse
    import sys
    from .config import BfpConfig
    from .engine import Decoder
    ap = argparse.ArgumentParser(description="decode on the GPU and print like `bfp_client tokens`")
    ap.add_argument("--image", required=True, help="<PREFIX>DDR3.bin")
    ap.add_argument("--roms", required=True, help="directory with the <PREFIX>*.hex ROM files")
    ap.add_argument("--prefix", default="lbfp_full_")
    ap.add_argument("--vocab", default=None, help="BFPV vocabulary blob (bfp_vocab.bin)")
    ap.add_argument("--n-gen", type=int, default=15)
    ap.add_argument("--feed", choices=["sim", "rtl"], default="rtl")
    ap.add_argument("--device", type=int, default=0)
    a = ap.parse_args(argv)
    vocab = Vocab.load(a.vocab) if a.vocab else None
    with Decoder(BfpConfig.from_env(MAX_CTX=48 + a.n_gen, max_seqs=1), device=a.device) as dec:
        dec.load_image(a.image)
        dec.load_roms(a.roms, a.prefix)
        toks = dec.generate(None, a.n_gen, feed_mode=a.feed)[0]
    sys.stdout.buffer.write(format_tokens(toks, vocab))
    sys.stdout.flush()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
