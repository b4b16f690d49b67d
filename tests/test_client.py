"""Client-compatible output (bfp_client.cpp:876-1027, 1503-1524): the BFPV
vocabulary blob format, the mojibake repair and the RTL_TOKENS / DECODED
printout.  Host logic only."""
import pytest

from bfp200.client import Vocab, VocabError, decode_tokens, fix_mojibake, format_tokens


def _vocab():
    toks = [b"Hello", b",", b" world", b"\xe2\x80", b"\x94", b" caf", b"\xc3\xa9", b"\xff", b"\x00x", b""]
    return Vocab.from_tokens(toks)


def test_blob_round_trip_and_layout():
    v = _vocab()
    data = v.to_bytes()
    assert data[:4] == b"BFPV" and data[4:8] == (1).to_bytes(4, "little")
    assert int.from_bytes(data[8:12], "little") == 10
    w = Vocab.from_bytes(data)
    assert [w.bytes_for(i) for i in range(10)] == [v.bytes_for(i) for i in range(10)]
    assert w.bytes_for(10) == b"" and w.bytes_for(-1) == b""


def test_blob_errors():
    data = _vocab().to_bytes()
    with pytest.raises(VocabError):
        Vocab.from_bytes(b"XXXX" + data[4:])
    with pytest.raises(VocabError):
        Vocab.from_bytes(data[:4] + (2).to_bytes(4, "little") + data[8:])
    with pytest.raises(VocabError):
        Vocab.from_bytes(data[:-1])
    # an entry pointing past the blob decodes to nothing
    bad = Vocab([(0, 3), (2, 5)], b"abcd")
    assert bad.bytes_for(0) == b"abc" and bad.bytes_for(1) == b""


@pytest.mark.parametrize("raw,want", [
    (b"plain ascii", b"plain ascii"),
    ("café".encode(), "café".encode()),                                   # valid UTF-8 kept
    ("—".encode(), "—".encode()),                                         # em dash from byte tokens
    ("â€”".encode(), "—".encode()),                                       # UTF-8 read as cp1252
    ("itâ€™s".encode(), "it’s".encode()),
    ("Ã©tÃ©".encode(), "Ã©tÃ©".encode()),                                # repairs only reaching > U+00FF
    (b"\xff", "ÿ".encode()),                                              # invalid byte stands for itself
    (b"a\xe2\x80", "aâ\u0080".encode()),                                  # truncated sequence
    ("€".encode(), "€".encode()),                                         # one special alone: no gain
])
def test_fix_mojibake(raw, want):
    assert fix_mojibake(raw) == want


def test_decode_and_format():
    v = _vocab()
    assert decode_tokens(v, [0, 1, 2]) == b"Hello, world"
    assert decode_tokens(v, [5, 6, 3, 4]) == " café—".encode()
    assert format_tokens([0, 1, 2]) == b"RTL_TOKENS: 0 1 2\n"
    assert format_tokens([0, 2], v) == b"RTL_TOKENS: 0 2\nDECODED:\nHello world\n"
    assert format_tokens([0, 8, 2], v) == b"RTL_TOKENS: 0 8 2\nDECODED:\nHello\n"   # printf stops at NUL
    assert format_tokens([], v) == b"RTL_TOKENS:\nDECODED:\n\n"
