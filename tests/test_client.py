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


# --- pinned to the reference client's own C++ -------------------------------

def _client_fixture():
    import base64
    import json
    import os
    with open(os.path.join(os.path.dirname(__file__), "golden", "client.json")) as f:
        d = json.load(f)
    return Vocab.from_bytes(base64.b64decode(d["vocab_b64"])), d


def test_decode_tokens_matches_reference_client():
    """decode_tokens against bfp_client.cpp's decode_tokens
    (bfp_client.cpp:1020-1027), run by tests/golden/make_client_golden.py on
    304 streams over a vocabulary of split, mojibake, invalid and
    out-of-range entries."""
    v, d = _client_fixture()
    bad = [(ids, h) for ids, h in d["token_cases"] if decode_tokens(v, ids).hex() != h]
    assert len(d["token_cases"]) >= 300 and not bad, bad[:3]


def test_fix_mojibake_matches_reference_client():
    """fix_mojibake against bfp_client.cpp's fix_mojibake (:977-1018) on 366
    byte strings, random bytes included."""
    _, d = _client_fixture()
    bad = [(r, h) for r, h in d["mojibake_cases"] if fix_mojibake(bytes.fromhex(r)).hex() != h]
    assert len(d["mojibake_cases"]) >= 360 and not bad, bad[:3]


def test_fix_mojibake_against_live_reference_client(tmp_path):
    """Fresh random byte strings through the reference's own fix_mojibake,
    when oracle/build_client_ref.sh has built it from a reference checkout."""
    import os
    import subprocess
    import numpy as np
    exe = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref", "bfp_client_ref")
    if not os.path.exists(exe):
        pytest.skip("reference client not built (oracle/build_client_ref.sh needs the reference checkout)")
    v, _ = _client_fixture()
    vp = tmp_path / "v.bin"
    vp.write_bytes(v.to_bytes())
    rng = np.random.default_rng()
    pool = [v.bytes_for(i) for i in range(len(v.entries))] + [bytes([b]) for b in range(256)]
    cases = [b"".join(pool[int(i)] for i in rng.integers(0, len(pool), size=int(rng.integers(0, 12))))
             for _ in range(500)]
    streams = [rng.integers(0, len(v.entries) + 3, size=int(rng.integers(0, 16))).tolist() for _ in range(200)]
    lines = ["M " + c.hex() for c in cases] + ["T " + " ".join(map(str, s)) for s in streams]
    out = subprocess.run([exe, str(vp)], input="\n".join(lines) + "\n", capture_output=True, text=True,
                         check=True, timeout=60).stdout.split("\n")
    for k, c in enumerate(cases):
        assert fix_mojibake(c).hex() == out[k], c
    for k, s in enumerate(streams):
        assert decode_tokens(v, s).hex() == out[len(cases) + k], s
