"""Client text fixtures from the reference client's own C++.

Builds oracle/_ref/bfp_client_ref (oracle/build_client_ref.sh compiles
decode_tokens and fix_mojibake of rtl/vc707/host/bfp_client.cpp:904-1027
where they lie in the reference checkout), feeds it a seeded synthetic
vocabulary and seeded cases, and writes tests/golden/client.json:

    vocab_b64        the BFPV blob (format of gen_bfp_vocab_bin.py)
    token_cases      [[ids...], hex of decode_tokens(vocab, ids)]
    mojibake_cases   [hex of raw bytes, hex of fix_mojibake(raw)]

The real bfp_vocab.bin comes from the SmolLM2 tokenizer, which is not
available offline; the synthetic vocabulary instead holds the byte patterns
the repair logic distinguishes: ASCII, valid UTF-8 of 2-4 bytes, UTF-8 text
read as Windows-1252 and re-encoded (mojibake), split multi-byte sequences,
lone continuation and invalid lead bytes, NUL, the 0x80-0x9F specials, empty
entries and entries that point past the blob.

    python tests/golden/make_client_golden.py [reference checkout]
"""
import base64
import json
import os
import subprocess
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "tinyllm-fpga_b200"))
from bfp200.client import Vocab  # noqa: E402

BIN = os.path.join(REPO, "oracle", "_ref", "bfp_client_ref")

WORDS = ["Hello", " world", ",", " the", " caf", "é", " naïve", " über", "—", "’s", " “quote”", "…", "€", " ™",
         "日本", "語", " 😀", "🚀", "Ω", " Ž", "œ", "Ÿ", "ñ", "\n", "\t", " "]


def _mojibake(text: str) -> bytes:
    """UTF-8 text read as Windows-1252 and written back as UTF-8: the
    byte-level tokenizer artefact the client repairs."""
    raw = text.encode("utf-8")
    return raw.decode("cp1252", errors="ignore").encode("utf-8")


def token_pool(rng):
    toks = []
    for w in WORDS:
        toks.append(w.encode())
        toks.append(_mojibake(w))
        b = w.encode()
        if len(b) > 1:                                  # split sequences across tokens
            k = int(rng.integers(1, len(b)))
            toks += [b[:k], b[k:]]
    for _ in range(60):                                 # random valid code points, 1-4 bytes
        cp = int(rng.choice([rng.integers(0x20, 0x7F), rng.integers(0x80, 0x800),
                             rng.integers(0x800, 0xD800), rng.integers(0xE000, 0x10000),
                             rng.integers(0x10000, 0x110000)]))
        toks.append(chr(cp).encode("utf-8", errors="surrogatepass"))
    for _ in range(30):                                 # random bytes >= 0x80 (invalid leads, continuations)
        toks.append(bytes(rng.integers(0x80, 0x100, size=int(rng.integers(1, 4))).astype(np.uint8)))
    for cp in (0x20AC, 0x201A, 0x0192, 0x2026, 0x2122, 0x0153, 0x0178, 0x81, 0x8D, 0x9D):
        toks.append(chr(cp).encode())
    toks += [b"", b"\x00", b"a\x00b", b"\xc3", b"\xa9", b"\xe2\x80", b"\x9c", b"\xf0\x9f", b"\x98\x80"]
    return toks


def main(argv):
    ref = argv[1] if len(argv) > 1 else None
    cmd = ["sh", os.path.join(REPO, "oracle", "build_client_ref.sh")] + ([ref] if ref else [])
    subprocess.run(cmd, check=True)
    rng = np.random.default_rng(20251)
    toks = token_pool(rng)
    v = Vocab.from_tokens(toks)
    # two entries that point past the blob decode to nothing
    v = Vocab(v.entries + [(len(v.blob) - 2, 5), (len(v.blob) + 10, 1)], v.blob)
    n = len(v.entries)

    token_cases = [[], [n - 1], [n - 2], [n, 65535]]
    for _ in range(300):
        L = int(rng.integers(1, 24))
        ids = rng.integers(0, n, size=L).tolist()
        if rng.random() < 0.1:
            ids[int(rng.integers(0, L))] = int(rng.integers(n, 65536))   # id past the table
        token_cases.append([int(i) for i in ids])

    moji = [b"", b"\x80", b"\xff\xfe", "â€”".encode(), "Ã©".encode(), "â‚¬".encode()]
    for _ in range(300):
        parts = [toks[int(i)] for i in rng.integers(0, len(toks), size=int(rng.integers(1, 8)))]
        moji.append(b"".join(parts))
    for _ in range(60):
        moji.append(bytes(rng.integers(0, 256, size=int(rng.integers(1, 20))).astype(np.uint8)))

    vpath = os.path.join(REPO, "oracle", "_ref", "client_vocab.bin")
    with open(vpath, "wb") as f:
        f.write(v.to_bytes())
    lines = ["T " + " ".join(str(i) for i in ids) for ids in token_cases]
    lines += ["M " + b.hex() for b in moji]
    out = subprocess.run([BIN, vpath], input="\n".join(lines) + "\n", capture_output=True, text=True, check=True)
    res = out.stdout.split("\n")
    res = res[:len(lines)]
    assert len(res) == len(lines), (len(res), len(lines))
    nt = len(token_cases)
    doc = {
        "generator": "tests/golden/make_client_golden.py (reference bfp_client.cpp decode_tokens / fix_mojibake)",
        "vocab_b64": base64.b64encode(v.to_bytes()).decode(),
        "token_cases": [[ids, res[k]] for k, ids in enumerate(token_cases)],
        "mojibake_cases": [[b.hex(), res[nt + k]] for k, b in enumerate(moji)],
    }
    path = os.path.join(HERE, "client.json")
    with open(path, "w") as f:
        json.dump(doc, f, separators=(",", ":"))
    print(f"wrote {path}: {len(token_cases)} token cases, {len(moji)} mojibake cases, vocab {n} entries")


if __name__ == "__main__":
    main(sys.argv)
