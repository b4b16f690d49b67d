"""File surface of the reference packers: DDR3 image region map, .hex ROM
files, cfg.svh, PROMPT / GOLDEN_TOKENS files.

References (jrrk2/tinyllm-fpga):
* region order / 4 KiB alignment: rtl/vc707/host/gen_smollm_blockfp_ddr.py:155-241,
  rtl/vc707/src/smollm/lbfp_ddr3.svh:45-86 (the packer is authoritative where
  the two disagree: NORM_W_e follows a 4 KiB-aligned NORM_W_m region);
* .hex parsing: rtl/vc707/host/bfp_client.cpp:1162-1183 (parse_hex_file);
* ROM kinds: bfp_client.cpp:1140-1150 and :1381-1437 (load_roms);
* cfg.svh: rtl/vc707/host/gen_smollm_blockfp_cfg.py:61-77;
* PROMPT.hex: gen_smollm_blockfp_full.py:394-396;
* GOLDEN_TOKENS.txt: gen_smollm_blockfp_full.py:447-449;
* RTL_TOKENS line: bfp_client.cpp:1519-1521.
"""
from __future__ import annotations

import os
import re

import numpy as np

from .config import BfpConfig

ALIGN = 4096

ROM_KINDS = {0: "G1_m.hex", 1: "G1_e.hex", 2: "G2_m.hex", 3: "G2_e.hex",
             4: "NORM_W_m.hex", 5: "NORM_W_e.hex", 6: "PROMPT.hex"}


def align4k(n: int) -> int:
    return (n + ALIGN - 1) & ~(ALIGN - 1)


def matrix_specs(cfg: BfpConfig):
    """(tag, D_out, D_in) of the seven per-layer matrices, in image order."""
    kvd = cfg.H_KV * cfg.HD
    return [("WQ", cfg.D, cfg.D), ("WK", kvd, cfg.D), ("WV", kvd, cfg.D), ("WO", cfg.D, cfg.D),
            ("WG", cfg.FFN, cfg.D), ("WU", cfg.FFN, cfg.D), ("WDN", cfg.D, cfg.FFN)]


def region_map(cfg: BfpConfig):
    """Ordered list of (name, offset, unpadded size); last entry ('END', total, 0)."""
    out = []
    off = 0

    def add(name, size):
        nonlocal off
        out.append((name, off, size))
        off += align4k(size)

    for tag, dout, din in matrix_specs(cfg):
        add(f"{tag}_m", cfg.NL * (dout // 16) * din * 32)
        add(f"{tag}_e", cfg.NL * (dout // 16) * (din // 16) * 16)
    ntd = cfg.D // 16
    add("G1_m", cfg.NL * cfg.D * 2)
    add("G1_e", cfg.NL * ntd)
    add("G2_m", cfg.NL * cfg.D * 2)
    add("G2_e", cfg.NL * ntd)
    add("EMBED_m", cfg.VOCAB // 16 * cfg.D * 32)
    add("EMBED_e", cfg.VOCAB // 16 * ntd * 16)
    add("EMBED_LU_m", cfg.VOCAB * cfg.D * 2)
    add("EMBED_LU_e", cfg.VOCAB * 64)
    add("NORM_W_m", cfg.D * 2)
    add("NORM_W_e", ntd)
    out.append(("END", off, 0))
    return out


def image_size(cfg: BfpConfig) -> int:
    return region_map(cfg)[-1][1]


def write_offsets(path, cfg: BfpConfig, image_name="DDR3.bin"):
    """<PREFIX>DDR3.offsets.txt in the packer's format (:237-241)."""
    with open(path, "w") as f:
        f.write(f"# Region offsets in {image_name}\n")
        for name, off, _ in region_map(cfg)[:-1]:
            f.write(f"  {name:14s}  0x{off:08X}  ({off:,} B)\n")


# ---------------------------------------------------------------------------
# .hex files
# ---------------------------------------------------------------------------
_TOK = re.compile(r"\S+")


def parse_hex_file(path):
    """bfp_client.cpp:1162-1183: strip '//' and '#' comments, hex tokens,
    keep the low 16 bits, skip tokens that are not hex."""
    out = []
    with open(path) as f:
        for line in f:
            line = line.split("//", 1)[0].split("#", 1)[0]
            for tok in _TOK.findall(line):
                try:
                    out.append(int(tok, 16) & 0xFFFF)
                except ValueError:
                    pass
    return np.array(out, dtype=np.uint16)


def write_hex(path, values, digits):
    mask = (1 << (4 * digits)) - 1
    with open(path, "w") as f:
        for v in np.asarray(values).ravel():
            f.write(f"{int(v) & mask:0{digits}x}\n")


def rom_path(directory, prefix, name):
    """load_roms tries <dir>/<prefix><name> first, then <dir>/<name> (:1398-1403)."""
    p1 = os.path.join(directory, prefix + name)
    return p1 if os.path.exists(p1) else os.path.join(directory, name)


def read_roms(directory, prefix="lbfp_full_"):
    """All seven ROM files of a release directory -> {kind: uint16 array}."""
    prefix = os.environ.get("MGRT_PREFIX", prefix)
    return {k: parse_hex_file(rom_path(directory, prefix, n)) for k, n in ROM_KINDS.items()}


def write_roms(directory, prefix, g1, g2, norm_w, prompt_ids):
    """Writes the ROM set (gen_smollm_blockfp_full.py:164-175, 394-403).
    g1/g2: lists of (m, e) per layer; norm_w: (m, e)."""
    os.makedirs(directory, exist_ok=True)
    write_hex(os.path.join(directory, prefix + "G1_m.hex"), np.concatenate([m.ravel() for m, _ in g1]), 4)
    write_hex(os.path.join(directory, prefix + "G1_e.hex"), np.concatenate([e.ravel() for _, e in g1]), 2)
    write_hex(os.path.join(directory, prefix + "G2_m.hex"), np.concatenate([m.ravel() for m, _ in g2]), 4)
    write_hex(os.path.join(directory, prefix + "G2_e.hex"), np.concatenate([e.ravel() for _, e in g2]), 2)
    write_hex(os.path.join(directory, prefix + "NORM_W_m.hex"), norm_w[0].ravel(), 4)
    write_hex(os.path.join(directory, prefix + "NORM_W_e.hex"), norm_w[1].ravel(), 2)
    write_hex(os.path.join(directory, prefix + "PROMPT.hex"), np.asarray(prompt_ids), 4)


# ---------------------------------------------------------------------------
# cfg.svh, prompt and token files
# ---------------------------------------------------------------------------
def write_cfg_svh(path, cfg: BfpConfig, n_prompt: int, n_gen: int):
    """gen_smollm_blockfp_cfg.py:61-77 (VOCAB already LANES-padded)."""
    with open(path, "w") as f:
        f.write(f"`define LBFP_FULL_D           {cfg.D}\n")
        f.write(f"`define LBFP_FULL_HQ          {cfg.H_Q}\n")
        f.write(f"`define LBFP_FULL_HKV         {cfg.H_KV}\n")
        f.write(f"`define LBFP_FULL_HD          {cfg.HD}\n")
        f.write(f"`define LBFP_FULL_FFN         {cfg.FFN}\n")
        f.write(f"`define LBFP_FULL_NL          {cfg.NL}\n")
        f.write(f"`define LBFP_FULL_MAX_CTX     {cfg.MAX_CTX}\n")
        f.write(f"`define LBFP_FULL_VOCAB       {cfg.VOCAB}\n")
        f.write(f"`define LBFP_FULL_NPROMPT     {n_prompt}\n")
        f.write(f"`define LBFP_FULL_NPROMPT_MAX {cfg.NPROMPT_MAX}\n")
        f.write(f"`define LBFP_FULL_NGEN        {n_gen}\n")


def read_cfg_svh(path) -> BfpConfig:
    vals = {}
    with open(path) as f:
        for line in f:
            m = re.match(r"`define\s+LBFP_FULL_(\w+)\s+(\S+)", line)
            if m:
                vals[m.group(1)] = int(m.group(2))
    return BfpConfig(D=vals["D"], H_Q=vals["HQ"], H_KV=vals["HKV"], HD=vals["HD"], FFN=vals["FFN"],
                     NL=vals["NL"], MAX_CTX=vals["MAX_CTX"], VOCAB=vals["VOCAB"],
                     NPROMPT_MAX=vals.get("NPROMPT_MAX", 48), N_GEN=vals.get("NGEN", 15))


def write_token_lines(path, tokens):
    """GOLDEN_TOKENS.txt / PROMPT_TOKENS.txt: one id per line."""
    with open(path, "w") as f:
        for t in tokens:
            f.write(f"{int(t)}\n")


def read_token_lines(path):
    with open(path) as f:
        return [int(x) for x in f.read().split()]


def rtl_tokens_line(tokens) -> str:
    """The client's `RTL_TOKENS:` line (bfp_client.cpp:1519-1521)."""
    return "RTL_TOKENS:" + "".join(f" {int(t)}" for t in tokens)
