"""Build step: extract the IQ2/IQ3 codebook grids from the reference sources.

The IQ2_XXS / IQ2_XS / IQ2_S / IQ3_XXS / IQ3_S formats decode every 8 (IQ2) or
4 (IQ3) weights through a fixed codebook of packed u8 grid points.  The
codebooks are part of the GGUF format: a decoder that uses any other values is
not decoding GGUF.  They are therefore not written out by hand here; this
script reads them at build time from the reference's own Rust tables

    crates/hayai-model/src/iq2.rs  IQ2XXS_GRID (:30), IQ2XS_GRID (:98), IQ2S_GRID (:230)
    crates/hayai-model/src/iq3.rs  IQ3XXS_GRID (:29), IQ3S_GRID (:65)
    crates/hayai-model/src/iq4.rs  KVALUES_IQ4NL (:15), the 16 signed levels of IQ4_NL / IQ4_XS

and writes them as a C header (``_gen/iq_tables.h``) that both the CUDA
library and the CPU oracle include.  The generated header is a build product
(git-ignored), like the shared libraries compiled from it.

The sign table ``KSIGNS_IQ2XS`` (iq2.rs:18) is not extracted: entry ``i`` is
``i`` with bit 7 set to the parity of ``i`` (so every sign byte has an even
number of set bits); both the kernels and the oracle compute it from that rule.

Usage: python gen_iq_tables.py <reference_root> <out_header>
"""
from __future__ import annotations

import os
import re
import sys

TABLES = [
    # (rust file, rust name, C name, element C type, expected length)
    ("crates/hayai-model/src/iq2.rs", "IQ2XXS_GRID", "hc_iq2xxs_grid", "uint64_t", 256),
    ("crates/hayai-model/src/iq2.rs", "IQ2XS_GRID", "hc_iq2xs_grid", "uint64_t", 512),
    ("crates/hayai-model/src/iq2.rs", "IQ2S_GRID", "hc_iq2s_grid", "uint64_t", 1024),
    ("crates/hayai-model/src/iq3.rs", "IQ3XXS_GRID", "hc_iq3xxs_grid", "uint32_t", 256),
    ("crates/hayai-model/src/iq3.rs", "IQ3S_GRID", "hc_iq3s_grid", "uint32_t", 512),
]


def extract(src: str, name: str, n: int) -> list[int]:
    m = re.search(r"static\s+" + name + r"\s*:\s*\[u(?:32|64);\s*(\d+)\]\s*=\s*\[(.*?)\];", src, re.S)
    if not m:
        raise SystemExit(f"gen_iq_tables: table {name} not found")
    if int(m.group(1)) != n:
        raise SystemExit(f"gen_iq_tables: {name} declared with {m.group(1)} entries, want {n}")
    vals = [int(tok, 16) for tok in re.findall(r"0x[0-9a-fA-F]+", m.group(2))]
    if len(vals) != n:
        raise SystemExit(f"gen_iq_tables: {name} has {len(vals)} entries, want {n}")
    return vals


SIGNED = [
    # (rust file, rust name, C name, expected length): decimal i8 tables
    ("crates/hayai-model/src/iq4.rs", "KVALUES_IQ4NL", "hc_iq4nl_values", 16),
]


def extract_i8(src: str, name: str, n: int) -> list[int]:
    m = re.search(r"const\s+" + name + r"\s*:\s*\[i8;\s*(\d+)\]\s*=\s*\[(.*?)\];", src, re.S)
    if not m:
        raise SystemExit(f"gen_iq_tables: table {name} not found")
    vals = [int(tok) for tok in re.findall(r"-?\d+", m.group(2))]
    if int(m.group(1)) != n or len(vals) != n or any(v < -128 or v > 127 for v in vals):
        raise SystemExit(f"gen_iq_tables: {name} is not {n} int8 values")
    return vals


def main(argv: list[str]) -> int:
    if len(argv) != 3:
        print(__doc__)
        return 2
    ref, out = argv[1], argv[2]
    lines = [
        "/* Generated at build time by gen_iq_tables.py from the reference's IQ codebooks. */",
        "#pragma once",
        "#include <stdint.h>",
        "/* Storage qualifier: plain static const for host code; CUDA code defines",
        "   HC_IQ_QUAL as `static __device__ const` before including. */",
        "#ifndef HC_IQ_QUAL",
        "#define HC_IQ_QUAL static const",
        "#endif",
        "",
    ]
    cache: dict[str, str] = {}
    for path, rname, cname, ctype, n in TABLES:
        full = os.path.join(ref, path)
        if full not in cache:
            with open(full, encoding="utf-8") as f:
                cache[full] = f.read()
        vals = extract(cache[full], rname, n)
        width = 16 if ctype == "uint64_t" else 8
        suffix = "ull" if ctype == "uint64_t" else "u"
        lines.append(f"#define {cname.upper()}_LEN {n}")
        lines.append(f"HC_IQ_QUAL {ctype} {cname}[{n}] = {{")
        per = 4 if ctype == "uint64_t" else 8
        for i in range(0, n, per):
            chunk = ", ".join(f"0x{v:0{width}x}{suffix}" for v in vals[i:i + per])
            lines.append(f"    {chunk},")
        lines.append("};")
        lines.append("")
    for path, rname, cname, n in SIGNED:
        full = os.path.join(ref, path)
        if full not in cache:
            with open(full, encoding="utf-8") as f:
                cache[full] = f.read()
        vals = extract_i8(cache[full], rname, n)
        lines.append(f"HC_IQ_QUAL int8_t {cname}[{n}] = {{{', '.join(str(v) for v in vals)}}};")
        lines.append("")
    os.makedirs(os.path.dirname(os.path.abspath(out)), exist_ok=True)
    tmp = out + ".tmp"
    with open(tmp, "w", encoding="utf-8") as f:
        f.write("\n".join(lines))
    os.replace(tmp, out)
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv))
