"""Writes quant_grids.h: the codebooks of the IQ2_S, IQ3_S and IQ4_XS GGUF
codecs, which every decoder of those formats must use unchanged (ggml's
iq2s_grid, iq3s_grid and kvalues_iq4nl, MIT licence), taken from the table
header the reference engine decodes with:

    python gpeed_b200/csrc/make_quant_grids.py <reference root>

The output pins each table's SHA-256; tests/test_codecs.py re-checks the
digests and, where the reference tree exists, the values themselves.
"""
import hashlib
import os
import re
import struct
import sys

HERE = os.path.dirname(os.path.abspath(__file__))


def table(text: str, name: str) -> list[int]:
    m = re.search(name + r"\s*\[[^\]]*\]\s*=\s*\{(.*?)\};", text, re.S)
    if not m:
        raise SystemExit(f"table {name} not found")
    return [int(t, 0) for t in m.group(1).replace("\n", " ").split(",") if t.strip()]


def rows(vals, fmt, per):
    out = []
    for i in range(0, len(vals), per):
        out.append("    " + " ".join(fmt.format(v) + "," for v in vals[i:i + per]))
    return " \\\n".join(out)


def main() -> int:
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("GPEED_REFERENCE_ROOT", "")
    text = open(os.path.join(ref, "cpp", "core", "include", "glm5", "quant_tables.h")).read()
    g2 = table(text, "kIq2sGrid")
    g3 = table(text, "kIq3sGrid")
    v4 = table(text, "kValuesIq4nl")
    assert len(g2) == 1024 and len(g3) == 512 and len(v4) == 16
    d2 = hashlib.sha256(struct.pack("<1024Q", *g2)).hexdigest()
    d3 = hashlib.sha256(struct.pack("<512I", *g3)).hexdigest()
    d4 = hashlib.sha256(struct.pack("<16b", *v4)).hexdigest()
    hdr = f"""// Codebooks of the IQ2_S, IQ3_S and IQ4_XS GGUF codecs.  Format data, not
// code: every decoder of these formats must use exactly these values (they are
// ggml's iq2s_grid, iq3s_grid and kvalues_iq4nl, MIT licence, the tables the
// reference engine decodes with in cpp/core/include/glm5/quant_tables.h).
// Written by make_quant_grids.py; tests/test_codecs.py checks the digests.
//   IQ2_S grid  1024 x u64: eight unsigned magnitudes per entry, one per byte
//   IQ3_S grid   512 x u32: four unsigned magnitudes per entry
//   IQ4_NL/XS values 16 x i8
#pragma once
#include <stdint.h>

#define GPEED_IQ2S_GRID_SHA256 "{d2}"
#define GPEED_IQ3S_GRID_SHA256 "{d3}"
#define GPEED_IQ4NL_VALUES_SHA256 "{d4}"

#define GPEED_IQ2S_GRID_VALUES \\
{rows(g2, "0x{:016x}ull", 4)}

#define GPEED_IQ3S_GRID_VALUES \\
{rows(g3, "0x{:08x}u", 8)}

#define GPEED_IQ4NL_VALUES \\
{rows(v4, "{:d}", 16)}
"""
    with open(os.path.join(HERE, "quant_grids.h"), "w") as fh:
        fh.write(hdr)
    print("wrote", os.path.join(HERE, "quant_grids.h"))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
