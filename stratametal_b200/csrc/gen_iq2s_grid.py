"""Regenerate ``iq2s_grid.inc``: the IQ2_S codebook (ggml type 22) as a C initializer list.

The table is format data, not code: an IQ2_S weight block stores 10-bit indices into this
1024-entry codebook, each entry packing 8 unsigned int8 magnitudes.  A kernel that decodes IQ2_S
must use exactly these 1024 values, so they are extracted mechanically (never retyped) from the
StrataMetal header ``metal/include/strata/metal/iq_grids.hpp`` (``iq2s_grid``, lines 5-262), which
itself was generated from ggml's ``ggml-common.h`` (MIT licence, Copyright (c) 2023-2024 The ggml
authors).  The header is only present in the build container; the generated ``.inc`` is committed.

usage: python gen_iq2s_grid.py /path/to/strata/metal/include/strata/metal/iq_grids.hpp
"""
import re
import sys
from pathlib import Path


def extract(header_text: str) -> list[int]:
    m = re.search(r"iq2s_grid\[1024\]\s*=\s*\{(.*?)\};", header_text, re.S)
    if not m:
        raise SystemExit("iq2s_grid[1024] not found")
    vals = [int(v, 16) for v in re.findall(r"0x([0-9a-fA-F]+)ull", m.group(1))]
    if len(vals) != 1024:
        raise SystemExit(f"expected 1024 entries, found {len(vals)}")
    return vals


def main() -> None:
    src = Path(sys.argv[1])
    vals = extract(src.read_text())
    out = Path(__file__).with_name("iq2s_grid.inc")
    lines = [
        "/* IQ2_S codebook (ggml type 22): 1024 entries, 8 unsigned int8 magnitudes each, byte j = value j.",
        " * Format data from ggml's ggml-common.h, MIT licence, Copyright (c) 2023-2024 The ggml authors,",
        " * extracted mechanically by gen_iq2s_grid.py from StrataMetal's iq_grids.hpp (iq2s_grid).",
        " * Do not edit by hand. */",
    ]
    for i in range(0, 1024, 4):
        lines.append(", ".join(f"0x{v:016x}ull" for v in vals[i:i + 4]) + ",")
    out.write_text("\n".join(lines) + "\n")
    print(f"wrote {out} ({len(vals)} entries)")


if __name__ == "__main__":
    main()
