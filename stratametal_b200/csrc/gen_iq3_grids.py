"""Regenerate ``iq3xxs_grid.inc`` and ``iq3s_grid.inc``: the IQ3_XXS (ggml type 18) and IQ3_S (type 21) codebooks as
C initializer lists.

The tables are format data, not code: an IQ3 weight block stores indices into these codebooks (256 entries for
IQ3_XXS, 512 for IQ3_S), each entry packing 4 unsigned int8 magnitudes.  A decoder must use exactly these values, so
they are extracted mechanically (never retyped) from the StrataMetal header
``metal/include/strata/metal/iq_grids.hpp`` (``iq3xxs_grid``, ``iq3s_grid``), which itself was generated from ggml's
``ggml-common.h`` (MIT licence, Copyright (c) 2023-2024 The ggml authors).  The header is only present in the build
container; the generated ``.inc`` files are committed.

usage: python gen_iq3_grids.py /path/to/strata/metal/include/strata/metal/iq_grids.hpp
"""
import re
import sys
from pathlib import Path


def extract(header_text: str, name: str, n: int) -> list[int]:
    m = re.search(name + r"\[" + str(n) + r"\]\s*=\s*\{(.*?)\};", header_text, re.S)
    if not m:
        raise SystemExit(f"{name}[{n}] not found")
    vals = [int(v, 16) for v in re.findall(r"0x([0-9a-fA-F]+)u", m.group(1))]
    if len(vals) != n:
        raise SystemExit(f"{name}: expected {n} entries, found {len(vals)}")
    return vals


def main() -> None:
    text = Path(sys.argv[1]).read_text()
    for name, n, ggml_type in (("iq3xxs_grid", 256, "IQ3_XXS, type 18"), ("iq3s_grid", 512, "IQ3_S, type 21")):
        vals = extract(text, name, n)
        out = Path(__file__).with_name(name + ".inc")
        lines = [
            f"/* {ggml_type} codebook: {n} entries, 4 unsigned int8 magnitudes each, byte j = value j.",
            " * Format data from ggml's ggml-common.h, MIT licence, Copyright (c) 2023-2024 The ggml authors,",
            f" * extracted mechanically by gen_iq3_grids.py from StrataMetal's iq_grids.hpp ({name}).",
            " * Do not edit by hand. */",
        ]
        for i in range(0, n, 8):
            lines.append(", ".join(f"0x{v:08x}u" for v in vals[i:i + 8]) + ",")
        out.write_text("\n".join(lines) + "\n")
        print(f"wrote {out} ({len(vals)} entries)")


if __name__ == "__main__":
    main()
