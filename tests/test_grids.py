"""The codebooks committed as .inc files (IQ2_S, IQ3_XXS, IQ3_S) have their formats' sizes and equal the tables of
the reference's grid header they were extracted from.  The second check runs only where the reference tree is
present (located as the oracle's Makefile locates it, REF_ROOT), like the oracle's own reference build."""
import importlib.util
import os
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
CSRC = ROOT / "stratametal_b200" / "csrc"
GRIDS = [("iq2s_grid.inc", 1024, "gen_iq2s_grid.py"), ("iq3xxs_grid.inc", 256, "gen_iq3_grids.py"),
         ("iq3s_grid.inc", 512, "gen_iq3_grids.py")]


def inc_values(name: str) -> list[int]:
    return [int(v, 16) for v in re.findall(r"0x([0-9a-f]+)u", (CSRC / name).read_text())]


def ref_header() -> Path | None:
    # the Makefile's default: a checkout named `reference` beside this repository
    root = os.environ.get("REF_ROOT", str(ROOT.parent / "reference"))
    p = Path(root) / "metal" / "include" / "strata" / "metal" / "iq_grids.hpp"
    return p if root and p.exists() else None


def load(script: str):
    spec = importlib.util.spec_from_file_location(script[:-3], CSRC / script)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.mark.parametrize("inc,n,_gen", GRIDS)
def test_codebook_sizes(inc, n, _gen):
    assert len(inc_values(inc)) == n


@pytest.mark.parametrize("inc,n,gen", GRIDS)
def test_codebooks_equal_the_reference_header(inc, n, gen):
    h = ref_header()
    if h is None:
        pytest.skip("the reference tree is absent here")
    text = h.read_text()
    mod = load(gen)
    want = mod.extract(text) if gen == "gen_iq2s_grid.py" else mod.extract(text, inc[:-4], n)
    assert inc_values(inc) == want
