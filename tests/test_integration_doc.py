"""CPU: the ctypes stubs of the integration guide (what a maintainer would
paste into the reference's client) match the library's real signatures."""
import ctypes
import re
from pathlib import Path

from fack_b200 import _lib

DOC = Path(__file__).resolve().parents[1] / "INTEGRATION.md"
ALIASES = {"i": ctypes.c_int, "i64": ctypes.c_int64, "p": ctypes.c_void_p, "sz": ctypes.c_size_t}


def parse_type(tok: str):
    tok = tok.strip()
    m = re.fullmatch(r"ctypes\.POINTER\((\w+)\)", tok)
    if m:
        return ctypes.POINTER(ALIASES[m.group(1)])
    return ALIASES[tok]


def stubs():
    text = DOC.read_text()
    found = {}
    for m in re.finditer(r"lib\.(fack_\w+)\.argtypes = \[(.*?)\]\n", text, flags=re.S):
        toks = [t for t in re.split(r",\s*", " ".join(m.group(2).split())) if t]
        found[m.group(1)] = [parse_type(t) for t in toks]
    return found


def test_every_stub_matches_the_library_signature():
    found = stubs()
    assert {"fack_gemm_bs_ex", "fack_gemm_bs_plan", "fack_quant_act", "fack_gemm_tn"} <= set(found)
    for name, args in found.items():
        want = _lib.SIGNATURES[name][1]
        assert len(args) == len(want), (name, len(args), len(want))
        for k, (a, w) in enumerate(zip(args, want)):
            assert a == w or (getattr(a, "_type_", None) is getattr(w, "_type_", None)
                              and a.__name__.startswith("LP_") and w.__name__.startswith("LP_")), (name, k, a, w)
