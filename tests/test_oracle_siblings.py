"""CPU: the sibling-family oracle against golden vectors made by the
reference's own gemm_driver.prepare() (tests/golden/make_golden_siblings.py)."""
import json

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from oracle import siblings as sib

INDEX = json.loads((GOLDEN / "index_siblings.json").read_text())


def load(name):
    z = np.load(GOLDEN / f"sib_{name}.npz")
    g = {k: z[k] for k in z.files}
    fam = INDEX[name]["family"]
    if fam == "bf16":
        g["a"] = torch.from_numpy(g["a"]).view(torch.bfloat16)
        g["b"] = torch.from_numpy(g["b"]).view(torch.bfloat16)
    else:
        for k in ("a", "b", "sa", "sb", "bias"):
            g[k] = torch.from_numpy(g[k])
    g["reference"] = torch.from_numpy(g["reference"]).view(torch.bfloat16)
    return fam, g


@pytest.mark.parametrize("name", sorted(INDEX))
def test_oracle_matches_reference_driver_bitwise(name):
    fam, g = load(name)
    m, n, k = INDEX[name]["m"], INDEX[name]["n"], INDEX[name]["k"]
    if fam == "bf16":
        y = sib.reference_bf16_tn(g["a"], g["b"])
    else:
        assert int(g["a_row_stride"][0]) == k + 128          # the driver's padded activation rows
        assert g["a"].abs().max() <= 16 and g["b"].abs().max() <= 16
        y = sib.reference_i8_per_token(g["a"], g["b"], g["sa"], g["sb"], g["bias"])
    assert tuple(y.shape) == (m, n)
    assert torch.equal(y.view(torch.int16), g["reference"].view(torch.int16)), name


def test_i8_oracle_is_exact_beyond_fp32_integers():
    # sums past 2^24 are formed exactly and rounded once
    a = torch.full((1, 4096), 127, dtype=torch.int8)
    b = torch.full((2, 4096), 127, dtype=torch.int8)
    b[1] = -128
    exact = sib.exact_i8_sum(a, b)
    assert exact[0, 0].item() == 127 * 127 * 4096 and exact[0, 1].item() == -127 * 128 * 4096
    one = torch.ones(1)
    y = sib.reference_i8_per_token(a, b, one, torch.ones(2))
    assert y.float()[0, 0].item() == torch.tensor(float(127 * 127 * 4096)).bfloat16().float().item()
