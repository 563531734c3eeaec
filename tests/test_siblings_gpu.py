"""GPU parity of the sibling GEMM families (fack_gemm_tn) against the oracle.

INT8: bitwise -- the s32 accumulation is exact and the epilogue rounds
(acc * sa) * sb + bias in fp32 in the reference's order, so every bf16 output
equals the reference driver's.  BF16: within rtol = atol = 1e-2 of the fp32
oracle (the summation order differs).  Outputs are NaN-poisoned first.
"""
import json

import numpy as np
import pytest
import torch

import fack_b200 as fb
from conftest import GOLDEN
from fack_b200 import siblings
from oracle import siblings as sib

pytestmark = pytest.mark.gpu

INDEX = json.loads((GOLDEN / "index_siblings.json").read_text())
RTOL = ATOL = 1e-2


def load(name, dev):
    z = np.load(GOLDEN / f"sib_{name}.npz")
    fam = INDEX[name]["family"]
    g = {"fam": fam, "m": INDEX[name]["m"], "n": INDEX[name]["n"], "k": INDEX[name]["k"]}
    if fam == "bf16":
        g["a"] = torch.from_numpy(z["a"]).view(torch.bfloat16).to(dev)
        g["b"] = torch.from_numpy(z["b"]).view(torch.bfloat16).to(dev)
    else:
        k = g["k"]
        # the driver's padded rows: a view of [M, K + 128]
        padded = torch.zeros((g["m"], int(z["a_row_stride"][0])), dtype=torch.int8, device=dev)
        padded[:, :k] = torch.from_numpy(z["a"]).to(dev)
        g["a"] = padded[:, :k]
        for key in ("b", "sa", "sb", "bias"):
            g[key] = torch.from_numpy(z[key]).to(dev)
    g["reference"] = torch.from_numpy(z["reference"]).view(torch.bfloat16)
    return g


def poisoned(M, N, dev):
    return torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=dev)


def check(y, ref, exact, what):
    y = y.cpu()
    assert torch.isfinite(y.float()).all(), f"{what}: unwritten output"
    if exact:
        bad = (y.view(torch.int16) != ref.view(torch.int16))
        assert not bad.any(), f"{what}: {int(bad.sum())} outputs differ from the oracle bitwise"
    else:
        err = (y.float() - ref.float()).abs()
        bad = err > ATOL + RTOL * ref.float().abs()
        assert not bad.any(), f"{what}: {int(bad.sum())} off, max err {float(err.max()):.4g}"


def run_family(g, out, b, **kw):
    if g["fam"] == "bf16":
        return fb.gemm_a16w16_asm(g["a"], b, out, **kw)
    return fb.gemm_a8w8_asm(g["a"], b, g["sa"], g["sb"], out, bias=g["bias"], **kw)


@pytest.mark.parametrize("name", sorted(INDEX))
def test_golden_through_reference_call_form(cuda_device, name):
    """gemm_driver.py:54 / :77 in spirit: splitK=1, a gfx942 symbol, the driver's bpreshuffle."""
    g = load(name, cuda_device)
    shuffled = INDEX[name]["bpreshuffle"]
    b = fb.shuffle_weight(g["b"]) if shuffled else g["b"]
    sym = ("_ZN5aiter35bf16gemm_fp32bf16_tn_48x64_pf3_splitkE" if g["fam"] == "bf16"
           else "_ZN5aiter38I8gemm_bf16_perTokenI8_BpreShuffle_128x128E")
    out = poisoned(g["m"], g["n"], cuda_device)
    r = run_family(g, out, b, splitK=1, kernelName=sym, bpreshuffle=shuffled)
    assert r is out
    check(out, g["reference"], g["fam"] == "i8", name)


@pytest.mark.parametrize("name", sorted(INDEX))
@pytest.mark.parametrize("packed", [False, True])
def test_golden_every_tile_and_split(cuda_device, name, packed):
    g = load(name, cuda_device)
    if packed and g["n"] % 128:
        pytest.skip("the packed layout needs N % 128")
    b = fb.shuffle_weight(g["b"]) if packed else g["b"]
    chunks = g["k"] * (2 if g["fam"] == "bf16" else 1) // 128
    for tile_m in (128, 256):                      # 256 = a CTA pair sharing each MMA
        for tile in (64, 128, 256):
            if g["n"] % tile:
                continue
            for split in range(1, min(8 if tile_m == 128 else 4, chunks) + 1):
                out = poisoned(g["m"], g["n"], cuda_device)
                run_family(g, out, b, splitK=split,
                           kernelName=f"fack_tn_sm100_{g['fam']}_t{tile_m}x{tile}_s{split}", bpreshuffle=packed)
                check(out, g["reference"], g["fam"] == "i8",
                      f"{name} tile={tile_m}x{tile} split={split} packed={packed}")


@pytest.mark.parametrize("m", [1, 96, 256, 300])
def test_i8_decode_shapes_full_range_bitwise(cuda_device, m):
    """Full int8 range (sums past 2^24, rounded once), no bias, library plan."""
    gen = torch.Generator().manual_seed(m)
    N, K = 3072, 7168
    a = torch.randint(-128, 128, (m, K), generator=gen, dtype=torch.int8)
    b = torch.randint(-128, 128, (N, K), generator=gen, dtype=torch.int8)
    sa = 0.001 + 0.01 * torch.rand((m, 1), generator=gen)
    sb = 0.001 + 0.01 * torch.rand((N, 1), generator=gen)
    ref = sib.reference_i8_per_token(a, b, sa, sb)
    d = cuda_device
    out = poisoned(m, N, d)
    fb.gemm_a8w8_asm(a.to(d), fb.shuffle_weight(b.to(d)), sa.to(d), sb.to(d), out)
    check(out, ref, True, f"int8 M={m}")


@pytest.mark.parametrize("m", [1, 256, 1000])
def test_bf16_shapes_vs_oracle(cuda_device, m):
    gen = torch.Generator().manual_seed(m)
    N, K = 3072, 7168
    a = (torch.randn((m, K), generator=gen) * 0.25).bfloat16()
    b = (torch.randn((N, K), generator=gen) * 0.25).bfloat16()
    bias = 0.1 * torch.randn(N, generator=gen)
    ref = sib.reference_bf16_tn(a, b, bias)
    d = cuda_device
    y = fb.gemm_tn(a.to(d), b.to(d), bias=bias.to(d))
    check(y, ref, False, f"bf16 M={m}")
    y2 = fb.gemm_tn(a.to(d), fb.shuffle_weight(b.to(d)), bias=bias.to(d))
    assert torch.equal(y.view(torch.int16), y2.view(torch.int16))   # same plan, same bits


@pytest.mark.parametrize("kind", ["bf16", "i8"])
def test_pairs_on_larger_shapes(cuda_device, kind):
    """CTA-pair plans at 640 x 1536 x 2048 (row tiles off the 256 pair size) against the oracle."""
    d = cuda_device
    gen = torch.Generator().manual_seed(9)
    M, N, K = 640 + 33, 1536, 2048
    if kind == "bf16":
        a = (torch.randn((M, K), generator=gen) * 0.25).bfloat16()
        b = (torch.randn((N, K), generator=gen) * 0.25).bfloat16()
        ref = sib.reference_bf16_tn(a, b)
    else:
        a = torch.randint(-128, 128, (M, K), generator=gen, dtype=torch.int8)
        b = torch.randint(-128, 128, (N, K), generator=gen, dtype=torch.int8)
        sa, sb = 0.001 + 0.01 * torch.rand(M, generator=gen), 0.001 + 0.01 * torch.rand(N, generator=gen)
        ref = sib.reference_i8_per_token(a, b, sa, sb)
    for packed in (False, True):
        bb = fb.shuffle_weight(b.to(d)) if packed else b.to(d)
        for tile, split in ((256, 1), (128, 2), (64, 4), (256, 3)):
            kw = {} if kind == "bf16" else {"a_scale": sa.to(d), "b_scale": sb.to(d)}
            y = fb.gemm_tn(a.to(d), bb, tile_m=256, tile_n=tile, split_k=split, **kw)
            check(y, ref, kind == "i8", f"{kind} pair 256x{tile} split={split} packed={packed}")


def test_split_k_bitwise_reproducible_and_strided_out(cuda_device):
    d = cuda_device
    gen = torch.Generator().manual_seed(5)
    a = (torch.randn((200, 4096), generator=gen) * 0.25).bfloat16().to(d)
    b = (torch.randn((1024, 4096), generator=gen) * 0.25).bfloat16().to(d)
    first = fb.gemm_tn(a, b, split_k=6)
    for _ in range(5):
        assert torch.equal(fb.gemm_tn(a, b, split_k=6).view(torch.int16), first.view(torch.int16))
    big = torch.full((200, 1024 + 64), float("nan"), dtype=torch.bfloat16, device=d)
    view = big[:, 32:32 + 1024]
    fb.gemm_tn(a, b, out=view, split_k=6)
    assert torch.equal(view.view(torch.int16), first.view(torch.int16))
    assert torch.isnan(big[:, :32].float()).all() and torch.isnan(big[:, 32 + 1024:].float()).all()


@pytest.mark.parametrize("name", sorted(INDEX))
def test_public_entries_one_asm_call(cuda_device, name):
    """gemm_a8w8_ASM / gemm_a16w16 (dispatch_driver.py:55-56, :86-87): the
    library's plan, a fresh output, the same bits as the asm-level entry."""
    g = load(name, cuda_device)
    d = cuda_device
    packed = g["n"] % 128 == 0
    b = fb.shuffle_weight(g["b"]) if packed else g["b"]
    want = poisoned(g["m"], g["n"], d)
    if g["fam"] == "bf16":
        y = fb.gemm_a16w16(g["a"], b, bias=None, otype=torch.bfloat16)
        fb.gemm_a16w16_asm(g["a"], b, want, bpreshuffle=packed)
    else:
        y = fb.gemm_a8w8_ASM(g["a"], b, g["sa"], g["sb"], bias=g["bias"], dtype=torch.bfloat16)
        fb.gemm_a8w8_asm(g["a"], b, g["sa"], g["sb"], want, bias=g["bias"], bpreshuffle=packed)
    assert y.shape == (g["m"], g["n"]) and y.dtype == torch.bfloat16
    check(y, g["reference"], g["fam"] == "i8", name + " public")
    assert torch.equal(y.view(torch.int16), want.view(torch.int16))


@pytest.mark.parametrize("public,asm,dtype", [("gemm_a8w8_ASM", "gemm_a8w8_asm", torch.int8),
                                              ("gemm_a16w16", "gemm_a16w16_asm", torch.bfloat16)])
def test_public_entry_makes_exactly_one_asm_call(cuda_device, monkeypatch, public, asm, dtype):
    """The reference's dispatch check (dispatch_driver.py:43-99) patches the
    asm-level operator in the module the public entry resolves it from and
    requires exactly one call with the configured kernelName and splitK; here
    that module is fack_b200.siblings."""
    d = cuda_device
    M, N, K = 48, 512, 1024
    g = torch.Generator().manual_seed(3)
    if dtype == torch.int8:
        a = torch.randint(-8, 9, (M, K), generator=g, dtype=torch.int8).to(d)
        b = torch.randint(-8, 9, (N, K), generator=g, dtype=torch.int8).to(d)
    else:
        a = (0.1 * torch.randn((M, K), generator=g)).to(torch.bfloat16).to(d)
        b = (0.1 * torch.randn((N, K), generator=g)).to(torch.bfloat16).to(d)
    b = fb.shuffle_weight(b)
    real = getattr(siblings, asm)
    seen = []

    def spy(*args, **kw):
        seen.append(kw)
        return real(*args, **kw)
    monkeypatch.setattr(siblings, asm, spy)
    if dtype == torch.int8:
        sa, sb = torch.ones((M, 1), device=d), torch.ones((N, 1), device=d)
        y = getattr(fb, public)(a, b, sa, sb, bias=None, dtype=torch.bfloat16)
    else:
        y = getattr(fb, public)(a, b, bias=None, otype=torch.bfloat16)
    cfg = siblings.get_config(siblings.KINDS[dtype], M, N, K)
    assert len(seen) == 1, f"{public} made {len(seen)} calls of {asm}"
    assert seen[0]["kernelName"] == cfg["kernelName"] and seen[0]["splitK"] == cfg["splitK"]
    assert y.shape == (M, N) and torch.isfinite(y.float()).all()


def test_public_config_and_contract_errors(cuda_device):
    cfg = siblings.get_config(siblings.KINDS[torch.int8], 256, 3072, 7168)
    assert cfg["kernelName"].startswith("fack_tn_sm100_i8_t") and cfg["splitK"] >= 1
    d = cuda_device
    a = torch.zeros((4, 256), dtype=torch.int8, device=d)
    b = torch.zeros((256, 256), dtype=torch.int8, device=d)
    s4, s256 = torch.ones((4, 1), device=d), torch.ones((256, 1), device=d)
    out = torch.empty((4, 256), dtype=torch.bfloat16, device=d)
    with pytest.raises(ValueError):
        fb.gemm_a8w8_asm(a, b, s4, s256, out)                       # bpreshuffle=True but b is row-major
    with pytest.raises(ValueError):
        fb.gemm_a8w8_asm(a, b, s256, s256, out, bpreshuffle=False)  # sa has the wrong length
    with pytest.raises(ValueError):
        fb.gemm_a8w8_asm(a, b, s4, s256, out, bpreshuffle=False, kernelName="fack_tn_sm100_bf16_t128x64_s1")
    y = fb.gemm_a8w8_asm(a, b, s4, s256, out, bpreshuffle=False)
    assert (y.float() == 0).all()
