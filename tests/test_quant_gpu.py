"""GPU parity of the fused activation quantisation (fack_quant_act) against
the oracle's restatement of the benchmark construction: bit-exact codes and
scales, both scale layouts, fp32 and bf16 input, and the end-to-end path
quantise -> GEMM against the fp32 reference."""
import pytest
import torch

import fack_b200 as fb
from fack_b200 import data
from oracle import blockscale as orc

pytestmark = pytest.mark.gpu


def _check(x, layout):
    xq, xs = fb.quantize_activations(x, layout=layout)
    torch.cuda.synchronize()
    rq, rs = orc.quantize_activations_ref(x)
    M, K = x.shape
    if layout == "aiter":  # bytes are K/128-major with M contiguous
        xs = xs.reshape(-1).view(K // 128, M).t()
    assert torch.equal(xs.cpu(), rs), "scales differ"
    assert torch.equal(xq.cpu().view(torch.uint8), rq.view(torch.uint8)), (
        f"{int((xq.cpu().view(torch.uint8) != rq.view(torch.uint8)).sum())} codes differ")


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("M,K", [(1, 128), (33, 640), (256, 7168), (1000, 1024)])
@pytest.mark.parametrize("layout", ["aiter", "logical"])
def test_quant_matches_oracle(cuda_device, dtype, M, K, layout):
    g = torch.Generator().manual_seed(M * 7 + K)
    x = torch.randn((M, K), generator=g)
    x[0, :128] = 0.0                                   # all-zero group -> scale 1
    if M > 2:
        x[1] *= 1e-30                                  # codes deep in the subnormal range
        x[2, ::7] = -0.0                               # signed zeros
    hit = torch.rand((M, K), generator=g) < 1e-3
    x = torch.where(hit, x * 50.0, x)                  # outliers, as in the prefill inputs
    _check(x.to(dtype).to(cuda_device), layout)


def test_quant_strided_rows_and_wide_range(cuda_device):
    g = torch.Generator().manual_seed(3)
    big = torch.randn((64, 2048 + 256), generator=g) * torch.exp2(torch.randint(-20, 20, (64, 1), generator=g).float())
    x = big[:, 128:128 + 2048]                         # row stride 2304 elements
    _check(x.to(cuda_device), "logical")


def test_quant_feeds_gemm(cuda_device):
    """Quantise fp32 activations on the GPU and run the GEMM in the reference's
    call form; compare with the fp32 oracle on the oracle's own quantisation."""
    d = cuda_device
    M, N, K = 200, 1024, 2048
    g = torch.Generator().manual_seed(9)
    x = torch.randn((M, K), generator=g)
    wq, ws = data.make_weights(N, K, "normal", seed=4)
    xq, xs_packed = fb.quantize_activations(x.to(d), layout="aiter")
    out = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=d)
    fb.gemm_a8w8_blockscale_bpreshuffle_asm(xq, fb.shuffle_weight(wq.to(d)), out, xs_packed, ws.to(d), splitK=None)
    torch.cuda.synchronize()
    rq, rs = orc.quantize_activations_ref(x)
    ref = orc.reference_gemm(rq, wq, rs, ws)
    err = (out.float().cpu() - ref.float()).abs()
    assert torch.isfinite(out.float()).all()
    assert bool((err <= 1e-2 + 1e-2 * ref.float().abs()).all())


@pytest.mark.parametrize("s", [1.0, 3.0, 0.7, 1e-3, 5e4])
def test_quant_rounding_midpoints(cuda_device, s):
    """Values that scale onto e4m3 rounding midpoints (and within a few fp32
    ulps of them), and around the subnormal boundary 2^-6: the codes must
    equal the correctly rounded division's, whatever shortcut the kernel takes."""
    mids = []
    for e in range(-6, 8):                        # e4m3 normal binades up to 240
        for mant in range(8):
            lo = (1 + mant / 8) * 2.0 ** e
            mids.append(lo + 2.0 ** e / 16)       # halfway to the next code
    mids = torch.tensor([m for m in mids if m < 240], dtype=torch.float32)
    vals = []
    for k in range(-8, 9):                        # nudge by k fp32 ulps
        vals.append(torch.nextafter(mids, torch.full_like(mids, float("inf") if k > 0 else 0.0)) if k else mids)
        for _ in range(abs(k) - 1):
            vals[-1] = torch.nextafter(vals[-1], torch.full_like(mids, float("inf") if k > 0 else 0.0))
    v = torch.cat(vals + [torch.tensor([2.0 ** -6, 2.0 ** -6 * (1 - 2 ** -20), 2.0 ** -6 * (1 + 2 ** -20),
                                        2.0 ** -7 * 1.5, 2.0 ** -9 * 0.5])])
    n = (v.numel() + 126) // 127 * 127
    v = torch.cat([v, torch.ones(n - v.numel())])
    groups = v.view(-1, 127) * s
    x = torch.cat([torch.full((groups.shape[0], 1), 240.0 * s), groups], dim=1)   # amax pins scale = s
    x = torch.cat([x, -x], dim=0)
    _check(x.to(cuda_device), "logical")
