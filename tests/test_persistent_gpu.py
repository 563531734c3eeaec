"""GPU: the persistent kernel (unsplit 128-token plans with more tiles than
SMs: one CTA per SM walks its tiles while two store warps drain the previous
tile).  Without a tail split it gives the same bits as the one-tile kernel,
which a subprocess runs with FACK_PERSISTENT=0.  With the tail split (the last
T mod G tiles cut into K slices, summed by a fix-up launch) every element
agrees with the dequantise-then-matmul reference, the result is bitwise
reproducible, and it differs from the unsplit result only inside the tail
tiles.  Every output element is written (NaN poison)."""
import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

import fack_b200 as fb
from _persistent_cases import CASES, CASES_224, grouped_tile, inputs
from oracle.blockscale import reference_gemm
from test_gemm_gpu import _device_reference, assert_close

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def one_tile_outputs(tmp_path_factory, cuda_device):
    path = tmp_path_factory.mktemp("persist") / "ref.pt"
    env = dict(os.environ, FACK_PERSISTENT="0")
    res = subprocess.run(["timeout", "-k", "10", "300", sys.executable, str(ROOT / "tests" / "_persistent_ref_worker.py"),
                          str(path)], capture_output=True, text=True, cwd=ROOT, env=env)
    assert res.returncode == 0, res.stdout[-2000:] + res.stderr[-3000:]
    return torch.load(path)


def run(case, dev, tail):
    M, N, K, tn = {**CASES, **CASES_224}[case]
    xq, xs, wq, ws = inputs(M, N, K, dev)
    out = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=dev)
    fb.gemm_blockscale(xq, fb.shuffle_weight(wq), xs, ws, out=out, tile_n=tn, tile_m=128, split_k=1, tail=tail)
    torch.cuda.synchronize()
    return out, (xq, xs, wq, ws)


@pytest.mark.parametrize("name", list(CASES))
def test_persistent_matches_one_tile_kernel(cuda_device, one_tile_outputs, name):
    M, N, K, tn = CASES[name]
    assert (M + 127) // 128 * (N // tn) > torch.cuda.get_device_properties(0).multi_processor_count
    out, (xq, xs, wq, ws) = run(name, cuda_device, tail=False)
    y = out.cpu()
    assert torch.isfinite(y.float()).all(), "unwritten output elements"
    ref = one_tile_outputs[name]
    assert torch.equal(y.view(torch.int16), ref.view(torch.int16)), (
        f"{int((y.view(torch.int16) != ref.view(torch.int16)).sum())} elements differ from the one-tile kernel")
    rows = torch.linspace(0, M - 1, 12).long()
    assert_close(y[rows], reference_gemm(xq[rows.to(cuda_device)].cpu(), wq.cpu(), xs[rows.to(cuda_device)].cpu(),
                                         ws.cpu()), name)
    assert fb.device_status() == 0


@pytest.mark.parametrize("name", list(CASES))
def test_tail_split(cuda_device, name):
    M, N, K, tn = CASES[name]
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    m_tiles, n_tiles = (M + 127) // 128, N // tn
    T = m_tiles * n_tiles
    rem = T % sms
    split = min(8, sms // rem if rem else 0, K // 128 // 2)
    nb = fb.tail_workspace_size(M, N, K, 128, tn, 1)
    assert nb == (rem * split * 128 * tn * 4 if split >= 2 else 0), (nb, rem, split)
    y1, (xq, xs, wq, ws) = run(name, cuda_device, tail=True)
    y2, _ = run(name, cuda_device, tail=True)
    assert torch.isfinite(y1.float()).all(), "unwritten output elements"
    assert torch.equal(y1.view(torch.int16), y2.view(torch.int16)), "tail split not bitwise reproducible"
    assert_close(y1, _device_reference(xq, xs, wq, ws), name + " tail split")
    plain, _ = run(name, cuda_device, tail=False)
    diff = (y1.view(torch.int16) != plain.view(torch.int16))
    if nb == 0:
        assert not diff.any()
    else:
        tail_mask = torch.zeros((M, N), dtype=torch.bool, device=cuda_device)
        for lin in range(T - rem, T):
            mt, nt = grouped_tile(lin, n_tiles, m_tiles)
            tail_mask[mt * 128:(mt + 1) * 128, nt * tn:(nt + 1) * tn] = True
        assert not (diff & ~tail_mask).any(), "a tile outside the tail changed with the tail split"
    assert fb.device_status() == 0


@pytest.mark.parametrize("name", list(CASES_224))
@pytest.mark.parametrize("packed", [True, False])
def test_224_wide_tiles(cuda_device, name, packed):
    """The 224-wide weight tile (four per 896 columns), packed weights in 32-row
    boxes and row-major in one box; a thread's 112 columns may take two
    w_scale blocks.  Every element against the fp64 reference, sampled rows
    against the oracle, the tail split bitwise reproducible."""
    M, N, K, tn = CASES_224[name]
    xq, xs, wq, ws = inputs(M, N, K, cuda_device)
    b = fb.shuffle_weight(wq) if packed else wq
    ys = []
    for _ in range(2):
        out = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=cuda_device)
        fb.gemm_blockscale(xq, b, xs, ws, out=out, tile_n=224, tile_m=128, split_k=1)
        torch.cuda.synchronize()
        ys.append(out)
    assert torch.isfinite(ys[0].float()).all(), "unwritten output elements"
    assert torch.equal(ys[0].view(torch.int16), ys[1].view(torch.int16))
    assert_close(ys[0], _device_reference(xq, xs, wq, ws), name + " 224")
    rows = torch.linspace(0, M - 1, 12).long()
    assert_close(ys[0][rows.to(cuda_device)], reference_gemm(xq[rows.to(cuda_device)].cpu(), wq.cpu(),
                                                             xs[rows.to(cuda_device)].cpu(), ws.cpu()), name)
    assert fb.device_status() == 0
