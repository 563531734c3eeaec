"""GPU: the persistent kernel (unsplit 128-token plans with more tiles than
SMs: one CTA per SM walks its tiles while two store warps drain the previous
tile) gives the same bits as the one-tile kernel, which a subprocess runs with
FACK_PERSISTENT=0, and agrees with the oracle on sampled rows; every output
element is written (NaN poison)."""
import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

import fack_b200 as fb
from oracle.blockscale import reference_gemm
from _persistent_cases import CASES, inputs
from test_gemm_gpu import assert_close

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


@pytest.mark.parametrize("name", list(CASES))
def test_persistent_matches_one_tile_kernel(cuda_device, one_tile_outputs, name):
    M, N, K, tn = CASES[name]
    assert (M + 127) // 128 * (N // tn) > torch.cuda.get_device_properties(0).multi_processor_count
    xq, xs, wq, ws = inputs(M, N, K, cuda_device)
    out = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=cuda_device)
    fb.gemm_blockscale(xq, fb.shuffle_weight(wq), xs, ws, out=out, tile_n=tn, tile_m=128, split_k=1)
    torch.cuda.synchronize()
    y = out.cpu()
    assert torch.isfinite(y.float()).all(), "unwritten output elements"
    ref = one_tile_outputs[name]
    assert torch.equal(y.view(torch.int16), ref.view(torch.int16)), (
        f"{int((y.view(torch.int16) != ref.view(torch.int16)).sum())} elements differ from the one-tile kernel")
    rows = torch.linspace(0, M - 1, 12).long()
    assert_close(y[rows], reference_gemm(xq[rows.to(cuda_device)].cpu(), wq.cpu(), xs[rows.to(cuda_device)].cpu(),
                                         ws.cpu()), name)
    assert fb.device_status() == 0
