"""Subprocess for tests/test_persistent_gpu.py: computes the GEMM with the
persistent kernel switched off (FACK_PERSISTENT=0, read once per process) and
saves the outputs, so the test can compare the two kernels bit for bit."""
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402

import fack_b200 as fb  # noqa: E402
sys.path.insert(0, str(ROOT / "tests"))
from _persistent_cases import CASES, inputs  # noqa: E402


def main(out_path):
    d = torch.device("cuda", 0)
    res = {}
    for name, (M, N, K, tn) in CASES.items():
        xq, xs, wq, ws = inputs(M, N, K, d)
        res[name] = fb.gemm_blockscale(xq, fb.shuffle_weight(wq), xs, ws, tile_n=tn, tile_m=128, split_k=1,
                                       tail=False).cpu()
    torch.save(res, out_path)


if __name__ == "__main__":
    main(sys.argv[1])
