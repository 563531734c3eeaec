"""Shapes for the persistent-kernel tests: unsplit 128-token plans with more
tiles than a B200 has SMs (so the library runs them persistently), each
weight tile width, ragged M."""
from fack_b200 import data

# name -> (M, N, K, weight tile)
CASES = {
    "t256_ragged": (1000, 8192, 1024, 256),   # 8 x 32 = 256 tiles, last token tile 104 rows
    "t128": (1280, 2560, 768, 128),           # 10 x 20 = 200 tiles
    "t64": (640, 2048, 512, 64),              # 5 x 32 = 160 tiles
    "t256_one_kb": (2048, 4096, 128, 256),    # 16 x 16 = 256 tiles of a single K block
}


def inputs(M, N, K, device):
    xq, xs = data.make_activations(M, K, "outlier", seed=M + 1, device=device)
    wq, ws = data.make_weights(N, K, "uniform_logscale", seed=N + 2, device=device)
    return xq, xs, wq, ws
