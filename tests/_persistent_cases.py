"""Shapes for the persistent-kernel tests: unsplit 128-token plans with more
tiles than a B200 has SMs (so the library runs them persistently), each
weight tile width, ragged M, and tails that split 2 to 8 ways."""
from fack_b200 import data

# name -> (M, N, K, weight tile); tiles and the tail on 148 SMs in the comments
CASES = {
    "t256_ragged": (1000, 8192, 1024, 256),   # 8 x 32 = 256 tiles (last token tile 104 rows); tail 108: no split
    "t128": (1280, 2560, 768, 128),           # 10 x 20 = 200 tiles; tail 52 tiles split 2 ways
    "t64": (640, 2048, 512, 64),              # 5 x 32 = 160 tiles; tail 12 tiles split 2 ways (K/128 = 4)
    "t256_one_kb": (2048, 4096, 128, 256),    # 16 x 16 = 256 tiles of a single K block: no split
    "t256_tail8": (2000, 7168, 2048, 256),    # 16 x 28 = 448 tiles; tail 4 tiles split 8 ways, ragged rows
}


def inputs(M, N, K, device):
    xq, xs = data.make_activations(M, K, "outlier", seed=M + 1, device=device)
    wq, ws = data.make_weights(N, K, "uniform_logscale", seed=N + 2, device=device)
    return xq, xs, wq, ws


def grouped_tile(lin, n_tiles, m_tiles, group=16):
    """(token tile, weight tile) of tile `lin` in the kernels' grouped launch order."""
    per_group = group * n_tiles
    g = lin // per_group
    first = g * group
    gm = min(group, m_tiles - first)
    r = lin - g * per_group
    return first + r % gm, r // gm

# 224-wide tiles (persistent kernel only): no one-tile kernel to compare bit
# for bit; checked against the fp64 reference and the oracle instead
CASES_224 = {
    "t224_shard": (1024, 896, 2048, 224),      # 8 x 4 = 32 tiles (< SMs): one round; packed rows cross tiles
    "t224_tail": (1280, 3584, 2048, 224),      # 10 x 16 = 160 tiles: tail 12 tiles split 8 ways
    "t224_ragged": (1000, 7168, 1024, 224),    # 8 x 32 = 256 tiles, last token tile 104 rows; tail 108: no split
}
