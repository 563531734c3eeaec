"""GPU: exact-shape rows of the tuned table drive the automatic plan, and the
plans the shipped table selects match the oracle (rtol = atol = 1e-2)."""
import csv
import ctypes

import pytest
import torch

import fack_b200 as fb
from fack_b200 import _lib, data
from oracle import blockscale as orc
from test_gemm_gpu import assert_close

pytestmark = pytest.mark.gpu


@pytest.fixture()
def fresh_table():
    lib = _lib.load()
    lib.fack_gemm_bs_tuned_clear()
    yield lib
    lib.fack_gemm_bs_tuned_clear()
    for table in _lib.tuned_tables():
        _lib.load_tuned(table, lib)


def run_public(M, N, K, seed, dev):
    xq, xs = data.make_activations(M, K, "normal", seed)
    wq, ws = data.make_weights(N, K, "normal", seed + 1)
    ref = orc.reference_gemm(xq, wq, xs, ws)
    y = fb.gemm_a8w8_blockscale_bpreshuffle(xq.to(dev), fb.shuffle_weight(wq.to(dev)),
                                            data.to_aiter_xscale(xs).to(dev), ws.to(dev))
    return y, ref


def test_row_overrides_the_cost_model(cuda_device, fresh_table):
    lib = fresh_table
    cu = torch.cuda.get_device_properties(0).multi_processor_count
    M, N, K = 33, 384, 640
    model = fb.get_config(M, N, K)
    model_next = fb.get_config(M + 1, N, K)
    row = (256, 128, 2) if model["kernelName"] != "fack_bs_sm100_t256x128_s2" else (128, 64, 3)
    assert lib.fack_gemm_bs_tuned_set(cu, M, N, K, *row) == 0
    cfg = fb.get_config(M, N, K)
    assert (cfg["tile_m"], cfg["tile_n"], cfg["splitK"]) == row
    assert fb.get_config(M + 1, N, K) == model_next     # exact shapes only: M + 1 keeps the model's plan
    y, ref = run_public(M, N, K, 7, cuda_device)
    assert_close(y, ref, f"override {row}")
    # the C ABI's own automatic path (split_k = 0) takes the row too
    tn, sk = ctypes.c_int(), ctypes.c_int()
    assert lib.fack_gemm_bs_select(M, N, K, 0, ctypes.byref(tn), ctypes.byref(sk)) == 0
    assert (tn.value, sk.value) == row[1:]
    # an explicit split bypasses the table
    assert fb.get_config(M, N, K, split_k=1)["splitK"] == 1


def shipped_rows():
    if not _lib.TUNED_TABLE.exists():
        return []
    lines = [ln for ln in _lib.TUNED_TABLE.read_text().splitlines() if not ln.startswith("#")]
    return sorted(csv.DictReader(lines), key=lambda r: int(r["M"]) * int(r["N"]) * int(r["K"]))


@pytest.mark.parametrize("row", shipped_rows(), ids=lambda r: f"{r['M']}x{r['N']}x{r['K']}")
def test_shipped_rows_select_their_plan_and_match_oracle(cuda_device, row):
    """Every shipped row: the public entry takes the row's plan at the row's
    shape; its whole output agrees with the dequantise-then-matmul on the
    device and up to 24 evenly spaced rows with the CPU oracle."""
    from test_gemm_gpu import _device_reference
    M, N, K = int(row["M"]), int(row["N"]), int(row["K"])
    cu = torch.cuda.get_device_properties(0).multi_processor_count
    if int(row["cu_num"]) != cu:
        pytest.skip(f"row is for {row['cu_num']} SMs, device has {cu}")
    assert fb.get_config(M, N, K)["kernelName"] == row["kernelName"]
    d = cuda_device
    xq, xs = data.make_activations(M, K, "normal", 40 + M, device=d)
    wq, ws = data.make_weights(N, K, "normal", 41 + M, device=d)
    y = fb.gemm_a8w8_blockscale_bpreshuffle(xq, fb.shuffle_weight(wq), data.to_aiter_xscale(xs), ws)
    assert_close(y, _device_reference(xq, xs, wq, ws), row["kernelName"] + " (device reference)")
    rows = torch.linspace(0, M - 1, min(M, 24)).long().unique()
    ref = orc.reference_gemm(xq[rows.to(d)].cpu(), wq.cpu(), xs[rows.to(d)].cpu(), ws.cpu())
    assert_close(y[rows.to(d)], ref, row["kernelName"] + " (oracle rows)")
