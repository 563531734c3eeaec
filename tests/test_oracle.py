"""CPU: the oracle against the reference's own golden vectors, and the data
construction it is fed."""
import pytest
import torch

from conftest import golden_names, load_golden
from oracle import blockscale as orc
from fack_b200 import data


@pytest.mark.parametrize("name", golden_names())
def test_oracle_matches_reference_driver_bit_exact(name):
    g = load_golden(name)
    y = orc.reference_gemm(g["a"], g["b"], g["sa"], g["sb"])
    assert y.dtype == torch.bfloat16 and y.shape == (g["m"], g["n"])
    assert torch.equal(y.view(torch.int16), g["reference"].view(torch.int16))


@pytest.mark.parametrize("name", golden_names())
def test_packed_xscale_is_transposed_contiguous(name):
    g = load_golden(name)
    # driver.py:22 -- packed_sa = sa.T.contiguous().view_as(sa)
    assert torch.equal(g["packed_sa"], g["sa"].T.contiguous().view_as(g["sa"]))
    assert torch.equal(orc.unpack_aiter_xscale(g["packed_sa"]), g["sa"])
    assert torch.equal(data.to_aiter_xscale(g["sa"]), g["packed_sa"])


@pytest.mark.parametrize("name", golden_names())
def test_golden_inputs_follow_reference_construction(name):
    g = load_golden(name)
    m, n, k = g["m"], g["n"], g["k"]
    assert g["a"].shape == (m, k) and g["b"].shape == (n, k)
    assert g["sa"].shape == (m, k // 128) and g["sb"].shape == (n // 128, k // 128)
    # sa, sb = 0.5 + U[0,1)  (driver.py:16-17)
    for s in (g["sa"], g["sb"]):
        assert float(s.min()) >= 0.5 and float(s.max()) < 1.5


def test_golden_error_is_bf16_rounding():
    g = load_golden("manifest_256x256x1024")
    exact = orc.exact_gemm_f64(g["a"], g["b"], g["sa"], g["sb"])
    err = (g["reference"].double() - exact).abs()
    assert float((err / exact.abs().clamp_min(1.0)).max()) <= 2.0 ** -8


def test_quantizers_codes_exact_in_fnuz_and_bounded():
    gen = torch.Generator().manual_seed(0)
    x = torch.randn(64, 512, generator=gen) * 3
    x[0, :128] = 0.0  # all-zero group -> scale 1, codes 0
    q, s = data.quantize_act(x)
    assert q.dtype == torch.float8_e4m3fn and s.shape == (64, 4)
    qf = q.float()
    assert float(qf.abs().max()) <= 240.0
    assert float(s[0, 0]) == 1.0 and float(qf[0, :128].abs().max()) == 0.0
    # every e4m3fn code with |v| <= 240 survives a round trip through e4m3fnuz
    assert torch.equal(q.to(torch.float8_e4m3fnuz).float(), qf)
    # each group's max code reaches +-240 (scale = amax / 240)
    assert float(qf[1:].reshape(63, 4, 128).abs().amax(dim=2).min()) == 240.0
    w = torch.randn(256, 384, generator=gen) * 0.02
    wq, ws = data.quantize_weight(w)
    assert ws.shape == (2, 3)
    deq = wq.float() * ws.repeat_interleave(128, 0).repeat_interleave(128, 1)
    assert float(((deq - w).abs() / w.abs().max()).max()) < 2 ** -3


def test_workload_shapes_and_accounting():
    wl = data.WORKLOADS["decode"]
    assert (wl.M, wl.N, wl.K) == (256, 3072, 7168)
    # bytes / flops as stated for the benchmark configs
    assert data.algorithmic_bytes(32, 8192, 7168) == pytest.approx(59.50e6, rel=2e-3)
    assert data.algorithmic_bytes(256, 3072, 7168) == pytest.approx(25.49e6, rel=2e-3)
    assert data.algorithmic_bytes(8192, 7168, 16384) == pytest.approx(373.3e6, rel=2e-3)
    assert data.flops(256, 3072, 7168) == 2 * 256 * 3072 * 7168
    assert len(data.SWEEP_M) == 11 and 1 in data.SWEEP_M and 512 in data.SWEEP_M


def test_wide_weights_scales_are_logscale_powers_of_two():
    wq, ws = data.make_weights(256, 1024, "uniform_logscale", seed=3)
    e = torch.log2(ws)
    assert torch.equal(e, e)  # finite
    assert float(e.min()) >= -12.0 and float(e.max()) <= 2.0
    xq, xs = data.make_activations(4, 1024, "constant", seed=3)
    assert torch.all(xq.float() == 240.0) and torch.allclose(xs, torch.full_like(xs, 1 / 240))


def test_small_generated_case_against_float64():
    xq, xs, wq, ws = data.make_inputs(data.Workload("t", 16, 256, 512), seed=5)
    y = orc.reference_gemm(xq, wq, xs, ws).double()
    exact = orc.exact_gemm_f64(xq, wq, xs, ws)
    assert torch.allclose(y, exact, rtol=1e-2, atol=1e-2)


def test_outlier_and_uniform_activation_distributions():
    """Prefill X: N(0,1) with 0.1 % of entries x50; wide-layer X: U(-1, 1).
    Checked on the dequantised values (codes x per-group scale)."""
    xq, xs = data.make_activations(512, 2048, "outlier", seed=5)
    x = xq.float() * xs.repeat_interleave(128, dim=1)
    big = int((x.abs() > 8).sum())              # a plain N(0,1) value beyond 8 has probability ~1e-15
    expected = x.numel() * 1e-3 * 0.873          # P(|50 z| > 8) = P(|z| > 0.16) = 0.873
    assert 0.8 * expected < big < 1.2 * expected, (big, expected)
    assert float(x.abs().max()) > 100            # some outliers reach several sigma x 50
    xq, xs = data.make_activations(64, 2048, "uniform", seed=6)
    x = xq.float() * xs.repeat_interleave(128, dim=1)
    assert float(x.abs().max()) <= 1.0 and abs(float(x.mean())) < 0.02
    assert abs(float((x.abs() < 0.5).float().mean()) - 0.5) < 0.02
