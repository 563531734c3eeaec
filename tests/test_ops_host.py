"""CPU: the aiter-compatible Python entry points refuse bad calls on the host
(ValueError before any launch), as the reference driver does."""
import pytest
import torch

import fack_b200 as fb
from fack_b200 import ops

FP8 = torch.float8_e4m3fn


def cpu_case(M=32, N=256, K=512):
    a = torch.zeros(M, K, dtype=FP8)
    b = torch.zeros(N, K, dtype=FP8)
    out = torch.empty(M, N, dtype=torch.bfloat16)
    xs = torch.ones(M, K // 128)
    ws = torch.ones(N // 128, K // 128)
    return a, b, out, xs, ws


def test_bias_is_rejected():
    a, b, out, xs, ws = cpu_case()
    with pytest.raises(ValueError, match="bias"):
        fb.gemm_a8w8_blockscale_bpreshuffle_asm(a, b, out, xs, ws, bias=torch.zeros(1, 256))


def test_unknown_kernel_rejected_and_aiter_symbols_accepted_by_name():
    a, b, out, xs, ws = cpu_case()
    with pytest.raises(ValueError, match="unknown blockscale kernel"):
        fb.gemm_a8w8_blockscale_bpreshuffle_asm(a, b, out, xs, ws, kernelName="no_such_kernel")
    assert len(fb.AITER_SYMBOLS) == 6
    assert "_ZN5aiter43fp8gemm_bf16_blockscale_BpreShuffle_128x128E" in fb.AITER_SYMBOLS


def test_bpreshuffle_flag_must_match_weight():
    a, b, out, xs, ws = cpu_case()
    with pytest.raises(ValueError, match="bpreshuffle"):
        fb.gemm_a8w8_blockscale_bpreshuffle_asm(a, b, out, xs, ws, bpreshuffle=True)


def test_cpu_tensors_rejected_no_fallback():
    a, b, out, xs, ws = cpu_case()
    with pytest.raises(ValueError, match="CUDA"):
        fb.gemm_a8w8_blockscale_bpreshuffle_asm(a, b, out, xs, ws, bpreshuffle=False)
    with pytest.raises(ValueError, match="CUDA"):
        fb.gemm_blockscale(a, b, xs, ws, out=out)
    with pytest.raises(ValueError):
        fb.shuffle_weight(b)


def test_public_entry_rejects_non_bf16_output():
    a, b, out, xs, ws = cpu_case()
    with pytest.raises(ValueError, match="bfloat16"):
        fb.gemm_a8w8_blockscale_bpreshuffle(a, b, xs, ws, dtype=torch.float16)


def test_kernel_names_are_stable():
    assert ops.kernel_name(128, 256, 6) == "fack_bs_sm100_t128x256_s6"


def test_kernel_name_round_trip():
    assert ops.parse_kernel_name(ops.kernel_name(128, 128, 3)) == (128, 128, 3)
    assert ops.parse_kernel_name(ops.kernel_name(256, 64, 4)) == (256, 64, 4)
    assert ops.parse_kernel_name(None) == (0, 0, 0)
    assert ops.parse_kernel_name("_ZN5aiter42fp8gemm_bf16_blockscale_BpreShuffle_96x128E") == (0, 0, 0)
    assert ops.parse_kernel_name(ops.kernel_name(16, 128, 6)) == (16, 128, 6)   # swapped small-M tile
    for bad in ("fack_bs_sm100_t128x96_s2", "fack_bs_sm100_t128x128_s9", "fack_bs_sm100_t256x128_s6",
                "fack_bs_sm100_t64x256_s1", "fack_bs_sm100_t48x128_s1"):
        with pytest.raises(ValueError):
            ops.parse_kernel_name(bad)


def test_ck_sibling_contract():
    """gemm_a8w8_blockscale_bpreshuffle_ck (optest_driver.py:79-81): CK
    instance names and asm symbols are refused, and the weight must be
    pre-shuffled, before anything launches."""
    a, b, out, xs, ws = cpu_case()
    for bad in ("some_ck_instance", "_ZN5aiter42fp8gemm_bf16_blockscale_BpreShuffle_32x128E"):
        with pytest.raises(ValueError, match="CK kernel"):
            fb.gemm_a8w8_blockscale_bpreshuffle_ck(a, b, xs, ws, out, kernelName=bad)
    with pytest.raises(ValueError, match="shuffle_weight"):
        fb.gemm_a8w8_blockscale_bpreshuffle_ck(a, b, xs, ws, out)


def test_outgrown_workspace_stays_allocated(monkeypatch):
    """A graph captured with the smaller workspace still launches into it on
    replay, so growing the per-(device, stream) workspace keeps the old one."""
    monkeypatch.setattr(ops, "_stream_handle", lambda device: 12345)
    monkeypatch.setattr(torch.cuda, "is_current_stream_capturing", lambda: False)
    monkeypatch.setattr(ops, "_workspaces", {})
    monkeypatch.setattr(ops, "_retired_workspaces", [])
    dev = torch.device("cpu")
    small = ops._workspace(dev, 256)
    assert ops._workspace(dev, 128) is small               # fits: reused
    big = ops._workspace(dev, 4096)
    assert big is not small and big.numel() == 4096
    assert any(w is small for w in ops._retired_workspaces)
    assert ops._workspace(dev, 0) is None


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    """No CPU or library fallback: without libfack_gemm.so every entry raises."""
    from fack_b200 import _lib
    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setattr(_lib, "LIB_PATH", tmp_path / "libfack_gemm.so")
    with pytest.raises(RuntimeError, match="no fallback"):
        _lib.load()
    with pytest.raises(RuntimeError, match="no fallback"):
        fb.get_config(256, 3072, 7168)


def test_public_sibling_entries_refuse_before_any_device_query():
    """gemm_a8w8_ASM / gemm_a16w16 (dispatch_driver.py:55-56, :86-87)."""
    a8, b8 = torch.zeros(4, 256, dtype=torch.int8), torch.zeros(256, 256, dtype=torch.int8)
    s4, s256 = torch.ones(4, 1), torch.ones(256, 1)
    with pytest.raises(ValueError, match="bfloat16 output"):
        fb.gemm_a8w8_ASM(a8, b8, s4, s256, dtype=torch.float16)
    with pytest.raises(ValueError, match="int8 operands"):
        fb.gemm_a8w8_ASM(a8.float(), b8, s4, s256)
    with pytest.raises(ValueError, match="CUDA tensor"):
        fb.gemm_a8w8_ASM(a8, b8, s4, s256)
    abf, bbf = torch.zeros(4, 256, dtype=torch.bfloat16), torch.zeros(256, 256, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="bfloat16 output"):
        fb.gemm_a16w16(abf, bbf, otype=torch.float32)
    with pytest.raises(ValueError, match="bfloat16 operands"):
        fb.gemm_a16w16(a8, bbf)
    with pytest.raises(ValueError, match="CUDA tensor"):
        fb.gemm_a16w16(abf, bbf)


def test_quantize_activations_refuses_before_launch():
    with pytest.raises(ValueError, match="CUDA"):
        fb.quantize_activations(torch.zeros(4, 256))
    with pytest.raises(ValueError, match="2-D"):
        fb.quantize_activations(torch.zeros(256))


def test_case_bench_cli_without_a_device():
    """The ncu case driver parses its arguments and refuses to run without a GPU."""
    import torch
    from fack_b200 import case_bench
    if torch.cuda.is_available():
        return
    assert case_bench.main(["256", "3072", "7168", "--plan", "128,256,5"]) == 2


def test_kernel_names_with_224_wide_tiles():
    """fack_bs_sm100_t128x224_s1 names the persistent 224-wide plan; other
    token tiles or splits with 224 are not plans."""
    from fack_b200 import ops
    assert ops.parse_kernel_name("fack_bs_sm100_t128x224_s1") == (128, 224, 1)
    for bad in ("fack_bs_sm100_t128x224_s2", "fack_bs_sm100_t256x224_s1", "fack_bs_sm100_t64x224_s1"):
        with pytest.raises(ValueError):
            ops.parse_kernel_name(bad)


def test_kernel_names_of_the_small_m_kernel():
    """fack_bs_sm100_t16x16_s1 names the warp-MMA small-M kernel; it has no
    other token tile and no split."""
    from fack_b200 import ops
    assert ops.parse_kernel_name("fack_bs_sm100_t16x16_s1") == (16, 16, 1)
    assert ops.kernel_name(16, 16, 1) == "fack_bs_sm100_t16x16_s1"
    for bad in ("fack_bs_sm100_t32x16_s1", "fack_bs_sm100_t16x16_s2", "fack_bs_sm100_t128x16_s1"):
        with pytest.raises(ValueError):
            ops.parse_kernel_name(bad)
