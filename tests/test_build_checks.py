"""CPU: the build's ptxas gate (``fack_b200.build.check_ptxas``) on
synthetic ``-Xptxas -v`` reports: a spill in any kernel, or a register-split
FP8 kernel variant off its launch register count, fails the build."""
import pytest

from fack_b200 import build


def entry(name, regs, spill_st=0, spill_ld=0):
    return (f"ptxas info    : Compiling entry function '{name}' for 'sm_100a'\n"
            f"ptxas info    : Function properties for {name}\n"
            f"    0 bytes stack frame, {spill_st} bytes spill stores, {spill_ld} bytes spill loads\n"
            f"ptxas info    : Used {regs} registers, used 1 barriers, 900 bytes cmem[0]\n")


SPLIT = ([f"_ZN4fack14gemm_bs_kernelILi{bn}ELb{p}EEEv14CUtensorMap_st" for bn in (64, 128, 256) for p in (0, 1)] +
         [f"_ZN4fack25gemm_bs_persistent_kernelILi{bn}EEEv14CUtensorMap_st" for bn in (64, 128, 224, 256)])


def clean():
    log = "".join(entry(n, build.GEMM_LAUNCH_REGS) for n in SPLIT)
    log += entry("_ZN4fack19gemm_bs_swap_kernelILi32EEEv14CUtensorMap_st", 98)
    log += entry("_ZN7fack_tn14gemm_tn_kernelILi1ELi256ELb1EEEv14CUtensorMap_s", 128)
    log += entry("_ZN10fack_quant16quant_act_kernelIfEEvPKT_", 40)
    return log


def test_clean_report_passes():
    build.check_ptxas(clean())


def test_spill_in_any_kernel_fails():
    log = clean() + entry("_ZN7fack_tn14gemm_tn_kernelILi0ELi64ELb0EEEv14CUtensorMap_st", 255, 64, 64)
    with pytest.raises(RuntimeError, match="spills"):
        build.check_ptxas(log)


def test_split_kernel_register_count_and_variant_count():
    bad = clean().replace(f"Used {build.GEMM_LAUNCH_REGS} registers", "Used 160 registers", 1)
    with pytest.raises(RuntimeError, match="expected 168"):
        build.check_ptxas(bad)
    missing = "".join(entry(n, build.GEMM_LAUNCH_REGS) for n in SPLIT[:-1])
    with pytest.raises(RuntimeError, match=f"{len(SPLIT) - 1} register-split kernel variants"):
        build.check_ptxas(missing)
