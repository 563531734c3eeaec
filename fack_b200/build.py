"""Build recipe for the in-tree C-ABI library ``fack_b200/libfack_gemm.so``.

The library is compiled straight with nvcc for sm_100a only (B200); there is
no torch extension and no JIT cache, so the built ``.so`` sits beside this
file and travels with the source tree.  ``python -m fack_b200.build`` builds it;
``build(verbose=True)`` prints ptxas register / spill / shared-memory usage.
"""
from __future__ import annotations

import os
import re
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
CSRC = HERE / "csrc"
LIB = HERE / "libfack_gemm.so"
SOURCES = [CSRC / "gemm_bs_sm100.cu", CSRC / "gemm_tn_sm100.cu", CSRC / "quant_act_sm100.cu",
           CSRC / "tuned_table.cpp"]
HEADERS = [CSRC / "sm100_ptx.cuh", CSRC / "tuned_table.h", CSRC / "fack_internal.h", ROOT / "include" / "fack_gemm.h"]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found; the FP8 GEMM library needs CUDA 12.8+ for sm_100a")
    return cand


def needs_build() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    return any(p.stat().st_mtime > t for p in SOURCES + HEADERS)


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile the library if any source is newer than it (or ``force``)."""
    if not force and not needs_build():
        return LIB
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [
        nvcc_path(), *ARCH_FLAGS, "-O3", "-lineinfo", "-std=c++17",
        "-Xcompiler", "-fPIC", "-shared", "--expt-relaxed-constexpr",
        "-I", str(ROOT / "include"), "-Xptxas", "-v",
        *map(str, SOURCES), "-o", str(tmp),
    ]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + res.stdout + res.stderr)
    if verbose:
        sys.stdout.write(res.stdout + res.stderr)
    check_ptxas(res.stdout + res.stderr)
    os.replace(tmp, LIB)
    return LIB


GEMM_LAUNCH_REGS = 168  # the FP8 kernel's setmaxnreg split is sized for this count
GEMM_SPLIT_VARIANTS = 10  # gemm_bs_kernel<64|128|256, single CTA|pair> + gemm_bs_persistent_kernel<64|128|224|256>


def check_ptxas(log: str) -> None:
    """No kernel spills registers, and every variant of the register-split FP8
    kernels (``gemm_bs_kernel``, ``gemm_bs_persistent_kernel``) uses exactly
    GEMM_LAUNCH_REGS registers, which the host also checks before it launches
    one."""
    entry, found = None, 0
    for line in log.splitlines():
        m = re.search(r"Compiling entry function '(\S+)'", line)
        if m:
            entry = m.group(1)
            continue
        if not entry:
            continue
        m = re.search(r"(\d+) bytes spill stores, (\d+) bytes spill loads", line)
        if m and (int(m.group(1)) or int(m.group(2))):
            raise RuntimeError(f"{entry} spills registers: {line.strip()}")
        m = re.search(r"Used (\d+) registers", line)
        if m and ("gemm_bs_kernel" in entry or "gemm_bs_persistent_kernel" in entry):
            found += 1
            if int(m.group(1)) != GEMM_LAUNCH_REGS:
                raise RuntimeError(f"{entry} uses {m.group(1)} registers, expected {GEMM_LAUNCH_REGS}")
    if found != GEMM_SPLIT_VARIANTS:
        raise RuntimeError(f"ptxas report lists {found} register-split kernel variants, expected {GEMM_SPLIT_VARIANTS}")


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
