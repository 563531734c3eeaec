"""Generate golden vectors by executing the reference's own blockscale driver.

Runs ``prepare()`` from client/aiter/hsa/gfx942/driver.py (read from the
reference checkout, unmodified) in this container, where no GPU and no aiter
exist, by:

* a stub ``aiter`` package: ``dtypes.fp8`` = ``torch.float8_e4m3fn`` (the
  B200 e4m3 format; randn values are far inside +-240, so every code drawn is
  also exact in the reference's e4m3fnuz), ``shuffle_weight`` = identity and
  the ASM operator = a no-op (only the inputs and the fp32 reference are
  kept);
* a ``torch`` proxy that maps ``device="cuda"`` to the CPU for the
  generator and the tensor factories the driver calls (Generator, randn,
  rand, empty, zeros); everything else is the real torch.

The driver's own line 19-20 then computes the fp32 reference on the CPU.  Each
case is saved as ``<name>.npz`` with the e4m3 bytes of ``a`` and ``b``, the
logical ``sa``, the transposed-contiguous ``packed_sa``, ``sb`` and the bf16
reference bits, plus the SHA-256 of the driver file.

Run from the repository root:  python tests/golden/make_golden.py [reference_root]
"""
from __future__ import annotations

import hashlib
import importlib.util
import json
import os
import sys
import types
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
SYMBOL = "_ZN5aiter42fp8gemm_bf16_blockscale_BpreShuffle_32x128E"

# (name, m, n, k, seed): shapes the reference itself uses, plus edge cases.
CASES = [
    ("manifest_256x256x1024", 256, 256, 1024, 123),   # client/aiter/hsa/gfx942/manifest.json:9, seed default 123
    ("dispatch_192x1280x1024", 192, 1280, 1024, 987),  # unittests/test_aiter_dispatch.py:378-381 (contract shape)
    ("min_1x128x128", 1, 128, 128, 0),                 # smallest legal problem
    ("ragged_33x384x640", 33, 384, 640, 7),            # M off every tile size, odd K/128
]


def _cpu_torch_proxy():
    proxy = types.ModuleType("torch")

    def strip(kw):
        kw = dict(kw)
        kw.pop("device", None)
        return kw

    proxy.__getattr__ = lambda name: getattr(torch, name)  # module-level __getattr__ (PEP 562)
    proxy.Generator = lambda device=None: torch.Generator(device="cpu")
    proxy.randn = lambda *a, **kw: torch.randn(*a, **strip(kw))
    proxy.rand = lambda *a, **kw: torch.rand(*a, **strip(kw))
    proxy.empty = lambda *a, **kw: torch.empty(*a, **strip(kw))
    proxy.zeros = lambda *a, **kw: torch.zeros(*a, **strip(kw))
    return proxy


def _stub_aiter():
    calls = []
    aiter = types.ModuleType("aiter")
    aiter.dtypes = SimpleNamespace(fp8=torch.float8_e4m3fn)
    ops = types.ModuleType("aiter.ops")
    shuffle = types.ModuleType("aiter.ops.shuffle")
    shuffle.shuffle_weight = lambda b, layout=(16, 16): b.clone()
    gemm = types.ModuleType("aiter.ops.gemm_op_a8w8")
    gemm.gemm_a8w8_blockscale_bpreshuffle_asm = lambda *a, **kw: calls.append((a, kw))
    mods = {"aiter": aiter, "aiter.ops": ops, "aiter.ops.shuffle": shuffle, "aiter.ops.gemm_op_a8w8": gemm}
    return mods, calls


def run_reference_prepare(ref_root: Path, m: int, n: int, k: int, seed: int):
    driver_path = ref_root / "client/aiter/hsa/gfx942/driver.py"
    spec = importlib.util.spec_from_file_location("fack_reference_blockscale_driver", driver_path)
    driver = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(driver)
    mods, calls = _stub_aiter()
    saved = {name: sys.modules.get(name) for name in list(mods) + ["torch"]}
    try:
        sys.modules.update(mods)
        sys.modules["torch"] = _cpu_torch_proxy()
        case = driver.prepare({"m": m, "n": n, "k": k}, SYMBOL, seed)
        case["run"]()
    finally:
        for name, mod in saved.items():
            if mod is None:
                sys.modules.pop(name, None)
            else:
                sys.modules[name] = mod
    assert len(calls) == 1, "driver.run() must call the ASM operator exactly once"
    args, kw = calls[0]
    assert kw.get("splitK") == 1 and kw.get("bpreshuffle") is True and kw.get("kernelName") == SYMBOL
    return case, hashlib.sha256(driver_path.read_bytes()).hexdigest()


def main(ref_root: Path) -> None:
    index = {}
    for name, m, n, k, seed in CASES:
        case, sha = run_reference_prepare(ref_root, m, n, k, seed)
        inp = case["_inputs"]
        ref = case["reference"][0]
        np.savez_compressed(
            HERE / f"{name}.npz",
            a=inp["a"].view(torch.uint8).numpy(), b=inp["b"].view(torch.uint8).numpy(),
            sa=inp["sa"].numpy(), packed_sa=inp["packed_sa"].numpy(), sb=inp["sb"].numpy(),
            reference=ref.view(torch.int16).numpy(), mnk=np.array([m, n, k, seed], dtype=np.int64))
        index[name] = {"m": m, "n": n, "k": k, "seed": seed, "flops": case["flops"],
                       "driver_sha256": sha}
        print(f"{name}: max|ref| = {ref.float().abs().max().item():.3f}")
    (HERE / "index.json").write_text(json.dumps(index, indent=2) + "\n")


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("FACK_REFERENCE_ROOT")
    if not root:
        sys.exit(f"usage: python {Path(__file__).name} REFERENCE_ROOT  (or set FACK_REFERENCE_ROOT): "
                 "the reference checkout whose driver generates the vectors")
    main(Path(root))
