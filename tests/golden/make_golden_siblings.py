"""Generate golden vectors for the sibling GEMM families by executing the
reference's own driver, client/aiter/hsa/gfx942/gemm_driver.py (read from the
reference checkout, unmodified), in this container where no GPU and no aiter
exist:

* a stub ``aiter`` package: ``shuffle_weight`` = identity, the two ASM
  operators (``gemm_a16w16_asm``, ``gemm_a8w8_asm``) record their call and do
  nothing -- only the inputs and the driver's references are kept;
* a ``torch`` proxy mapping ``device="cuda"`` to the CPU for the generator and
  the factories the driver calls (Generator, randn, rand, randint, empty,
  zeros); everything else is the real torch.

``prepare()`` then builds its inputs from its seeded generator and computes
its own references (line 50 for BF16, 73 for INT8) on the CPU.  Each
case is saved as ``sib_<name>.npz``: a, b (bf16 as int16 bits / int8), and for
INT8 sa, sb, bias and the padded row stride of a, plus the bf16 reference
bits; ``index_siblings.json`` records the shapes and the driver's SHA-256.

Run from the repository root:
    python tests/golden/make_golden_siblings.py [reference_root]
"""
from __future__ import annotations

import hashlib
import importlib.util
import json
import os
import sys
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
SYMBOLS = {"bf16": "golden_bf16gemm_fp32bf16_tn", "i8": "golden_I8gemm_bf16_perTokenI8_BpreShuffle_tn"}

# (name, family, m, n, k, bpreshuffle, seed); N % 64 (bf16) / % 256 (int8), K % 128 (gemm_driver.py:41-42)
CASES = [
    ("bf16_32x128x256", "bf16", 32, 128, 256, False, 11),
    ("bf16_ragged_33x192x384", "bf16", 33, 192, 384, False, 12),
    ("bf16_256x512x1024_shuffled", "bf16", 256, 512, 1024, True, 13),
    ("i8_32x256x256", "i8", 32, 256, 256, True, 21),
    ("i8_ragged_33x512x640", "i8", 33, 512, 640, True, 22),
    ("i8_160x768x1024", "i8", 160, 768, 1024, True, 23),
]


def _cpu_torch_proxy():
    proxy = types.ModuleType("torch")

    def cpu(fn):
        def call(*a, **kw):
            kw.pop("device", None)
            return fn(*a, **kw)
        return call

    proxy.__getattr__ = lambda name: getattr(torch, name)
    proxy.Generator = lambda device=None: torch.Generator(device="cpu")
    for name in ("randn", "rand", "randint", "empty", "zeros"):
        setattr(proxy, name, cpu(getattr(torch, name)))
    return proxy


def _stub_aiter(calls):
    aiter = types.ModuleType("aiter")
    ops = types.ModuleType("aiter.ops")
    shuffle = types.ModuleType("aiter.ops.shuffle")
    shuffle.shuffle_weight = lambda b, layout=(16, 16): b.clone()
    a16 = types.ModuleType("aiter.ops.gemm_op_a16w16")
    a16.gemm_a16w16_asm = lambda *a, **kw: calls.append(("bf16", a, kw))
    a8 = types.ModuleType("aiter.ops.gemm_op_a8w8")
    a8.gemm_a8w8_asm = lambda *a, **kw: calls.append(("i8", a, kw))
    return {"aiter": aiter, "aiter.ops": ops, "aiter.ops.shuffle": shuffle,
            "aiter.ops.gemm_op_a16w16": a16, "aiter.ops.gemm_op_a8w8": a8}


def run_reference_prepare(ref_root: Path, family, m, n, k, bpreshuffle, seed):
    path = ref_root / "client/aiter/hsa/gfx942/gemm_driver.py"
    spec = importlib.util.spec_from_file_location("fack_reference_gemm_driver", path)
    driver = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(driver)
    calls = []
    mods = _stub_aiter(calls)
    saved = {name: sys.modules.get(name) for name in list(mods) + ["torch"]}
    try:
        sys.modules.update(mods)
        sys.modules["torch"] = _cpu_torch_proxy()
        case = driver.prepare({"family": family, "m": m, "n": n, "k": k, "bpreshuffle": bpreshuffle},
                              SYMBOLS[family], seed)
        case["run"]()
    finally:
        for name, mod in saved.items():
            if mod is None:
                sys.modules.pop(name, None)
            else:
                sys.modules[name] = mod
    assert len(calls) == 1 and calls[0][0] == family, "run() must call its ASM operator once"
    assert calls[0][2].get("splitK") == 1 and calls[0][2].get("kernelName") == SYMBOLS[family]
    return case, hashlib.sha256(path.read_bytes()).hexdigest()


def main(ref_root: Path) -> None:
    index = {}
    for name, family, m, n, k, shuffled, seed in CASES:
        case, sha = run_reference_prepare(ref_root, family, m, n, k, shuffled, seed)
        inp = case["_inputs"]
        ref = case["reference"][0]
        arrays = {"reference": ref.view(torch.int16).numpy(),
                  "mnk": np.array([m, n, k, seed, int(shuffled)], dtype=np.int64)}
        if family == "bf16":
            arrays.update(a=inp["a"].view(torch.int16).numpy(), b=inp["b"].view(torch.int16).numpy())
        else:
            arrays.update(a=inp["a"].contiguous().numpy(), b=inp["b"].numpy(), sa=inp["sa"].numpy(),
                          sb=inp["sb"].numpy(), bias=inp["bias"].numpy(),
                          a_row_stride=np.array([inp["a"].stride(0)], dtype=np.int64))
        np.savez_compressed(HERE / f"sib_{name}.npz", **arrays)
        index[name] = {"family": family, "m": m, "n": n, "k": k, "bpreshuffle": shuffled, "seed": seed,
                       "flops": case["flops"], "driver_sha256": sha}
        print(f"{name}: max|ref| = {ref.float().abs().max().item():.3f}")
    (HERE / "index_siblings.json").write_text(json.dumps(index, indent=2) + "\n")


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("FACK_REFERENCE_ROOT")
    if not root:
        sys.exit(f"usage: python {Path(__file__).name} REFERENCE_ROOT  (or set FACK_REFERENCE_ROOT): "
                 "the reference checkout whose driver generates the vectors")
    main(Path(root))
