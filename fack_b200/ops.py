"""PyTorch operator surface of the B200 FP8 block-scaled GEMM.

Two layers:

* the aiter-compatible entry points a user of the reference calls, with the
  same names, argument order and meaning:

  - ``gemm_a8w8_blockscale_bpreshuffle_asm(a, b, out, x_scale, w_scale,
    bias=None, splitK=None, kernelName=None, bpreshuffle=True,
    zero_bias_buf=None)`` -- the low-level operator the reference times
    (client/aiter/hsa/gfx942/driver.py:26-29; signature observed at
    client/aiter/hsa/gfx942/dispatch_driver.py:62-63);
  - ``gemm_a8w8_blockscale_bpreshuffle_ck(x, weight, x_scale, w_scale, out,
    kernelName="")`` -- the CK sibling the reference's op_test tier checks
    the asm operator against (client/aiter/hsa/gfx942/optest_driver.py:79-81);
  - ``gemm_a8w8_blockscale_bpreshuffle(x, weight, x_scale, w_scale,
    dtype=torch.bfloat16)`` -- the public entry that picks the kernel and
    split-K itself and allocates ``out``
    (client/aiter/hsa/gfx942/dispatch_driver.py:72-74);
  - ``shuffle_weight(b, layout=(16, 16))`` -- the weight pre-pack step
    (client/aiter/hsa/gfx942/driver.py:21), here producing this library's own
    tile-blocked, pre-swizzled layout;
  - ``get_config(M, N, K)`` -- the tuned-config lookup stand-in
    (client/aiter/dispatch.py:23-35), returning this library's choice.

  As in aiter, ``x_scale`` for these entry points carries the reference's
  transposed-contiguous bytes: a contiguous ``(M, K/128)`` view whose storage
  is ``K/128``-major (``sa.T.contiguous().view_as(sa)``,
  client/aiter/hsa/gfx942/driver.py:22).  A non-contiguous ``(M, K/128)``
  view with strides ``(1, M)`` (the same bytes) is accepted too.

* ``gemm_blockscale(xq, wq, x_scale, w_scale, out=None, split_k=0)`` -- the
  native entry, which reads ``x_scale`` through its logical strides, so a
  plain row-major ``[M, K/128]`` tensor works as is.

Every entry validates on the host and raises ``ValueError`` for a contract
violation before launching, like the reference driver
(client/aiter/hsa/gfx942/driver.py:11-12).  Split-K slices are combined
through the thread-block cluster's distributed shared memory
(``reduce="global"`` instead uses a workspace cached per (device, stream)).
A single-slice plan with more tiles than SMs runs persistently and takes the
same cached workspace for its tail split (``tail=True``, the default).  A
workspace grows only outside CUDA-graph capture -- during capture a call that
would need a larger one runs its plan unsplit instead -- so every call is
capturable.
"""
from __future__ import annotations

import ctypes
import re
from typing import Optional

import torch

from . import _lib

FP8 = torch.float8_e4m3fn
BLOCK = 128

# gfx942 tile symbols the reference reviews (client/aiter/hsa/gfx942/optest_driver.py:20-24).
# They name AMD code objects; on B200 they are accepted and map to this
# library's own tile choice.
AITER_SYMBOLS = frozenset(
    "_ZN5aiter{}fp8gemm_bf16_blockscale_BpreShuffle_{}x128E".format(43 if t == 128 else 42, t)
    for t in (32, 48, 64, 80, 96, 128))
KERNEL_PREFIX = "fack_bs_sm100"

_workspaces: dict = {}
# workspaces outgrown by a larger plan stay allocated: a CUDA graph captured
# with one of them still launches into it on replay
_retired_workspaces: list = []


def _stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def kernel_name(tile_m: int, tile_n: int, split_k: int) -> str:
    return f"{KERNEL_PREFIX}_t{tile_m}x{tile_n}_s{split_k}"


def parse_kernel_name(name) -> tuple:
    """(tile_m, tile_n, split_k) encoded in one of this library's kernel names,
    else (0, 0, 0).

    The reviewed gfx942 symbols name AMD code objects and carry no tile that
    applies here, so they (and None / "") leave the choice to the library."""
    if not name or name in AITER_SYMBOLS:
        return 0, 0, 0
    m = re.fullmatch(KERNEL_PREFIX + r"_t(16|32|64|128|256)x(16|64|128|224|256)_s([1-8])", str(name))
    small = m is not None and m.group(2) == "16"       # the warp-MMA small-M kernel: 16 tokens, no split
    if not m or (small and (m.group(1) != "16" or m.group(3) != "1")) \
            or (m.group(1) == "256" and int(m.group(3)) > 4) \
            or (not small and int(m.group(1)) < 128 and m.group(2) != "128") \
            or (m.group(2) == "224" and (m.group(1) != "128" or m.group(3) != "1")):
        raise ValueError(f"unknown blockscale kernel {name!r}")
    return int(m.group(1)), int(m.group(2)), int(m.group(3))


def plan(M: int, N: int, K: int, tile_m: int = 0, tile_n: int = 0, split_k: int = 0) -> tuple:
    """(tile_m, tile_n, split_k, workspace_bytes) the library uses; 0 = library choice."""
    lib = _lib.load()
    tm, tn, sk, nb = ctypes.c_int(), ctypes.c_int(), ctypes.c_int(), ctypes.c_size_t()
    _lib.check(lib.fack_gemm_bs_plan(int(M), int(N), int(K), int(tile_m), int(tile_n), int(split_k),
                                     ctypes.byref(tm), ctypes.byref(tn), ctypes.byref(sk), ctypes.byref(nb)),
               "fack_gemm_bs_plan")
    return tm.value, tn.value, sk.value, nb.value


def plan_estimate(M: int, N: int, K: int, tile_m: int, tile_n: int, split_k: int) -> Optional[float]:
    """The planner's cost-model estimate of an explicit plan in SM cycles on
    the current device; None if the model would not offer the plan."""
    lib = _lib.load()
    cyc = ctypes.c_double()
    _lib.check(lib.fack_gemm_bs_plan_estimate(int(M), int(N), int(K), int(tile_m), int(tile_n), int(split_k),
                                              ctypes.byref(cyc)), "fack_gemm_bs_plan_estimate")
    return None if cyc.value >= 1e29 else cyc.value


def get_config(M: int, N: int, K: int, split_k: int = 0) -> dict:
    """Kernel and split-K this library uses for (M, N, K) on the current device."""
    tm, tn, sk, _ = plan(M, N, K, 0, 0, split_k)
    return {"libtype": "asm", "kernelName": kernel_name(tm, tn, sk), "splitK": sk, "tile_m": tm, "tile_n": tn}


def workspace_size(M: int, N: int, K: int, split_k: int = 0, tile_m: int = 0, tile_n: int = 0) -> int:
    """Bytes of split-K workspace for the plan (only used with reduce="global")."""
    return plan(M, N, K, tile_m, tile_n, split_k)[3]


def _workspace(device: torch.device, nbytes: int) -> Optional[torch.Tensor]:
    if nbytes == 0:
        return None
    key = (device.index, _stream_handle(device))
    ws = _workspaces.get(key)
    if ws is None or ws.numel() < nbytes:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError(
                "split-K workspace must grow during CUDA-graph capture; call the operator once "
                "with this shape before capturing")
        if ws is not None:
            _retired_workspaces.append(ws)
        ws = torch.empty(nbytes, dtype=torch.uint8, device=device)
        _workspaces[key] = ws
    return ws


_tail_sizes: dict = {}


def tail_workspace_size(M: int, N: int, K: int, tile_m: int = 0, tile_n: int = 0, split_k: int = 0) -> int:
    """Bytes of the optional workspace that lets a single-slice plan spread its
    last partial round of tiles over all SMs (fack_gemm_bs_tail_workspace_size);
    0 when the plan has no such tail.  Cached per device and shape."""
    key = (torch.cuda.current_device(), M, N, K, tile_m, tile_n, split_k)
    nb = _tail_sizes.get(key)
    if nb is None:
        lib = _lib.load()
        b = ctypes.c_size_t()
        _lib.check(lib.fack_gemm_bs_tail_workspace_size(int(M), int(N), int(K), int(tile_m), int(tile_n),
                                                        int(split_k), ctypes.byref(b)),
                   "fack_gemm_bs_tail_workspace_size")
        nb = _tail_sizes[key] = b.value
    return nb


def _tail_workspace(device: torch.device, nbytes: int) -> Optional[torch.Tensor]:
    """The cached workspace for a tail split, or None (the launch then runs
    unsplit) when it would have to grow during CUDA-graph capture."""
    if nbytes == 0:
        return None
    ws = _workspaces.get((device.index, _stream_handle(device)))
    if torch.cuda.is_current_stream_capturing() and (ws is None or ws.numel() < nbytes):
        return None
    return _workspace(device, nbytes)


def _check_common(xq, wq, w_scale, out, M, N, K):
    for name, t in (("XQ", xq), ("WQ", wq), ("w_scale", w_scale), ("out", out)):
        if not isinstance(t, torch.Tensor) or not t.is_cuda:
            raise ValueError(f"{name} must be a CUDA tensor")
    if xq.dtype != FP8 or wq.dtype != FP8:
        raise ValueError("XQ and WQ must be torch.float8_e4m3fn")
    if w_scale.dtype != torch.float32 or out.dtype != torch.bfloat16:
        raise ValueError("w_scale must be float32 and out bfloat16")
    if M < 1 or N % BLOCK or K % BLOCK or N <= 0 or K <= 0:
        raise ValueError("blockscale GEMM requires positive M and N%128 == K%128 == 0")
    if tuple(wq.shape) != (N, K) or tuple(out.shape) != (M, N):
        raise ValueError(f"shape mismatch: XQ {tuple(xq.shape)}, WQ {tuple(wq.shape)}, out {tuple(out.shape)}")
    if tuple(w_scale.shape) != (N // BLOCK, K // BLOCK) or not w_scale.is_contiguous():
        raise ValueError(f"w_scale must be a contiguous [{N // BLOCK}, {K // BLOCK}] float32 tensor")
    if xq.stride(1) != 1 or wq.stride(1) != 1 or not wq.is_contiguous() or out.stride(1) != 1:
        raise ValueError("XQ, WQ and out must be K-contiguous / row-contiguous")
    devs = {t.device for t in (xq, wq, w_scale, out)}
    if len(devs) != 1:
        raise ValueError("all tensors must be on one device")


def _launch(xq, wq, packed, x_scale, xs_sm, xs_sk, w_scale, out, split_k, tile_m=0, tile_n=0,
            reduce="dsmem", peer_outs=(), xchg=None, tail=True):
    """reduce = "dsmem": split-K slices combine through the cluster's shared
    memory (no workspace, nothing allocated); "global": through a cached
    workspace in global memory.  ``tail``: a single-slice plan whose tiles
    outnumber the SMs gets the cached workspace for its tail split
    (:func:`tail_workspace_size`; grown outside CUDA-graph capture only,
    else the launch runs unsplit).  ``peer_outs``: device addresses (this
    process's mappings of other GPUs' memory) of more copies of ``out``'s
    block, same row stride; every result is stored to each of them too.
    ``xchg`` (with ``peer_outs`` for every other rank, in rank order): the
    exchange state of the fused all-gather (attributes ``rank``, ``world``,
    ``ptr`` and ``peer_ptrs``); the launch then completes only once every
    rank's block has landed in this rank's output (fack_gemm_bs_allgather)."""
    M, K = xq.shape
    N = wq.shape[0]
    dev = xq.device
    lib = _lib.load()
    with torch.cuda.device(dev):
        tm, tn, sk, need = plan(M, N, K, tile_m, tile_n, split_k)
        if sk > 1:
            ws = _workspace(dev, need) if reduce == "global" else None
        else:
            ws = _tail_workspace(dev, tail_workspace_size(M, N, K, tm, tn, sk)) if tail else None
        args = (xq.data_ptr(), xq.stride(0), wq.data_ptr(), _lib.FACK_W_PACKED if packed else _lib.FACK_W_ROW_MAJOR,
                x_scale.data_ptr(), int(xs_sm), int(xs_sk), w_scale.data_ptr(), out.data_ptr(), out.stride(0))
        tail = (M, N, K, tm, tn, sk, _ptr(ws), 0 if ws is None else ws.numel(), _stream_handle(dev))
        if xchg is not None:
            if len(peer_outs) != xchg.world - 1 or len(xchg.peer_ptrs) != xchg.world - 1:
                raise ValueError("the fused all-gather needs one peer output and one peer state per other rank")
            peers = (ctypes.c_void_p * len(peer_outs))(*[int(a) for a in peer_outs])
            pstates = (ctypes.c_void_p * len(xchg.peer_ptrs))(*[int(a) for a in xchg.peer_ptrs])
            st = lib.fack_gemm_bs_allgather(*args, peers, int(xchg.ptr), pstates, int(xchg.rank), int(xchg.world),
                                            *tail)
            what = "fack_gemm_bs_allgather"
        elif peer_outs:
            peers = (ctypes.c_void_p * len(peer_outs))(*[int(a) for a in peer_outs])
            st = lib.fack_gemm_bs_bcast(*args, peers, len(peer_outs), *tail)
            what = "fack_gemm_bs_bcast"
        else:
            st = lib.fack_gemm_bs_ex(*args, *tail)
            what = "fack_gemm_bs_ex"
    _lib.check(st, what)
    return out


def xchg_barrier(xchg, device) -> None:
    """One exchange step alone on the current stream of ``device``
    (fack_xchg_barrier): no rank's next fused all-gather stores into an output
    before every rank's work queued before this point is complete."""
    lib = _lib.load()
    dev = torch.device(device)
    pstates = (ctypes.c_void_p * len(xchg.peer_ptrs))(*[int(a) for a in xchg.peer_ptrs])
    with torch.cuda.device(dev):
        st = lib.fack_xchg_barrier(int(xchg.ptr), pstates, int(xchg.rank), int(xchg.world), _stream_handle(dev))
    _lib.check(st, "fack_xchg_barrier")


def gemm_blockscale(xq: torch.Tensor, wq: torch.Tensor, x_scale: torch.Tensor, w_scale: torch.Tensor,
                    out: Optional[torch.Tensor] = None, split_k: int = 0, tile_n: int = 0, tile_m: int = 0,
                    reduce: str = "dsmem", peer_outs=(), xchg=None, tail: bool = True) -> torch.Tensor:
    """Y = blockscale(XQ, WQ) with x_scale read through its logical strides.

    ``wq`` may be a row-major ``[N, K]`` e4m3 tensor or the output of
    :func:`shuffle_weight` (detected by its ``is_shuffled`` mark).
    ``peer_outs`` (up to 7 device addresses of peer mappings, each the same
    block as ``out`` in another GPU's output, same row stride) makes the
    kernel store every result there too (``fack_gemm_bs_bcast``); with
    ``xchg`` as well (one peer output per other rank, the exchange state of
    :class:`fack_b200.dist.ExchangeState`) the launch also waits, on the
    device, until every rank's block has landed (``fack_gemm_bs_allgather``).
    ``tail=False`` keeps a persistent plan's last partial round of tiles
    unsplit (no workspace).
    """
    if len(peer_outs) > 7:
        raise ValueError("at most 7 peer outputs")
    if xq.dim() != 2 or wq.dim() != 2:
        raise ValueError("XQ and WQ must be 2-D")
    M, K = xq.shape
    N = wq.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=xq.device)
    _check_common(xq, wq, w_scale, out, M, N, K)
    if x_scale.dtype != torch.float32 or not x_scale.is_cuda or tuple(x_scale.shape) != (M, K // BLOCK):
        raise ValueError(f"x_scale must be a float32 CUDA tensor of shape [{M}, {K // BLOCK}]")
    sm, sk = x_scale.stride()
    if K // BLOCK == 1:
        sk = max(sk, 1)
    if M == 1:
        sm = max(sm, 1)
    if reduce not in ("dsmem", "global"):
        raise ValueError("reduce must be 'dsmem' or 'global'")
    return _launch(xq, wq, bool(getattr(wq, "is_shuffled", False)), x_scale, sm, sk, w_scale, out, split_k, tile_m,
                   tile_n, reduce, tuple(peer_outs), xchg, tail)


def _aiter_xscale_strides(x_scale: torch.Tensor, M: int, KB: int):
    """(stride_m, stride_kb) of the reference's transposed-contiguous x_scale."""
    if x_scale.dtype != torch.float32 or not x_scale.is_cuda or tuple(x_scale.shape) != (M, KB):
        raise ValueError(f"x_scale must be a float32 CUDA tensor of shape [{M}, {KB}]")
    if x_scale.is_contiguous() or x_scale.stride() == (1, M):
        # bytes are K/128-major with M contiguous, whatever the view's strides say
        return 1, M
    raise ValueError("x_scale must be the transposed-contiguous view sa.T.contiguous().view_as(sa)")


def gemm_a8w8_blockscale_bpreshuffle_asm(a, b, out, x_scale, w_scale, bias=None, splitK=None, kernelName=None,
                                         bpreshuffle=True, zero_bias_buf=None):
    """Drop-in for aiter's ``gemm_a8w8_blockscale_bpreshuffle_asm`` (writes and returns ``out``).

    ``bias`` must be None: the blockscale operator has no bias term
    (client/aiter/hsa/gfx942/dispatch_driver.py:65-66); ``zero_bias_buf`` is
    accepted and unused.  ``kernelName`` may be None, one of the reviewed
    gfx942 symbols (library choice of tile) or one of this library's names
    ``fack_bs_sm100_t{128|256}x{64|128|256}_s{S}`` (token tile 256 = a CTA
    pair, S <= 4 then; else S <= 8) or ``fack_bs_sm100_t128x224_s1`` (224-wide
    weight tiles, persistent kernel only), which fixes the tiles (and the split,
    unless ``splitK`` is given); ``splitK`` None/0 otherwise lets the library
    choose.  ``bpreshuffle=True`` requires ``b`` from
    :func:`shuffle_weight`.
    """
    if bias is not None:
        raise ValueError("the blockscale operator takes no bias")
    tile_m, tile_n, name_split = parse_kernel_name(kernelName)
    shuffled = bool(getattr(b, "is_shuffled", False))
    if bool(bpreshuffle) != shuffled:
        raise ValueError("bpreshuffle={} but the weight {} a shuffle_weight() output".format(
            bool(bpreshuffle), "is" if shuffled else "is not"))
    if a.dim() != 2 or b.dim() != 2:
        raise ValueError("a and b must be 2-D")
    M, K = a.shape
    N = b.shape[0]
    _check_common(a, b, w_scale, out, M, N, K)
    sm, sk = _aiter_xscale_strides(x_scale, M, K // BLOCK)
    split = name_split if splitK is None else int(splitK)
    return _launch(a, b, shuffled, x_scale, sm, sk, w_scale, out, split, tile_m, tile_n)


def gemm_a8w8_blockscale_bpreshuffle_ck(x, weight, x_scale, w_scale, out, kernelName=""):
    """Drop-in for aiter's CK sibling ``gemm_a8w8_blockscale_bpreshuffle_ck``,
    the independent implementation the reference's op_test tier compares the
    asm operator with (client/aiter/hsa/gfx942/optest_driver.py:79-81).

    Same operands and ``x_scale`` convention as
    :func:`gemm_a8w8_blockscale_bpreshuffle_asm`; writes and returns ``out``;
    no split-K argument.  The weight must be a :func:`shuffle_weight` output
    (the operator is the pre-shuffled one).  ``kernelName`` "" (CK's default
    instance, the one op_test pins) lets the library choose the plan; one of
    this library's ``fack_bs_sm100_...`` names fixes it; CK instance names
    and the gfx942 asm symbols are refused.
    """
    if kernelName and (kernelName in AITER_SYMBOLS or not str(kernelName).startswith(KERNEL_PREFIX)):
        raise ValueError(f"unknown blockscale CK kernel {kernelName!r}")
    if not getattr(weight, "is_shuffled", False):
        raise ValueError("the pre-shuffled CK operator takes a shuffle_weight() output")
    return gemm_a8w8_blockscale_bpreshuffle_asm(x, weight, out, x_scale, w_scale, None, None,
                                                kernelName or None, True)


def gemm_a8w8_blockscale_bpreshuffle(x, weight, x_scale, w_scale, dtype=torch.bfloat16):
    """Drop-in for aiter's public ``gemm_a8w8_blockscale_bpreshuffle``: selects
    the kernel and split-K for (M, N, K), allocates ``out`` and calls the
    low-level operator once (the behaviour pinned by
    unittests/test_aiter_dispatch.py:452-505)."""
    if dtype != torch.bfloat16:
        raise ValueError("only bfloat16 output is supported")
    M, K = x.shape
    N = weight.shape[0]
    cfg = get_config(M, N, K)
    out = torch.empty((M, N), dtype=dtype, device=x.device)
    return gemm_a8w8_blockscale_bpreshuffle_asm(x, weight, out, x_scale, w_scale, None, cfg["splitK"],
                                                cfg["kernelName"], bool(getattr(weight, "is_shuffled", False)))


def quantize_activations(x: torch.Tensor, layout: str = "aiter"):
    """Fused activation quantisation for the GEMM (``fack_quant_act``).

    ``x``: fp32 or bf16 CUDA tensor [M, K], K % 128 == 0, unit stride along K.
    Returns ``(xq, x_scale)``: e4m3 codes [M, K] and fp32 scales, one per token
    per 128-wide K group (scale = amax/240, the benchmark construction).
    ``layout="aiter"`` gives x_scale as the reference's transposed-contiguous
    view (``sa.T.contiguous().view_as(sa)``, client/aiter/hsa/gfx942/driver.py:22),
    ready for :func:`gemm_a8w8_blockscale_bpreshuffle_asm`; ``"logical"`` gives
    a row-major [M, K/128] tensor for :func:`gemm_blockscale`.
    """
    if x.dim() != 2 or not x.is_cuda:
        raise ValueError("x must be a 2-D CUDA tensor")
    if x.dtype not in (torch.float32, torch.bfloat16):
        raise ValueError("x must be float32 or bfloat16")
    if layout not in ("aiter", "logical"):
        raise ValueError("layout must be 'aiter' or 'logical'")
    M, K = x.shape
    if K % BLOCK:
        raise ValueError("K must be a multiple of 128")
    if x.stride(1) != 1:
        raise ValueError("x must be contiguous along K")
    dev = x.device
    xq = torch.empty((M, K), dtype=FP8, device=dev)
    xs = torch.empty((M, K // BLOCK), dtype=torch.float32, device=dev)
    sm, sk = (1, M) if layout == "aiter" else (K // BLOCK, 1)
    lib = _lib.load()
    with torch.cuda.device(dev):
        st = lib.fack_quant_act(x.data_ptr(), _lib.FACK_DTYPE_F32 if x.dtype == torch.float32 else _lib.FACK_DTYPE_BF16,
                                x.stride(0), M, K, xq.data_ptr(), xq.stride(0), xs.data_ptr(), sm, sk,
                                _stream_handle(dev))
    _lib.check(st, "fack_quant_act")
    return xq, xs


def shuffle_weight(b: torch.Tensor, layout=(16, 16)) -> torch.Tensor:
    """Pre-pack a ``[N, K]`` weight into this library's tile layout.

    Stand-in for aiter's ``shuffle_weight(b, layout=(16, 16))``
    (client/aiter/hsa/gfx942/driver.py:21; gemm_driver.py:51, :74 for the
    sibling families).  e4m3, bf16 and int8 weights are accepted: the layout
    is defined on bytes -- 128-row x 128-byte tiles (128 e4m3 / int8 or 64
    bf16 elements of K) in their 128-byte-swizzled shared-memory image -- so
    N % 128 == 0 and K x element size % 128 == 0.  The returned tensor has the
    same shape and dtype and is marked ``is_shuffled = True``.  ``layout`` is
    accepted for signature compatibility; the only supported value is
    ``(16, 16)``.
    """
    if tuple(layout) != (16, 16):
        raise ValueError("only layout=(16, 16) is supported")
    if not isinstance(b, torch.Tensor) or not b.is_cuda or b.dim() != 2 or \
            b.dtype not in (FP8, torch.bfloat16, torch.int8):
        raise ValueError("shuffle_weight needs a 2-D float8_e4m3fn, bfloat16 or int8 CUDA tensor")
    N, K = b.shape
    es = b.element_size()
    if N % BLOCK or (K * es) % BLOCK:
        raise ValueError("shuffle_weight requires N % 128 == 0 and K x element size % 128 == 0")
    if b.stride(1) != 1:
        raise ValueError("weight rows must be contiguous")
    packed = torch.empty((N, K), dtype=b.dtype, device=b.device)
    lib = _lib.load()
    with torch.cuda.device(b.device):
        st = lib.fack_gemm_bs_prepack_w(b.data_ptr(), b.stride(0) * es, None, N, K * es, packed.data_ptr(), None,
                                        _stream_handle(b.device))
    _lib.check(st, "fack_gemm_bs_prepack_w")
    packed.is_shuffled = True
    return packed


def gather_interleave(gathered: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    """out[m, r*ns + c] = gathered[r, m, c] on the GPU (N-sharded output assembly)."""
    if gathered.dim() != 3 or out.dim() != 2 or gathered.dtype != torch.bfloat16 or out.dtype != torch.bfloat16:
        raise ValueError("gathered must be bf16 [g, M, n_shard] and out bf16 [M, g*n_shard]")
    g, M, ns = gathered.shape
    if tuple(out.shape) != (M, g * ns) or not gathered.is_contiguous() or out.stride(1) != 1:
        raise ValueError("gather_interleave shape/layout mismatch")
    lib = _lib.load()
    with torch.cuda.device(out.device):
        st = lib.fack_gather_interleave(gathered.data_ptr(), g, M, ns, out.data_ptr(), out.stride(0),
                                        _stream_handle(out.device))
    _lib.check(st, "fack_gather_interleave")
    return out


def device_status(reset: bool = False) -> int:
    """Error flags set by kernels whose bounded waits expired (0 = none); synchronises."""
    lib = _lib.load()
    flags = ctypes.c_uint()
    st = lib.fack_device_status(_stream_handle(torch.device("cuda", torch.cuda.current_device())),
                                ctypes.byref(flags), 1 if reset else 0)
    if st not in (_lib.FACK_OK, _lib.FACK_ERR_DEVICE_TIMEOUT):
        _lib.check(st, "fack_device_status")
    return flags.value
