"""N-sharded (column-parallel) blockscale GEMM over several GPUs.

The reference runs one GPU per process and has no collective
(client/aiter/docs/validation.md:42-46).  For the wide and prefill layers this
library shards the output columns: rank r owns WQ rows [r*N/g, (r+1)*N/g) and
the matching w_scale rows, the activations are replicated, and each rank
computes its [M, N/g] block with the single-GPU kernel.  Two ways to assemble
the replicated row-major Y[M, N]:

* ``mode="fused"`` (GPUs): the GEMM's own epilogue stores each bf16 tile into
  column block r of every rank's Y through NVLink peer mappings (CUDA IPC),
  so the exchange overlaps the math tile by tile and no separate gather or
  interleave runs.  The launch orders itself against the other ranks on the
  device (``fack_gemm_bs_allgather``): each CTA counts its landed stores into
  every peer's exchange state over NVLink and CTA 0 waits, bounded, for every
  peer's counts, so the call holds no collective and its completion on the
  stream means Y is whole.
* ``mode="nccl"``: the block goes to this rank's slot of a [g, M, N/g] gather
  buffer, an in-place NCCL all-gather fills the other slots, and a
  column-interleave kernel assembles Y (also the gloo path of the CPU tests).

Only the bf16 output crosses NVLink; N/g stays a multiple of 128, so every
shard is made of whole 128x128 weight-scale blocks.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Optional

import torch
import torch.distributed as dist

BLOCK = 128
XCHG_BYTES = 128  # FACK_XCHG_BYTES: one rank's exchange state


@dataclass
class ExchangeState:
    """One rank's exchange state of the fused all-gather: ``ptr`` is this
    rank's FACK_XCHG_BYTES in its own device memory (held by ``tensor``),
    ``peer_ptrs`` every other rank's state mapped here, in rank order."""
    rank: int
    world: int
    ptr: int
    peer_ptrs: list
    tensor: torch.Tensor


def shard_bounds(N: int, world: int, rank: int):
    """Column range [n0, n1) owned by `rank`; N must split into whole 128-blocks."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad rank/world")
    if N % (BLOCK * world):
        raise ValueError(f"N={N} does not split into {world} shards of whole 128-column blocks")
    ns = N // world
    return rank * ns, (rank + 1) * ns


def shard_weight(wq: torch.Tensor, w_scale: torch.Tensor, rank: int, world: int):
    """This rank's (WQ rows, w_scale rows) of a full weight."""
    n0, n1 = shard_bounds(wq.shape[0], world, rank)
    return wq[n0:n1].contiguous(), w_scale[n0 // BLOCK:n1 // BLOCK].contiguous()


def _default_local_gemm(xq, wq, x_scale, w_scale, out):
    from .ops import gemm_blockscale
    return gemm_blockscale(xq, wq, x_scale, w_scale, out=out)


def _default_interleave(gathered, out):
    from .ops import gather_interleave
    return gather_interleave(gathered, out)


def _default_local_gemm_peers(xq, wq, x_scale, w_scale, out, peer_addrs, xchg):
    from .ops import gemm_blockscale
    return gemm_blockscale(xq, wq, x_scale, w_scale, out=out, peer_outs=peer_addrs, xchg=xchg)


def _default_xchg_barrier(xchg):
    from .ops import xchg_barrier
    xchg_barrier(xchg, xchg.tensor.device)


class CudaIpc:
    """Peer mappings through the library's CUDA IPC entry points."""

    HANDLE_BYTES = 64

    def handle(self, t: torch.Tensor) -> tuple:
        from . import _lib
        import ctypes
        lib = _lib.load()
        buf = ctypes.create_string_buffer(self.HANDLE_BYTES)
        off = ctypes.c_size_t()
        _lib.check(lib.fack_ipc_get_handle(t.data_ptr(), buf, self.HANDLE_BYTES, ctypes.byref(off)),
                   "fack_ipc_get_handle")
        return buf.raw, off.value

    def open(self, handle: bytes) -> int:
        from . import _lib
        import ctypes
        lib = _lib.load()
        base = ctypes.c_void_p()
        _lib.check(lib.fack_ipc_open_handle(ctypes.create_string_buffer(handle, len(handle)), ctypes.byref(base)),
                   "fack_ipc_open_handle")
        return int(base.value)

    def close(self, base: int) -> None:
        from . import _lib
        _lib.load().fack_ipc_close_handle(base)


def _layout(t: torch.Tensor) -> tuple:
    """(numel, element size, rows, row stride): what a peer's copy must match
    for the same byte offsets to address the same elements."""
    return (t.numel(), t.element_size(), t.shape[0] if t.dim() else 1, t.stride(0) if t.dim() else 1)


def exchange_peer_addresses(t: torch.Tensor, ipc, group=None) -> list:
    """Collective: every rank publishes (IPC handle, offset, layout) of its
    tensor ``t`` and maps every other rank's.  Returns, for each rank j != this
    rank in rank order, (mapped base, address of j's ``t``).

    Every rank's ``t`` must have the same layout (element count, element size,
    rows, row stride); otherwise every rank raises ``ValueError`` (they all see
    the same records) and nothing stays mapped."""
    world, rank = dist.get_world_size(group), dist.get_rank(group)
    h, off = ipc.handle(t)
    hb = ipc.HANDLE_BYTES
    if len(h) != hb:
        raise ValueError("IPC handle size mismatch")
    tail = [int(off)] + list(_layout(t))
    rec = torch.tensor(list(h) + [b for v in tail for b in int(v).to_bytes(8, "little")], dtype=torch.uint8)
    if dist.get_backend(group) == "nccl":
        rec = rec.to(t.device)
    recs = [torch.empty_like(rec) for _ in range(world)]
    dist.all_gather(recs, rec, group=group)
    raws = [bytes(r.cpu().tolist()) for r in recs]
    fields = [[int.from_bytes(raw[hb + 8 * i:hb + 8 * i + 8], "little") for i in range(len(tail))] for raw in raws]
    if any(f[1:] != fields[0][1:] for f in fields):
        raise ValueError("ranks registered buffers of different layouts (numel, element size, rows, row stride): "
                         + ", ".join(str(tuple(f[1:])) for f in fields))
    peers = []
    try:
        for j, raw in enumerate(raws):
            if j == rank:
                continue
            base = ipc.open(raw[:hb])
            peers.append((base, base + fields[j][0]))
    except BaseException:
        for base, _ in peers:       # release what was mapped before the failure
            ipc.close(base)
        raise
    return peers


class ShardedBlockscaleGemm:
    """Y[M, N] = blockscale(XQ, WQ) with WQ column-sharded over a process group.

    ``mode="nccl"``: ``local_gemm(xq, wq_shard, x_scale, ws_shard, out)`` and
    ``interleave(gathered, out)`` default to this library's CUDA kernels; the
    CPU tests substitute checkers to exercise the sharding and gather logic
    on gloo ranks.

    ``mode="fused"``: ``out`` (row-major [M, N], required) is registered with
    every rank on first use, and so is the exchange state on the first call
    (collectives: all ranks make the same calls in the same order, outside
    CUDA-graph capture).  Each call is one launch,
    ``local_gemm_peers(xq, wq_shard, x_scale, ws_shard, out_block, peer_addrs,
    xchg)``, which stores this rank's block into every rank's ``out`` and
    returns on the stream only once every rank's block has landed here.  A
    peer may store into ``out`` as soon as every rank has finished the
    previous call, so a call whose ``out`` is the previous call's ``out``
    first runs ``xchg_barrier(xchg)`` (one more exchange step: no rank writes
    before every rank's earlier work on its stream is complete).  Alternating
    between two registered outputs needs no such step.
    """

    def __init__(self, group=None, local_gemm: Optional[Callable] = None,
                 interleave: Optional[Callable] = None, mode: str = "nccl", ipc=None,
                 local_gemm_peers: Optional[Callable] = None, xchg_barrier: Optional[Callable] = None):
        if mode not in ("nccl", "fused"):
            raise ValueError("mode must be 'nccl' or 'fused'")
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.mode = mode
        self.local_gemm = local_gemm or _default_local_gemm
        self.local_gemm_peers = local_gemm_peers or _default_local_gemm_peers
        self.xchg_barrier = xchg_barrier or _default_xchg_barrier
        self.interleave = interleave or _default_interleave
        self.ipc = ipc
        self._gather = None
        # (data_ptr, numel) of a registered out -> (that out, peer addresses of
        # the same buffer).  Holding the tensor keeps its memory from being
        # reused by another tensor at the same address while the peers still
        # store into it; close() lets go.
        self._peers: dict = {}
        self._mapped: list = []    # mapped peer bases, released by close()
        self._xchg: Optional[ExchangeState] = None
        self._last_out = None      # key of the previous fused call's out
        self.barriers = 0          # exchange steps run on their own (same out twice in a row)

    def gather_buffer(self, M: int, ns: int, device) -> torch.Tensor:
        g = self._gather
        if g is None or g.shape != (self.world, M, ns) or g.device != torch.device(device):
            if torch.cuda.is_available() and torch.cuda.is_current_stream_capturing():
                raise RuntimeError("gather buffer must be sized before CUDA-graph capture")
            g = torch.empty((self.world, M, ns), dtype=torch.bfloat16, device=device)
            self._gather = g
        return g

    def register(self, out: torch.Tensor) -> list:
        """Peer addresses of ``out`` on the other ranks (collective on first use)."""
        key = (out.data_ptr(), out.numel())
        if key not in self._peers:
            if torch.cuda.is_available() and torch.cuda.is_current_stream_capturing():
                raise RuntimeError("register output buffers before CUDA-graph capture")
            if self.ipc is None:
                self.ipc = CudaIpc()
            pairs = exchange_peer_addresses(out, self.ipc, self.group)
            self._mapped += [base for base, _ in pairs]
            self._peers[key] = (out, [addr for _, addr in pairs])
        return self._peers[key][1]

    def exchange_state(self, device) -> ExchangeState:
        """This rank's exchange state, created and mapped by every rank on
        first use (a collective, outside CUDA-graph capture)."""
        x = self._xchg
        if x is None or x.tensor.device != torch.device(device):
            if x is not None:
                raise RuntimeError("the exchange state lives on one device; use one sharder per device")
            if torch.cuda.is_available() and torch.cuda.is_current_stream_capturing():
                raise RuntimeError("create the exchange state before CUDA-graph capture (call once eagerly)")
            if self.ipc is None:
                self.ipc = CudaIpc()
            t = torch.zeros(XCHG_BYTES // 8, dtype=torch.int64, device=device)
            pairs = exchange_peer_addresses(t, self.ipc, self.group)
            self._mapped += [base for base, _ in pairs]
            x = ExchangeState(self.rank, self.world, t.data_ptr(), [addr for _, addr in pairs], t)
            self._xchg = x
        return x

    def close(self) -> None:
        """Release the peer mappings, the registered outputs and the exchange
        state (before the process group is destroyed)."""
        for base in self._mapped:
            self.ipc.close(base)
        self._mapped, self._peers, self._xchg, self._last_out = [], {}, None, None

    def __call__(self, xq, wq_shard, x_scale, ws_shard, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        M = xq.shape[0]
        ns = wq_shard.shape[0]
        if ns % BLOCK:
            raise ValueError("weight shard must hold whole 128-row blocks")
        if self.mode == "fused":
            if out is None or tuple(out.shape) != (M, self.world * ns) or not out.is_contiguous():
                raise ValueError(f"fused mode needs a contiguous out of shape [{M}, {self.world * ns}]")
            peers = self.register(out)
            xchg = self.exchange_state(out.device)
            col = self.rank * ns
            nbytes = out.element_size() * col                 # byte offset of this rank's column block
            key = (out.data_ptr(), out.numel())
            if key == self._last_out:                         # a peer could overwrite what this rank still reads
                self.xchg_barrier(xchg)
                self.barriers += 1
            self.local_gemm_peers(xq, wq_shard, x_scale, ws_shard, out[:, col:col + ns],
                                  [a + nbytes for a in peers], xchg)
            self._last_out = key
            return out
        gathered = self.gather_buffer(M, ns, xq.device)
        mine = gathered[self.rank]
        self.local_gemm(xq, wq_shard, x_scale, ws_shard, mine)
        if self.world > 1:
            if dist.get_backend(self.group) == "nccl":
                # in place: this rank's input is its own slot of the output
                dist.all_gather_into_tensor(gathered.view(-1), mine.view(-1), group=self.group)
            else:
                dist.all_gather(list(gathered.unbind(0)), mine.clone(), group=self.group)
        if out is None:
            out = torch.empty((M, self.world * ns), dtype=torch.bfloat16, device=xq.device)
        self.interleave(gathered, out)
        return out
