"""CPU, gloo, world size 2: the N-sharded path's host logic.

Each rank owns a column shard of WQ / w_scale, computes its [M, N/g] block
into its own slot of the gather buffer, the all-gather fills the other slots
and the interleave assembles Y[M, N].  On CPU ranks the local GEMM is the
oracle and the interleave a torch permute (the product path uses the CUDA
kernels; here only the sharding and gather logic is under test).
"""
import os
import socket
import sys
from pathlib import Path

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _oracle_local(xq, wq, x_scale, w_scale, out):
    from oracle.blockscale import reference_gemm
    out.copy_(reference_gemm(xq, wq, x_scale, w_scale))
    return out


def _torch_interleave(gathered, out):
    g, M, ns = gathered.shape
    out.copy_(gathered.permute(1, 0, 2).reshape(M, g * ns))
    return out


def _worker(rank, world, port, M, N, K, result_dir):
    sys.path.insert(0, str(ROOT))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from fack_b200 import data
        from fack_b200.dist import ShardedBlockscaleGemm, shard_weight
        xq, xs, wq, ws = data.make_inputs(data.Workload("dist", M, N, K), seed=4)
        wq_r, ws_r = shard_weight(wq, ws, rank, world)
        gemm = ShardedBlockscaleGemm(local_gemm=_oracle_local, interleave=_torch_interleave)
        y = gemm(xq, wq_r, xs, ws_r)
        y2 = gemm(xq, wq_r, xs, ws_r)  # buffers reused on the second call
        torch.save({"y": y, "y2": y2}, os.path.join(result_dir, f"rank{rank}.pt"))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("M,N,K", [(16, 512, 256), (33, 768, 384)])
def test_sharded_gemm_two_gloo_ranks(tmp_path, M, N, K):
    world = 2
    if N % (128 * world):
        pytest.skip("shape does not shard")
    mp.start_processes(_worker, args=(world, _free_port(), M, N, K, str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    from fack_b200 import data
    from oracle.blockscale import reference_gemm
    from fack_b200.dist import shard_weight
    xq, xs, wq, ws = data.make_inputs(data.Workload("dist", M, N, K), seed=4)
    # the gathered result is exactly the shard results side by side ...
    shards = [reference_gemm(xq, *shard_weight(wq, ws, r, world)[:1], xs, shard_weight(wq, ws, r, world)[1])
              for r in range(world)]
    exact = torch.cat(shards, dim=1)
    # ... and agrees with the unsharded product within the parity tolerance
    full = reference_gemm(xq, wq, xs, ws)
    for r in range(world):
        res = torch.load(tmp_path / f"rank{r}.pt")
        for y in (res["y"], res["y2"]):
            assert torch.equal(y.view(torch.int16), exact.view(torch.int16))
            assert torch.allclose(y.float(), full.float(), rtol=1e-2, atol=1e-2)


def test_shard_bounds_and_weight_slices():
    from fack_b200.dist import shard_bounds, shard_weight
    assert shard_bounds(7168, 8, 0) == (0, 896) and shard_bounds(7168, 8, 7) == (6272, 7168)
    assert shard_bounds(65536, 8, 3) == (24576, 32768)
    with pytest.raises(ValueError):
        shard_bounds(3072, 16, 0)  # 192 columns per rank: not whole 128-column blocks
    with pytest.raises(ValueError):
        shard_bounds(640, 4, 0)   # 160 columns per rank: not whole 128-column blocks
    with pytest.raises(ValueError):
        shard_bounds(1024, 2, 2)
    wq = torch.arange(512 * 256, dtype=torch.float32).reshape(512, 256).to(torch.float8_e4m3fn)
    ws = torch.arange(4 * 2, dtype=torch.float32).reshape(4, 2)
    w1, s1 = shard_weight(wq, ws, 1, 2)
    assert w1.shape == (256, 256) and torch.equal(s1, ws[2:4])
    assert torch.equal(w1.view(torch.uint8), wq[256:512].view(torch.uint8))


# ---------------------------------------------------------------- fused mode --
# The fused path stores each rank's block into every rank's Y through peer
# mappings.  On CPU ranks the "GPU memory" of rank j is a shared-memory tensor
# ys[j]; the fake IPC layer hands out addresses (j + 1) << 40 + byte offset, and
# the fake GEMM resolves them, so the test checks the handle exchange, the
# offset arithmetic and when the real ShardedBlockscaleGemm adds an exchange
# step of its own.  On the GPU each CTA of the launch counts its landed stores
# into the peers' exchange states and CTA 0 waits for the peers' counts; here a
# gloo barrier after the stores stands in for it.

class _FakeIpc:
    """Handles name (rank, buffer id); rank j's buffer b maps to
    ((j + 1) << 40) | (b << 32), the tensor starting at the mapping's base.
    ``ids`` gives the buffer id of a tensor by data_ptr (default 0)."""
    HANDLE_BYTES = 64

    def __init__(self, rank, ids=None):
        self.rank = rank
        self.ids = ids or {}
        self.opened, self.closed = [], []

    def handle(self, t):
        return bytes([self.rank, self.ids.get(t.data_ptr(), 0)]) + bytes(62), 0

    def open(self, handle):
        j = handle[0]
        self.opened.append(j)
        return ((j + 1) << 40) | (handle[1] << 32)

    def close(self, base):
        self.closed.append(base)


def _fused_worker(rank, world, port, M, N, K, ys, alt):
    sys.path.insert(0, str(ROOT))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from fack_b200 import data
        from fack_b200.dist import XCHG_BYTES, ShardedBlockscaleGemm, shard_weight
        from oracle.blockscale import reference_gemm
        xq, xs, wq, ws = data.make_inputs(data.Workload("dist", M, N, K), seed=4)
        wq_r, ws_r = shard_weight(wq, ws, rank, world)
        calls = []

        def local(xq_, wq_, xs_, ws_, out_view, peer_addrs, xchg):
            block = reference_gemm(xq_, wq_, xs_, ws_)
            out_view.copy_(block)
            assert len(peer_addrs) == world - 1 and len(xchg.peer_ptrs) == world - 1
            assert (xchg.rank, xchg.world) == (rank, world) and xchg.tensor.numel() * 8 == XCHG_BYTES
            for a in peer_addrs:
                j, bid = (a >> 40) - 1, (a >> 32) & 0xFF
                assert j != rank and 0 <= j < world
                col = (a & ((1 << 32) - 1)) // 2          # byte offset inside Y_j, row 0
                (ys, alt)[bid][j][:, col:col + block.shape[1]].copy_(block)
            calls.append("gemm")
            dist.barrier()                                # the launch's own completion step

        def barrier(xchg):
            calls.append("barrier")
            dist.barrier()

        ipc = _FakeIpc(rank, ids={alt[rank].data_ptr(): 1})
        gemm = ShardedBlockscaleGemm(mode="fused", ipc=ipc, local_gemm_peers=local, xchg_barrier=barrier)
        outs = [ys[rank], alt[rank]]
        y = gemm(xq, wq_r, xs, ws_r, out=outs[0])
        assert y is outs[0]
        gemm(xq, wq_r, xs, ws_r, out=outs[1])             # alternating outputs: no extra step
        gemm(xq, wq_r, xs, ws_r, out=outs[0])
        gemm(xq, wq_r, xs, ws_r, out=outs[0])             # the same output twice in a row: one extra step
        assert calls == ["gemm", "gemm", "gemm", "barrier", "gemm"], calls
        assert gemm.barriers == 1
        # two outputs + the exchange state, each mapped from every peer once
        assert sorted(ipc.opened) == sorted([j for j in range(world) if j != rank] * 3)
        gemm.close()
        assert len(ipc.closed) == 3 * (world - 1)
    finally:
        dist.destroy_process_group()


def test_fused_mode_two_gloo_ranks():
    world, M, N, K = 2, 33, 768, 384
    ys = [torch.full((M, N), float("nan"), dtype=torch.bfloat16).share_memory_() for _ in range(world)]
    alt = [torch.full((M, N), float("nan"), dtype=torch.bfloat16).share_memory_() for _ in range(world)]
    mp.start_processes(_fused_worker, args=(world, _free_port(), M, N, K, ys, alt), nprocs=world,
                       start_method="spawn", join=True)
    from fack_b200 import data
    from fack_b200.dist import shard_weight
    from oracle.blockscale import reference_gemm
    xq, xs, wq, ws = data.make_inputs(data.Workload("dist", M, N, K), seed=4)
    exact = torch.cat([reference_gemm(xq, *shard_weight(wq, ws, r, world)[:1], xs, shard_weight(wq, ws, r, world)[1])
                       for r in range(world)], dim=1)
    for r in range(world):
        assert torch.equal(ys[r].view(torch.int16), exact.view(torch.int16)), f"rank {r}'s Y"
        assert torch.equal(alt[r].view(torch.int16), exact.view(torch.int16)), f"rank {r}'s second Y"


def test_fused_mode_contract():
    from fack_b200.dist import ShardedBlockscaleGemm
    with pytest.raises(ValueError):
        ShardedBlockscaleGemm.__init__(object.__new__(ShardedBlockscaleGemm), mode="ring")


class _FailingIpc(_FakeIpc):
    """Opens the first peer's handle, then fails (a mapping that cannot be made)."""

    def open(self, handle):
        if self.opened:
            raise RuntimeError("fack_ipc_open_handle: simulated failure")
        return super().open(handle)


def _registry_worker(rank, world, port, case, result_dir):
    sys.path.insert(0, str(ROOT))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from fack_b200.dist import ShardedBlockscaleGemm
        outcome = "ok"
        if case == "layout":
            # rank 1's Y has one row more: the byte offsets would address other elements
            gemm = ShardedBlockscaleGemm(mode="fused", ipc=_FakeIpc(rank))
            try:
                gemm.register(torch.zeros((8 + rank, 256), dtype=torch.bfloat16))
            except ValueError as e:
                outcome = "ValueError" if "layout" in str(e) else repr(e)
            assert gemm.ipc.opened == [] and gemm._mapped == []
        elif case == "open_fails":
            ipc = _FailingIpc(rank)
            gemm = ShardedBlockscaleGemm(mode="fused", ipc=ipc)
            try:
                gemm.register(torch.zeros((8, 384), dtype=torch.bfloat16))
            except RuntimeError:
                outcome = "RuntimeError"
            # the one mapping made before the failure was released, nothing is registered
            assert len(ipc.opened) == 1 and ipc.closed == [(ipc.opened[0] + 1) << 40], (ipc.opened, ipc.closed)
            assert gemm._mapped == [] and gemm._peers == {}
        (Path(result_dir) / f"{case}_{rank}").write_text(outcome)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("case,world,want", [("layout", 2, "ValueError"), ("open_fails", 3, "RuntimeError")])
def test_fused_registration_failures_leave_nothing_mapped(tmp_path, case, world, want):
    mp.start_processes(_registry_worker, args=(world, _free_port(), case, str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    for r in range(world):
        assert (tmp_path / f"{case}_{r}").read_text() == want, f"rank {r}"


def _holder_worker(rank, world, port):
    import gc
    import weakref
    sys.path.insert(0, str(ROOT))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from fack_b200.dist import ShardedBlockscaleGemm
        gemm = ShardedBlockscaleGemm(mode="fused", ipc=_FakeIpc(rank))
        out = torch.zeros((4, 256), dtype=torch.bfloat16)
        ref = weakref.ref(out)
        gemm.register(out)
        del out
        gc.collect()
        assert ref() is not None      # registered: its memory cannot go to another tensor at the same address
        gemm.close()
        gc.collect()
        assert ref() is None
    finally:
        dist.destroy_process_group()


def test_registered_output_is_held_until_close():
    mp.start_processes(_holder_worker, args=(2, _free_port()), nprocs=2, start_method="spawn", join=True)
