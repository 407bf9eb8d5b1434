"""Host-side logic of the N-slab mode, on CPU: slab bounds from the C ABI, and
the gather layout (P equal-size slab buffers, all-gathered, then re-laid out
into row-major C) exercised by two `gloo` ranks with CPU matmuls standing in
for the device GEMM."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from ridge_b200.sharded import slab_bounds, slab_width


@pytest.mark.parametrize("N,P", [(16384, 8), (4096, 2), (1000, 3), (300, 4), (8, 8), (0, 2),
                                 (11008, 8), (257, 2)])
def test_slab_bounds_partition_N(N, P):
    covered = []
    per = slab_width(N, P)
    for r in range(P):
        n0, ns = slab_bounds(N, P, r)
        assert 0 <= ns <= per
        if ns:
            assert n0 % 256 == 0          # every slab starts tile-aligned
            covered.extend(range(n0, n0 + ns))
    assert covered == list(range(N))      # disjoint, in order, complete


def test_slab_bounds_rejects_bad_arguments():
    from ridge_b200 import RidgeError
    for args in [(100, 0, 0), (100, 2, 2), (100, 2, -1), (-1, 2, 0)]:
        with pytest.raises(RidgeError):
            slab_bounds(*args)


def _relayout(slabs, M, N, per):
    """Row-major C from P slabs of M x per (what ridge_slabs_to_rowmajor does)."""
    return torch.cat([slabs[r] for r in range(slabs.shape[0])], dim=1)[:, :N]


def _worker(rank, world, port, M, N, K, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    g = torch.Generator().manual_seed(0)
    A = torch.rand((M, K), generator=g, dtype=torch.float64) * 2 - 1
    B = torch.rand((N, K), generator=g, dtype=torch.float64) * 2 - 1   # N x K storage
    n0, ns = slab_bounds(N, world, rank)
    per = slab_width(N, world)
    c_slab = torch.zeros((M, per), dtype=torch.float64)
    c_slab[:, :ns] = A @ B[n0:n0 + ns].T
    slabs = torch.empty((world, M, per), dtype=torch.float64)
    dist.all_gather_into_tensor(slabs.view(-1), c_slab.contiguous().view(-1))
    full = _relayout(slabs, M, N, per)
    err = (full - A @ B.T).abs().max().item()
    dist.destroy_process_group()
    q.put((rank, err))


@pytest.mark.parametrize("N", [1000, 1536])
def test_two_rank_gather_rebuilds_full_C(N):
    world, M, K = 2, 96, 64
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, M, N, K, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    errs = sorted(q.get() for _ in range(world))
    assert all(e < 1e-9 for _, e in errs), errs
