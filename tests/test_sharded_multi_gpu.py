"""ridge_gemm_sharded on two real GPUs: each rank computes its N-slab, the
slabs are all-gathered over the NCCL communicator torch.distributed created,
and every rank ends with the full C, equal bit for bit to a one-GPU launch of
the whole GEMM (split-K off, so each output tile is the same arithmetic).
Skipped with fewer than two GPUs."""

import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                                 reason="needs two CUDA GPUs")]

SHAPES = [(512, 1000, 384), (256, 4096, 1024)]


def _worker(rank, world, port, q):
    import torch.distributed as dist
    from datetime import timedelta

    import ridge_b200 as rb
    from ridge_b200.sharded import sharded_gemm
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=timedelta(seconds=60))
    try:
        cfg = rb.TileConfig(128, 256, 64, 4, 4, 8, 0, 1)
        for (M, N, K) in SHAPES:
            a, b = rb.synthetic_inputs(M, N, K, device=dev)
            c_slab, full = sharded_gemm(a, b, cfg, gather=True)
            whole = rb.gemm(a, b, config=cfg)
            torch.cuda.synchronize()
            assert rb.device_error() == 0
            assert torch.equal(full, whole), (rank, M, N, K)
        q.put((rank, "ok"))
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


def test_two_rank_sharded_gemm_gathers_the_whole_c():
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    results = dict(q.get(timeout=5) for _ in procs)
    assert results == {0: "ok", 1: "ok"}, results


def _worker_p2p(rank, world, port, q):
    import torch.distributed as dist
    from datetime import timedelta

    import ridge_b200 as rb
    from ridge_b200.sharded import PeerC, sharded_gemm, sharded_gemm_p2p, slab_bounds
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=timedelta(seconds=60))
    try:
        for cfg in (rb.TileConfig(128, 256, 64, 4, 4, 8), rb.TileConfig(256, 256, 64, 5, 4, 8, 2)):
            for (M, N, K) in SHAPES + [(1000, 1536, 512)]:
                a, b = rb.synthetic_inputs(M, N, K, device=dev)
                n0, ns = slab_bounds(N, world, rank)
                pc = PeerC(M, N)
                pc.local.fill_(float("nan"))
                torch.cuda.synchronize()
                dist.barrier()
                full = sharded_gemm_p2p(a, b[n0:n0 + ns], cfg, pc)
                _, ref = sharded_gemm(a, b, cfg, gather=True)   # NCCL all-gather path
                torch.cuda.synchronize()
                assert rb.device_error() == 0
                assert torch.equal(full, ref), (rank, cfg.tag(), M, N, K)
                pc.close()
        q.put((rank, "ok"))
    except Exception as e:
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


def test_two_rank_fused_p2p_gather_matches_the_nccl_gather():
    """ridge_gemm_sharded_p2p: every rank's epilogue writes its tiles into both
    ranks' C over NVLink; after the completion barrier each rank's C equals the
    NCCL all-gather result bit for bit (same slab GEMMs)."""
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker_p2p, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    results = dict(q.get(timeout=5) for _ in procs)
    assert results == {0: "ok", 1: "ok"}, results


def _worker_p2p_back_to_back(rank, world, port, q):
    import time
    from datetime import timedelta

    import torch.distributed as dist

    import oracle
    import ridge_b200 as rb
    from ridge_b200.sharded import PeerC, sharded_gemm_p2p, slab_bounds
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=timedelta(seconds=60))
    try:
        M, N, K = 768, 2048, 1024
        cfg = rb.TileConfig(256, 256, 64, 6, 4, 8, 2)
        rows = np.array([0, 1, 383, 500, M - 1], np.int64)
        cases = []
        for seed in (3, 4, 5):
            a, b = oracle.unit_inputs(M, N, K, seed=seed)
            n0, ns = slab_bounds(N, world, rank)
            cases.append((torch.from_numpy(a.view(np.float16)).to(dev),
                          torch.from_numpy(np.ascontiguousarray(b[n0:n0 + ns]).view(np.float16)).to(dev),
                          oracle.gemm_f64(a, b, rows=rows)))
        pc = PeerC(M, N)
        torch.cuda.synchronize()
        dist.barrier()
        # Back-to-back calls, no host barrier between them; rank 1 is slow to
        # read each result. The entry barrier keeps rank 0's next call from
        # overwriting rank 1's C before rank 1 has read it.
        for it in range(6):
            a_d, b_d, ref = cases[it % 3]
            full = sharded_gemm_p2p(a_d, b_d, cfg, pc)
            torch.cuda.synchronize()
            if rank == 1:
                time.sleep(0.3)
            got = full.cpu().numpy().view(np.uint16)[rows]
            rel, _m, excess = oracle.fp16_stats(got, ref)
            assert rel <= oracle.REL_FROB_TOL and excess <= oracle.MAX_ABS_EXCESS_TOL, (
                rank, it, rel, excess)
        assert rb.device_error() == 0
        pc.close()
        q.put((rank, "ok"))
    except Exception as e:
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


def test_two_rank_fused_p2p_back_to_back_calls():
    """Consecutive ridge_gemm_sharded_p2p calls with different inputs and no
    host barrier between them, one rank reading each result late: every
    result each rank reads matches the FP64 oracle on sampled rows."""
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker_p2p_back_to_back, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    results = dict(q.get(timeout=5) for _ in procs)
    assert results == {0: "ok", 1: "ok"}, results
