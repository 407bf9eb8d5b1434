"""Device side of the N-slab mode on one GPU: the slab re-layout kernel against
torch concatenation (bit-exact: it only moves bytes), and a slab GEMM
reproducing the matching columns of the whole GEMM."""

import numpy as np
import pytest

import oracle

torch = pytest.importorskip("torch")
pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")]


@pytest.mark.parametrize("M,N,P,ldc_pad,offset", [(64, 1000, 3, 0, 0), (128, 2048, 8, 8, 0),
                                                  (7, 257, 2, 3, 1), (1, 8, 8, 0, 0)])
def test_slabs_to_rowmajor_bit_exact(M, N, P, ldc_pad, offset):
    from ridge_b200.sharded import slab_width, slabs_to_rowmajor
    per = slab_width(N, P)
    slabs = torch.randn((P, M, per), device="cuda").half()
    ldc = N + ldc_pad
    buf = torch.full((M * ldc + offset,), float("nan"), dtype=torch.float16, device="cuda")
    C = buf[offset:].view(M, ldc)
    slabs_to_rowmajor(slabs, C, M, N, P, per)
    torch.cuda.synchronize()
    want = torch.cat([slabs[r] for r in range(P)], dim=1)[:, :N]
    assert torch.equal(C[:, :N], want)
    if ldc_pad:
        assert torch.isnan(C[:, N:]).all()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_slab_gemms_assemble_the_full_gemm(world):
    """Every rank's slab (simulated on one GPU) equals the matching columns of
    the whole GEMM, and the re-laid-out gather equals the whole C."""
    import ridge_b200 as rb
    from ridge_b200.sharded import slab_bounds, slab_gemm, slab_width, slabs_to_rowmajor
    M, N, K = 256, 1536, 512
    a, b = oracle.unit_inputs(M, N, K, seed=2)
    ad = torch.from_numpy(a.view(np.float16)).cuda()
    bd = torch.from_numpy(b.view(np.float16)).cuda()
    cfg = rb.TileConfig(128, 256, 64, 4, 4, 8)
    whole = rb.gemm(ad, bd, config=cfg)
    per = slab_width(N, world)
    slabs = torch.zeros((world, M, per), dtype=torch.float16, device="cuda")
    for r in range(world):
        n0, ns = slab_bounds(N, world, r)
        if ns:
            slab_gemm(ad, bd[n0:n0 + ns], slabs[r], cfg)
    full = torch.empty((M, N), dtype=torch.float16, device="cuda")
    slabs_to_rowmajor(slabs, full, M, N, world, per)
    torch.cuda.synchronize()
    ref = oracle.gemm_f64(a, b)
    rel, _, excess = oracle.fp16_stats(full.cpu().numpy().view(np.uint16), ref)
    assert rel <= oracle.REL_FROB_TOL and excess <= oracle.MAX_ABS_EXCESS_TOL
    assert torch.equal(full, whole)  # same tile config, same per-element arithmetic


def test_sharded_gemm_single_rank_gather():
    import ridge_b200 as rb
    from ridge_b200.sharded import sharded_gemm
    M, N, K = 200, 640, 256
    a, b = rb.synthetic_inputs(M, N, K)
    cfg = rb.TileConfig(128, 128, 64, 4, 4, 8)
    c_slab, full = sharded_gemm(a, b, cfg, gather=True, rank=0, world=1)
    torch.cuda.synchronize()
    assert torch.equal(full, rb.gemm(a, b, config=cfg))
