"""ridge_gemm_host: the end-to-end GEMM on host buffers, its copies pipelined
against the kernel by M-panels. Checked bit for bit against the device entry
point on the same data with split-K off (each panel then runs exactly the
tiles the whole launch runs), against the FP64 oracle, and on the cases the
pipeline adds: ragged panels, host pitches that are not multiples of 8,
pageable host memory, K = 0, buffer growth between calls, back-to-back calls."""

import numpy as np
import pytest

import oracle

torch = pytest.importorskip("torch")
pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")]


def _inputs(M, N, K, seed, pinned=True):
    a, b = oracle.unit_inputs(M, N, K, seed=seed)
    ah = torch.from_numpy(a.view(np.float16).copy())
    bh = torch.from_numpy(b.view(np.float16).copy())
    if pinned:
        ah, bh = ah.pin_memory(), bh.pin_memory()
    return a, b, ah, bh


def _device_ref(rb, ah, bh, cfg):
    c = rb.gemm(ah.cuda(), bh.cuda(), config=cfg)
    torch.cuda.synchronize()
    return c.cpu()


CASES = [
    # shape, config (split_k = 1: bit-exact against the unpanelled launch), panels
    ((1000, 777, 520), (128, 128, 64, 4, 4, 8, 0, 1), 0),
    ((2048, 1024, 1024), (256, 256, 64, 5, 4, 8, 2, 1), 4),
    ((2048, 1024, 1024), (256, 256, 64, 5, 4, 8, 2, 1), 1),
    ((513, 640, 96), (64, 128, 32, 3, 4, 8, 0, 1), 3),
    ((100, 256, 256), (128, 256, 64, 4, 4, 8, 0, 1), 8),
]


@pytest.mark.parametrize("shape,c,panels", CASES, ids=lambda x: str(x))
def test_host_gemm_matches_device_launch(shape, c, panels):
    import ridge_b200 as rb
    M, N, K = shape
    cfg = rb.TileConfig(*c)
    a, b, ah, bh = _inputs(M, N, K, seed=31)
    out = torch.full((M, N), float("nan"), dtype=torch.float16).pin_memory()
    rb.gemm_host(ah, bh, out, config=cfg, panels=panels)
    torch.cuda.synchronize()
    assert rb.device_error() == 0
    ref = _device_ref(rb, ah, bh, cfg)
    assert torch.equal(out, ref)
    ref64 = oracle.gemm_f64(a, b)
    rel, _mx, excess = oracle.fp16_stats(out.numpy().view(np.uint16), ref64)
    assert rel <= oracle.REL_FROB_TOL and excess <= oracle.MAX_ABS_EXCESS_TOL, (rel, excess)


def test_host_gemm_odd_pitches_pageable_and_split_k():
    """Host pitches that TMA could not take (not multiples of 8) are packed on
    the way in; pageable buffers work; a split-K config agrees with the oracle."""
    import ridge_b200 as rb
    M, N, K = 700, 333, 1029
    a, b = oracle.unit_inputs(M, N, K, seed=5)
    lda, ldb, ldc = K + 3, K + 1, N + 5
    ah = torch.zeros((M, lda), dtype=torch.float16)
    bh = torch.zeros((N, ldb), dtype=torch.float16)
    ah[:, :K] = torch.from_numpy(a.view(np.float16).reshape(M, K))
    bh[:, :K] = torch.from_numpy(b.view(np.float16).reshape(N, K))
    out = torch.full((M, ldc), float("nan"), dtype=torch.float16)
    cfg = rb.TileConfig(128, 128, 64, 4, 4, 8)
    rb.gemm_host(ah[:, :K], bh[:, :K], out[:, :N], config=cfg)
    torch.cuda.synchronize()
    assert rb.device_error() == 0
    assert torch.isnan(out[:, N:]).all()          # columns past N untouched
    ref64 = oracle.gemm_f64(a, b)
    got = out[:, :N].contiguous().numpy().view(np.uint16)
    rel, _mx, excess = oracle.fp16_stats(got, ref64)
    assert rel <= oracle.REL_FROB_TOL and excess <= oracle.MAX_ABS_EXCESS_TOL, (rel, excess)


def test_host_gemm_k0_growth_and_back_to_back():
    import ridge_b200 as rb
    cfg = rb.TileConfig(128, 128, 64, 4, 4, 8, 0, 1)
    # K = 0: C is zero
    ah = torch.empty((300, 0), dtype=torch.float16)
    bh = torch.empty((200, 0), dtype=torch.float16)
    out = torch.full((300, 200), float("nan"), dtype=torch.float16)
    rb.gemm_host(ah, bh, out, config=cfg)
    torch.cuda.synchronize()
    assert (out == 0).all()
    # a small call, then a larger one (buffers grow), then two queued back to
    # back without a synchronise in between
    outs, refs = [], []
    for (M, N, K, seed) in ((128, 128, 64, 1), (1536, 1024, 768, 2), (1536, 1024, 768, 3),
                            (640, 384, 512, 4)):
        _, _, ah, bh = _inputs(M, N, K, seed)
        o = torch.empty((M, N), dtype=torch.float16).pin_memory()
        rb.gemm_host(ah, bh, o, config=cfg)
        outs.append(o)
        refs.append((ah, bh))
    torch.cuda.synchronize()
    assert rb.device_error() == 0
    for o, (ah, bh) in zip(outs, refs):
        assert torch.equal(o, _device_ref(rb, ah, bh, cfg))


def test_host_gemm_rejects_device_tensors_and_bad_panels():
    import ridge_b200 as rb
    a = torch.zeros((16, 16), dtype=torch.float16, device="cuda")
    with pytest.raises(ValueError):
        rb.gemm_host(a, a)
    h = torch.zeros((16, 16), dtype=torch.float16)
    with pytest.raises(rb.RidgeError):
        rb.gemm_host(h, h, panels=-1)
