"""CPU checks of the native library: it loads, exports every function the C
header declares, and its host-side logic (variant table, config validation,
argument checking) behaves -- no kernel launches."""

import ctypes as C
import re
from pathlib import Path

import pytest

import ridge_b200 as rb
from ridge_b200 import TileConfig
from ridge_b200._native import RIDGE_EINVAL, RIDGE_OK, RIDGE_ERANGE, lib

HEADERS = sorted((Path(__file__).resolve().parent.parent / "include").glob("*.h"))


def declared_functions():
    text = re.sub(r"/\*.*?\*/", "", "".join(h.read_text() for h in HEADERS), flags=re.S)
    return sorted(set(re.findall(r"\b(ridge_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_function():
    names = declared_functions()
    assert len(names) >= 10
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, "declared in include/*.h but not exported: %s" % missing


def test_every_declared_function_has_a_python_signature():
    from ridge_b200._native import SIGNATURES
    assert sorted(SIGNATURES) == declared_functions()


def _smem_bytes(bm, bn, bk, s, w, cg):
    """Shared memory one CTA needs: operand ring + epilogue staging + fixed."""
    return 1024 + s * (bm // cg + bn // cg) * bk * 2 + w * 2 * 2048 + 256


def test_variant_table_is_the_valid_grid():
    """BM, BN in {64,128,256} x BK in {32,64} (widened with 128) x stages 2..6 x warps {4,8}, with
    BM=256 both as a 2-CTA pair and as one CTA: every point whose shared memory
    fits in 227 KB is registered, every other point is refused. The four grid
    points whose operand ring alone overflows are among the refused."""
    vs = rb.variants()
    keys = {(v.config.BM, v.config.BN, v.config.BK, v.config.stages, v.config.warps,
             v.config.cta_group) for v in vs}
    assert len(vs) == len(keys)
    expected = set()
    for bm in (64, 128, 256):
        for bn in (64, 128, 256):
            for bk in (32, 64, 128):
                for s in (2, 3, 4, 5, 6):
                    for w in (4, 8):
                        for cg in ((1, 2) if bm == 256 else (1,)):
                            fits = _smem_bytes(bm, bn, bk, s, w, cg) <= 232448
                            assert rb.config_ok(TileConfig(bm, bn, bk, s, w, 8, cg)) == fits
                            if fits:
                                expected.add((bm, bn, bk, s, w, cg))
    assert keys == expected
    for bm, bn, bk, s in [(128, 256, 64, 5), (256, 128, 64, 5), (256, 256, 64, 4),
                          (256, 256, 64, 5)]:
        for w in (4, 8):
            assert (bm, bn, bk, s, w, 1) not in keys
    for v in vs:
        assert v.smem_bytes <= 232448
        assert v.tmem_cols in (64, 128, 256, 512)
        assert v.threads == (2 + v.config.warps) * 32
        assert v.config.groupM == 8
        assert v.cluster_size == v.config.cta_group


@pytest.mark.parametrize("bad", [
    TileConfig(96, 128, 32, 3, 4, 8), TileConfig(128, 128, 48, 3, 4, 8),
    TileConfig(128, 128, 32, 1, 4, 8), TileConfig(128, 128, 32, 9, 4, 8),
    TileConfig(128, 128, 32, 3, 6, 8), TileConfig(128, 128, 32, 3, 4, 0),
])
def test_invalid_configs_rejected(bad):
    assert not rb.config_ok(bad)


def test_variant_index_range():
    v = rb._native.VariantInfoC()
    assert lib.ridge_variant(-1, C.byref(v)) == RIDGE_ERANGE
    assert lib.ridge_variant(rb.num_variants(), C.byref(v)) == RIDGE_ERANGE


def test_shape_validation():
    cfg = TileConfig(128, 128, 32, 3, 4, 8)
    assert rb.valid_for_shape(cfg, 100, 200, 72)            # tails are fine
    assert not rb.valid_for_shape(cfg, 100, 200, 33)        # lda = 33: not 16-byte pitch
    assert rb.valid_for_shape(cfg, 100, 200, 33, lda=40, ldb=40)
    assert not rb.valid_for_shape(cfg, 100, 200, 64, ldc=199)
    assert not rb.valid_for_shape(cfg, -1, 200, 64)
    assert not rb.valid_for_shape(cfg, 1 << 31, 8, 8)


def test_launch_rejects_bad_arguments_before_touching_a_device():
    cfg = TileConfig(128, 128, 32, 3, 4, 8)
    # invalid config / strides / alignment are refused with EINVAL
    assert rb.launch_raw(TileConfig(96, 128, 32, 3, 4, 8), 16, 16, 16, 8, 8, 8, 8, 8, 8) == RIDGE_EINVAL
    assert rb.launch_raw(cfg, 16, 16, 16, 8, 8, 12, 12, 12, 8) == RIDGE_EINVAL
    assert rb.launch_raw(cfg, 8, 16, 16, 8, 8, 8, 8, 8, 8) == RIDGE_EINVAL   # A not 16-byte aligned
    assert rb.launch_raw(cfg, 0, 16, 16, 8, 8, 8, 8, 8, 8) == RIDGE_EINVAL   # null A
    # empty problems are a successful no-op
    assert rb.launch_raw(cfg, 0, 0, 0, 0, 8, 8, 8, 8, 8) == RIDGE_OK
    assert rb.launch_raw(cfg, 0, 0, 0, 8, 0, 8, 8, 8, 8) == RIDGE_OK


def test_status_strings():
    for s in (0, -1, -2, -3, -4, -5):
        assert lib.ridge_status_string(s)


def test_bk128_needs_whole_k_atoms():
    cfg = TileConfig(128, 128, 128, 3, 4, 8)
    assert rb.config_ok(cfg)
    assert rb.valid_for_shape(cfg, 256, 256, 192)
    assert not rb.valid_for_shape(cfg, 256, 256, 200)


def test_gpu_test_configs_are_valid():
    """Every tile config the GPU parity tests launch is a valid config (so a
    typo fails here, on CPU, not on a GPU box)."""
    import importlib.util
    from pathlib import Path
    spec = importlib.util.spec_from_file_location(
        "gemm_gpu_cases", Path(__file__).parent / "test_gemm_gpu.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    for c in mod.CONFIGS + [c for _, c in mod.SPLITK_CASES]:
        assert rb.config_ok(TileConfig(*c)), c


def test_gemm_sharded_validates_before_touching_the_gpu():
    """ridge_gemm_sharded refuses bad ranks and a gather without its buffers or
    communicator up front (no launch, so this runs without a GPU)."""
    import ctypes as C
    from ridge_b200._native import RIDGE_EINVAL, lib
    cfg = rb.TileConfig(128, 128, 64, 4, 4, 8).to_c()
    args = lambda nranks, rank, gather, comm: (C.byref(cfg), None, None, None, 256, 1024, 64,
                                                 64, 64, nranks, rank, gather, comm, None, None,
                                                 1024, None)
    assert lib.ridge_gemm_sharded(*args(2, 2, 0, None)) == RIDGE_EINVAL     # rank out of range
    assert lib.ridge_gemm_sharded(*args(0, 0, 0, None)) == RIDGE_EINVAL     # no ranks
    assert lib.ridge_gemm_sharded(*args(2, 0, 1, None)) == RIDGE_EINVAL     # gather, no comm
    assert lib.ridge_status_string(-7).decode().startswith("NCCL")


def test_lcg_advance_matches_drawing_the_stream():
    """ridge_b200.lcg_advance(state, n) is the state after n draws, so a rank can
    start its slab of B without generating the rows before it."""
    import ctypes as C
    import numpy as np

    import oracle
    import ridge_b200 as rb
    for seed, n in [(0, 0), (0, 1), (5, 1000), (123456789, 4097)]:
        st = C.c_uint32(seed)
        buf = np.empty(max(n, 1), np.uint16)
        if n:
            oracle.lib.oracle_fill_unit(buf.ctypes.data_as(C.c_void_p), n, C.byref(st))
        assert rb.lcg_advance(seed, n) == st.value
