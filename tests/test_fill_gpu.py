"""The device LCG fill is bit-identical to the oracle's restatement of the
reference fill (bench/check-gemm.cu:139-145), for both value ranges and across
chained calls (A then B from one stream)."""

import numpy as np
import pytest

import oracle

torch = pytest.importorskip("torch")
pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")]


@pytest.mark.parametrize("n,seed", [(1, 0), (15, 0x1234), (16, 0x9abc), (1000003, 7)])
def test_reference_range_bit_exact(n, seed):
    import ctypes as C
    import ridge_b200 as rb
    out = torch.empty(n, dtype=torch.float16, device="cuda")
    st = C.c_uint32(seed)
    assert rb.lib.ridge_fill_lcg(out.data_ptr(), n, C.byref(st), 0, None) == 0
    got = out.cpu().numpy().view(np.uint16)
    assert np.array_equal(got, oracle.fill_reference(n, seed))


def test_unit_range_chained_matches_oracle():
    import ridge_b200 as rb
    M, N, K = 300, 200, 72
    a, b = rb.synthetic_inputs(M, N, K, seed=0)
    ra, rb_ = oracle.unit_inputs(M, N, K, seed=0)
    assert np.array_equal(a.cpu().numpy().view(np.uint16), ra)
    assert np.array_equal(b.cpu().numpy().view(np.uint16), rb_)
