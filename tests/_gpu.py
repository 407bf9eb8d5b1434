"""Helpers shared by the GPU tests: move oracle inputs to the device, run the
GEMM through the C ABI, and compare against the FP64 oracle."""

import numpy as np
import torch

import oracle
import ridge_b200 as rb


def to_dev(h: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(h).view(np.float16)).cuda()


def to_host_bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().numpy().view(np.uint16)


def run_gemm(cfg, a_dev, b_dev, M, N, K, ldc=None, fill=float("nan")):
    ldc = ldc or N
    c = torch.full((M, ldc), fill, dtype=torch.float16, device="cuda")
    st = rb.launch_raw(cfg, a_dev.data_ptr(), b_dev.data_ptr(), c.data_ptr(), M, N, K,
                       a_dev.stride(0), b_dev.stride(0), ldc, torch.cuda.current_stream().cuda_stream)
    assert st == 0, "launch %s -> %s" % (cfg.tag(), rb.lib.ridge_status_string(st).decode())
    torch.cuda.synchronize()
    assert rb.device_error() == 0, "device error word set after %s" % cfg.tag()
    return c


def assert_close(c_bits: np.ndarray, ref: np.ndarray, what: str):
    rel, max_abs, excess = oracle.fp16_stats(c_bits, ref)
    assert rel <= oracle.REL_FROB_TOL and excess <= oracle.MAX_ABS_EXCESS_TOL, (
        "%s: rel_frob %.3e (tol %.0e), max|dC| %.3e, excess over half-ulp %.3e (tol %.0e)"
        % (what, rel, oracle.REL_FROB_TOL, max_abs, excess, oracle.MAX_ABS_EXCESS_TOL))
    return rel, max_abs, excess
