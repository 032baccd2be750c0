"""Device-side failure detection without a GPU fault.

Every wait inside the kernels is bounded: when one runs out the kernel writes a
code into its error word, waits for the copies and MMAs it has in flight,
frees its TMEM and returns, and the host reports SDG_ERR_DEVICE. Here the
tensor-core GEMM is run with one pipeline stage that the producer never loads
(a barrier that nothing completes) and a 1 ms wait limit; the call must come
back with SDG_ERR_DEVICE, and the same CUDA context must then still give
correct results: a plain GEMM and a full UNet forward against the oracle.
"""
import numpy as np
import pytest
import torch

from oracle import unet_ref as R
from oracle import weights as W

pytestmark = pytest.mark.gpu
SDG_ERR_DEVICE = 8
TIMEOUT_CODES = ("0x101", "0x102", "0x103")   # full-stage, free-stage, accumulator waits


def test_expired_wait_reports_device_error_and_context_survives(sdg, cuda, engine, unet_weights):
    g = torch.Generator().manual_seed(11)
    M, N, K = 256, 128, 1024
    x = (torch.randn(M, K, generator=g) * 0.5).half().to(cuda)
    w = (torch.randn(N, K, generator=g) * 0.05).half().to(cuda)
    y = torch.empty(M, N, dtype=torch.float16, device=cuda)
    err = torch.zeros(64, dtype=torch.int32, device=cuda)
    P = sdg._ptr
    for stall_iter in (1, 0):            # a stage after the first, then the very first one
        code = sdg.lib().sdg_selftest_stalled_gemm(P(x), P(w), M, N, K, P(y), stall_iter, 1000, P(err), None)
        msg = sdg.last_error()
        assert code == SDG_ERR_DEVICE, (code, msg)
        assert any(c in msg for c in TIMEOUT_CODES), msg
        torch.cuda.synchronize()
        assert int(err[0].item()) == 0          # the call cleared the word it reported
    # the context is intact: the same GEMM without the stall is right ...
    ref = x.float() @ w.float().t()
    out = sdg.linear(x, w)
    torch.cuda.synchronize()
    assert R.rel_err_l1(out.float().cpu(), ref.cpu()) < 2e-3
    # ... and so is a whole UNet forward through the engine
    lat, t, ctx = W.make_inputs(2, 16, 16, seed=3)
    got = engine.forward(lat.numpy(), t.numpy(), ctx.numpy())
    with torch.no_grad():
        want = R.unet_forward(lat, t, ctx, unet_weights).numpy()
    assert np.isfinite(got).all()
    assert float(np.abs(got - want).sum() / np.abs(want).sum()) < 3e-3


def test_stalled_gemm_rejects_bad_arguments(sdg, cuda):
    x = torch.zeros(128, 128, dtype=torch.float16, device=cuda)
    err = torch.zeros(64, dtype=torch.int32, device=cuda)
    P = sdg._ptr
    L = sdg.lib()
    assert L.sdg_selftest_stalled_gemm(P(x), P(x), 128, 96, 128, P(x), 1, 1000, P(err), None) == 2   # N % 128
    assert L.sdg_selftest_stalled_gemm(P(x), P(x), 128, 128, 128, P(x), -1, 1000, P(err), None) == 2  # no stall
    assert L.sdg_selftest_stalled_gemm(P(x), P(x), 128, 128, 128, P(x), 1, 0, P(err), None) == 2      # no limit
