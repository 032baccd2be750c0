"""The GroupNorm entry point that allocates nothing (sdg_groupnorm_noalloc).

It exists for callers that cannot allocate device memory themselves — e.g. a
JNI front end that reaches the library only through its C ABI — and takes its
statistics scratch from a fixed array inside the library. Here its output is
compared, through the C ABI, with the allocating entry point (caller-provided
scratch) on two calls in a row, which also checks that the shared array's
leftover contents from the previous call do not leak into the next one.
Collected last on purpose (file name) so a failure here stops a -x run only
after every other test has run."""
import pytest
import torch

from oracle import unet_ref as R

pytestmark = pytest.mark.gpu
TOL = 2e-3   # the per-op tolerance of tests/test_ops_gpu.py


def _case(gen, B, C1, C2, H, cuda):
    x1 = (torch.randn(B, H * H, C1, generator=gen) * 1.3 + 0.7).half().to(cuda)
    x2 = None if C2 == 0 else (torch.randn(B, H * H, C2, generator=gen) - 0.5).half().to(cuda)
    gam = (torch.randn(C1 + C2, generator=gen) * 0.2 + 1.0).to(cuda)
    bet = (torch.randn(C1 + C2, generator=gen) * 0.2).to(cuda)
    return x1, x2, gam, bet


@pytest.mark.parametrize("B,C1,C2,H,silu,eps,groups", [
    (2, 320, 0, 64, True, 1e-5, 32),       # BASELINE config 1 GroupNorm+SiLU shapes
    (2, 1280, 0, 16, True, 1e-5, 32),
    (2, 1280, 640, 16, True, 1e-5, 32),    # concat input, groups straddle the two sources
    (1, 640, 0, 32, False, 1e-6, 32),      # transformer GroupNorm (no SiLU)
    # more than 32 groups: the two-launch path (the statistics kernel writes the (mean, rstd) pairs
    # into the library's array, the apply kernel reads them back), so stale contents would show here
    (2, 640, 0, 32, True, 1e-5, 64),
    (3, 1280, 640, 16, False, 1e-5, 64),
    (16, 640, 0, 32, True, 1e-5, 64),
])
def test_noalloc_groupnorm_matches_allocating_entry(sdg, cuda, B, C1, C2, H, silu, eps, groups):
    gen = torch.Generator().manual_seed(B * 1000 + C1 + C2 + H + groups)
    x1, x2, gam, bet = _case(gen, B, C1, C2, H, cuda)
    ref = sdg.groupnorm(x1, gam, bet, eps, silu, x2=x2, groups=groups)
    # a different input first, so the second call starts from stale scratch contents
    y1, y2, g2, b2 = _case(gen, B, C1, C2, H, cuda)
    other_ref = sdg.groupnorm(y1, g2, b2, eps, silu, x2=y2, groups=groups)
    other = sdg.groupnorm_noalloc(y1, g2, b2, eps, silu, x2=y2, groups=groups)
    got = sdg.groupnorm_noalloc(x1, gam, bet, eps, silu, x2=x2, groups=groups)
    torch.cuda.synchronize()
    assert R.rel_err_l1(other.float().cpu(), other_ref.float().cpu()) < TOL
    assert R.rel_err_l1(got.float().cpu(), ref.float().cpu()) < TOL
    # and against the oracle
    xin = x1.float().cpu() if x2 is None else torch.cat([x1, x2], -1).float().cpu()
    Bn, HW, C = xin.shape
    o = R.groupnorm(xin.permute(0, 2, 1).reshape(Bn, C, H, H), gam.cpu(), bet.cpu(), eps, silu, groups=groups)
    assert R.rel_err_l1(got.float().cpu(), o.reshape(Bn, C, HW).permute(0, 2, 1)) < TOL


def test_noalloc_groupnorm_rejects_bad_arguments(sdg, cuda):
    """Negative or zero channel counts are refused with SDG_ERR_ARG by both entry points."""
    x = torch.zeros((1, 16, 640), dtype=torch.float16, device=cuda)
    x2 = torch.zeros((1, 16, 320), dtype=torch.float16, device=cuda)
    g = torch.ones(960, device=cuda)
    y = torch.empty((1, 16, 960), dtype=torch.float16, device=cuda)
    st = torch.empty(1024, dtype=torch.float32, device=cuda)
    P = sdg._ptr
    for c1, c2 in ((640, -320), (0, 320), (-320, 640)):
        assert sdg.lib().sdg_groupnorm_noalloc(P(x), P(x2), 1, 16, c1, c2, 32, P(g), P(g), 1e-5, 1, P(y), None) == 2
        assert sdg.lib().sdg_groupnorm(P(x), P(x2), 1, 16, c1, c2, 32, P(g), P(g), 1e-5, 1, P(y), P(st), None) == 2


def test_noalloc_groupnorm_rejects_oversized_shapes(sdg, cuda):
    cap = sdg.lib().sdg_groupnorm_noalloc_max_scratch_bytes()
    assert cap == 64 << 10
    B, H, C = 300, 2, 64                     # 300 images x 32 groups needs 75 KiB of (mean, rstd) pairs
    assert sdg.lib().sdg_groupnorm_scratch_bytes(B, H * H, C, 32) > cap
    x = torch.zeros((B, H * H, C), dtype=torch.float16, device=cuda)
    g = torch.ones(C, device=cuda)
    with pytest.raises(sdg.SdgError) as ei:
        sdg.groupnorm_noalloc(x, g, g, 1e-5, True)
    assert ei.value.code == 3 and "scratch" in str(ei.value)
