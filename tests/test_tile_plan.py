"""Host logic of the GEMM tile chooser, through ``sdg_gemm_plan`` (no kernel runs, no GPU needed).

The plans depend on the device: without one the chooser assumes 148 SMs and num_sms / cluster-size
resident clusters; with one it asks the device how many clusters of each size fit
(cudaOccupancyMaxActiveClusters), so a plan checked here on a host without a GPU can differ from the
one a B200 runs. The invariants below hold either way.

Invariants the kernels rely on: the tile width divides N (or is the ragged 64 fallback), a K split
is either a workspace split or a cluster split of at most 10 CTAs (never both, never on a CTA pair or a
256-wide 1-CTA tile), every split owns at least one 64-deep k-block, and without a workspace no workspace
split is chosen.
"""
import pytest

# (M, N, K) of the SD1.5 UNet's GEMMs and 3x3 convolutions (K = 9 * Cin) at B=2, 64x64 latent
UNET_SHAPES = [
    (8192, 320, 64), (8192, 320, 320), (8192, 960, 320), (8192, 320, 1280), (8192, 2560, 320), (8192, 320, 2880),
    (8192, 320, 5760), (8192, 320, 8640), (2048, 640, 640), (2048, 1920, 640), (2048, 640, 2560), (2048, 640, 5760),
    (2048, 320, 2880), (2048, 640, 11520), (512, 1280, 1280), (512, 3840, 1280), (512, 1280, 5120), (512, 1280, 11520),
    (512, 1280, 23040), (512, 640, 5760), (128, 1280, 1280), (128, 1280, 11520), (128, 1280, 23040),
    (154, 640, 768), (154, 1280, 768), (300, 128, 192),
]


@pytest.mark.parametrize("with_ws", [True, False])
@pytest.mark.parametrize("M,N,K", UNET_SHAPES)
def test_plan_invariants(sdg, M, N, K, with_ws):
    pl = sdg.gemm_plan(M, N, K, workspace=with_ws)
    bn, pair, splits, csplit = pl["bn"], pl["pair"], pl["splits"], pl["csplit"]
    assert bn in (16, 64, 128, 160, 192, 256)
    assert N % bn == 0 or bn == 64
    assert splits >= 1 and 1 <= csplit <= 10
    assert not (splits > 1 and csplit > 1)
    assert not (pair and csplit > 1)
    assert not (bn == 256 and csplit > 1)
    if not with_ws:
        assert splits == 1
    kb = K // 64
    parts = max(splits, csplit)
    per = -(-kb // parts)
    assert (parts - 1) * per < kb, "a K split would own no k-block"


def test_deep_levels_split_k(sdg):
    # 8x8 level: M = 128 rows, a long K; one tile row cannot fill the GPU without a K split
    for K in (11520, 23040):
        pl = sdg.gemm_plan(128, 1280, K)
        assert pl["splits"] > 1 or pl["csplit"] > 1
        pl = sdg.gemm_plan(128, 1280, K, workspace=False)
        assert pl["csplit"] > 1


def test_large_m_single_pass(sdg):
    # 64x64 level: 64 row tiles already fill the GPU
    pl = sdg.gemm_plan(8192, 320, 2880)
    assert pl["splits"] == 1 and pl["csplit"] == 1


@pytest.mark.parametrize("args", [(0, 320, 320, 1), (8192, 320, 100, 1), (8192, 320, 320, 3), (8192, 320, 640, 9),
                                  (8192, -1, 320, 1)])
def test_plan_rejects_bad_arguments(sdg, args):
    M, N, K, taps = args
    with pytest.raises(sdg.SdgError):
        sdg.gemm_plan(M, N, K, taps=taps)
