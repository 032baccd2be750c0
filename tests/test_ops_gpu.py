"""Per-op parity of the CUDA kernels (through the C ABI) against the fp32
oracle ops on the same seeded inputs. Shapes: BASELINE config 1 (op
microbench) and config 2 (attention) plus small / ragged cases.

Tolerance: relErr = sum|got-ref|/sum|ref| (vk_engine.cpp:698-704) <= 2e-3 for
single ops with fp16 inputs/outputs and fp32 accumulation (fp16 output
rounding alone is ~2.5e-4)."""
import math

import pytest
import torch
import torch.nn.functional as F

from oracle import unet_ref as R

pytestmark = pytest.mark.gpu
TOL = 2e-3


def rel(got, ref):
    return R.rel_err_l1(got.float().cpu(), ref.float().cpu())


def rnd(*shape, std=1.0, dev="cuda", g=None):
    return (torch.randn(*shape, generator=g) * std).to(dev)


@pytest.fixture()
def gen():
    return torch.Generator().manual_seed(1234)


# ---------------------------------------------------------------- linear / GEMM
@pytest.mark.parametrize("M,N,K,bias,resid,act", [
    (8192, 320, 320, True, False, 0),      # proj_in / out-proj at 64x64 (BN 160)
    (8192, 2560, 320, True, True, 0),      # FF-proj width (BN 256) + residual
    (4096, 320, 1280, True, True, 0),      # FF-out
    (154, 640, 768, False, False, 0),      # cross K/V from context (ragged M)
    (300, 128, 192, True, False, 1),       # ragged M + SiLU
    (2048, 64, 64, True, False, 0),        # narrow N (BN 64)
    (1, 320, 1280, True, False, 0),        # single row
])
def test_linear(sdg, cuda, gen, M, N, K, bias, resid, act):
    x = rnd(M, K, g=gen).half()
    w = rnd(N, K, std=1 / math.sqrt(K), g=gen).half()
    b = rnd(N, std=0.1, g=gen).float() if bias else None
    r = rnd(M, N, g=gen).half() if resid else None
    y = sdg.linear(x, w, b, residual=r, act=act)
    torch.cuda.synchronize()
    ref = x.float() @ w.float().T
    if b is not None:
        ref = ref + b
    if r is not None:
        ref = ref + r.float()
    if act == 1:
        ref = F.silu(ref)
    assert rel(y, ref) < TOL


@pytest.mark.parametrize("M,C", [(4096, 320), (2048, 640), (512, 1280), (200, 320)])  # the UNet's FF-proj shapes
def test_linear_geglu(sdg, cuda, gen, M, C):
    x = rnd(M, C, g=gen).half()
    w = rnd(8 * C, C, std=1 / math.sqrt(C), g=gen).half()
    b = rnd(8 * C, std=0.1, g=gen).float()
    wp, bp = sdg.pack_geglu_weight(w, b)
    y = sdg.linear(x, wp, bp, act=2)
    torch.cuda.synchronize()
    ref = R.geglu(x.float() @ w.float().T + b)
    assert y.shape == (M, 4 * C)
    assert rel(y, ref) < TOL


def test_geglu_gelu_accuracy(sdg, cuda):
    """The GEGLU epilogue's GELU (erf from Abramowitz & Stegun 7.1.26) against exact erf GELU in
    fp64: value input 1 and gate input u swept over [-8, 8], so each output is fp16(gelu(u))."""
    M, K = 4096, 64
    u = torch.linspace(-8.0, 8.0, M).half()
    x = torch.zeros(M, K, dtype=torch.float16)
    x[:, 0] = u
    x[:, 1] = 1.0
    w = torch.zeros(256, K, dtype=torch.float16)   # rows 0..127 value, 128..255 gate
    w[:128, 1] = 1.0
    w[128:, 0] = 1.0
    wp, _ = sdg.pack_geglu_weight(w.to(cuda))
    y = sdg.linear(x.to(cuda), wp, torch.zeros(256, device=cuda), act=2)
    torch.cuda.synchronize()
    ref = F.gelu(u.double())
    got = y.double().cpu()
    assert torch.equal(got, got[:, :1].expand_as(got))        # every column holds the same value
    err = (got[:, 0] - ref).abs()
    assert bool((err <= ref.abs() * 2.0 ** -11 + 2e-6).all()), float(err.max())


# ---------------------------------------------------------------- conv
def nhwc(x):
    return x.permute(0, 2, 3, 1).contiguous()


def nchw(x):
    return x.permute(0, 3, 1, 2)


@pytest.mark.parametrize("B,Ci,Co,H", [
    (2, 320, 320, 64), (2, 640, 640, 32), (2, 1280, 1280, 16), (2, 1280, 1280, 8),   # config 1
    (1, 64, 64, 8), (2, 64, 128, 4), (3, 128, 64, 16),                               # small / ragged
])
def test_conv3x3(sdg, cuda, gen, B, Ci, Co, H):
    x = rnd(B, Ci, H, H, g=gen).half()
    w = rnd(Co, Ci, 3, 3, std=1 / math.sqrt(9 * Ci), g=gen).half()
    b = rnd(Co, std=0.1, g=gen).float()
    y = sdg.conv2d(nhwc(x), sdg.pack_conv_weight(w), b, Co, k=3)
    torch.cuda.synchronize()
    ref = F.conv2d(x.float(), w.float(), b, padding=1)
    assert rel(nchw(y), ref) < TOL


def test_conv3x3_concat_rowbias_residual(sdg, cuda, gen):
    B, C1, C2, Co, H = 2, 128, 64, 128, 16
    x1 = rnd(B, C1, H, H, g=gen).half()
    x2 = rnd(B, C2, H, H, g=gen).half()
    w = rnd(Co, C1 + C2, 3, 3, std=1 / math.sqrt(9 * (C1 + C2)), g=gen).half()
    b = rnd(Co, std=0.1, g=gen).float()
    rb = rnd(B, Co, std=0.5, g=gen).float()
    res = rnd(B, Co, H, H, g=gen).half()
    y = sdg.conv2d(nhwc(x1), sdg.pack_conv_weight(w), b, Co, k=3, x2=nhwc(x2), rowbias=rb, residual=nhwc(res))
    torch.cuda.synchronize()
    ref = F.conv2d(torch.cat([x1, x2], 1).float(), w.float(), b, padding=1) + rb[:, :, None, None] + res.float()
    assert rel(nchw(y), ref) < TOL


def test_conv1x1_skip(sdg, cuda, gen):
    B, Ci, Co, H = 2, 320, 640, 32                                                    # config 1 skip conv
    x = rnd(B, Ci, H, H, g=gen).half()
    w = rnd(Co, Ci, 1, 1, std=1 / math.sqrt(Ci), g=gen).half()
    b = rnd(Co, std=0.1, g=gen).float()
    y = sdg.conv2d(nhwc(x), sdg.pack_conv_weight(w), b, Co, k=1)
    torch.cuda.synchronize()
    assert rel(nchw(y), F.conv2d(x.float(), w.float(), b)) < TOL


def test_conv1x1_concat(sdg, cuda, gen):
    B, C1, C2, Co, H = 2, 640, 320, 320, 16
    x1 = rnd(B, C1, H, H, g=gen).half()
    x2 = rnd(B, C2, H, H, g=gen).half()
    w = rnd(Co, C1 + C2, 1, 1, std=1 / math.sqrt(C1 + C2), g=gen).half()
    b = rnd(Co, std=0.1, g=gen).float()
    y = sdg.conv2d(nhwc(x1), sdg.pack_conv_weight(w), b, Co, k=1, x2=nhwc(x2))
    torch.cuda.synchronize()
    assert rel(nchw(y), F.conv2d(torch.cat([x1, x2], 1).float(), w.float(), b)) < TOL


@pytest.mark.parametrize("B,C,H", [(2, 320, 64), (2, 640, 32), (2, 1280, 16),   # the three downsamplers
                                   (1, 1280, 16), (3, 640, 16), (1, 320, 8)])   # partial tiles, images per tile
def test_conv3x3_stride2(sdg, cuda, gen, B, C, H):
    x = rnd(B, C, H, H, g=gen).half()
    w = rnd(C, C, 3, 3, std=1 / math.sqrt(9 * C), g=gen).half()
    b = rnd(C, std=0.1, g=gen).float()
    y = sdg.conv2d(nhwc(x), sdg.pack_conv_weight(w), b, C, k=3, stride=2)
    torch.cuda.synchronize()
    assert rel(nchw(y), F.conv2d(x.float(), w.float(), b, stride=2, padding=1)) < TOL


# ---------------------------------------------------------------- norms
@pytest.mark.parametrize("B,C,H,silu,eps,shift", [
    (2, 320, 64, True, 1e-5, 0.0), (2, 1280, 16, True, 1e-5, 0.0),                   # config 1
    (2, 640, 32, False, 1e-6, 3.0), (1, 2560, 8, True, 1e-5, -2.0), (2, 960, 64, True, 1e-5, 0.5),
    (8, 960, 32, True, 1e-5, 0.0), (16, 320, 64, True, 1e-5, 1.0),    # larger batches
])
def test_groupnorm(sdg, cuda, gen, B, C, H, silu, eps, shift):
    x = (rnd(B, C, H, H, g=gen) * 1.5 + shift).half()
    gam = rnd(C, std=0.3, g=gen).float() + 1.0
    bet = rnd(C, std=0.3, g=gen).float()
    y = sdg.groupnorm(nhwc(x).reshape(B, H * H, C), gam, bet, eps, silu)
    torch.cuda.synchronize()
    ref = R.groupnorm(x.float(), gam, bet, eps, silu)
    assert rel(nchw(y.reshape(B, H, H, C)), ref) < TOL


@pytest.mark.parametrize("C,H", [(320, 64), (1280, 8)])
def test_groupnorm_offset_data_outlier_shift(sdg, cuda, gen, C, H):
    # the fused kernel sums values shifted by each group's pixel-0 element: a mean 40x the spread,
    # with pixel 0 a further 50 spreads away, still gives the two-pass result
    B = 2
    x = rnd(B, C, H, H, g=gen) * 0.5 + 20.0
    x[:, :, 0, 0] += 25.0
    x = x.half()
    gam = rnd(C, std=0.3, g=gen).float() + 1.0
    bet = rnd(C, std=0.3, g=gen).float()
    y = sdg.groupnorm(nhwc(x).reshape(B, H * H, C), gam, bet, 1e-5, True)
    torch.cuda.synchronize()
    ref = R.groupnorm(x.float(), gam, bet, 1e-5, True)
    assert rel(nchw(y.reshape(B, H, H, C)), ref) < TOL


def test_groupnorm_concat_straddling_groups(sdg, cuda, gen):
    # up_blocks.1.resnets.2: concat 1280 + 640 -> 1920 channels, 60 per group: groups straddle the sources
    B, C1, C2, H = 2, 1280, 640, 16
    x1 = rnd(B, C1, H, H, g=gen).half()
    x2 = (rnd(B, C2, H, H, g=gen) + 1.0).half()
    gam = rnd(C1 + C2, std=0.2, g=gen).float() + 1.0
    bet = rnd(C1 + C2, std=0.2, g=gen).float()
    y = sdg.groupnorm(nhwc(x1).reshape(B, H * H, C1), gam, bet, 1e-5, True, x2=nhwc(x2).reshape(B, H * H, C2))
    torch.cuda.synchronize()
    ref = R.groupnorm(torch.cat([x1, x2], 1).float(), gam, bet, 1e-5, True)
    assert rel(nchw(y.reshape(B, H, H, C1 + C2)), ref) < TOL


@pytest.mark.parametrize("M,C", [(8192, 320), (2048, 640), (512, 1280), (77, 320)])
def test_layernorm(sdg, cuda, gen, M, C):
    x = (rnd(M, C, g=gen) * 2 + 0.5).half()
    gam = rnd(C, std=0.3, g=gen).float() + 1.0
    bet = rnd(C, std=0.3, g=gen).float()
    y = sdg.layernorm(x, gam, bet, 1e-5)
    torch.cuda.synchronize()
    assert rel(y, R.layernorm(x.float(), gam, bet)) < TOL


# ---------------------------------------------------------------- attention (config 2)
@pytest.mark.parametrize("Sq,Sk,d", [
    (4096, 4096, 40), (1024, 1024, 80), (256, 256, 160),        # self-attention
    (4096, 77, 40), (256, 77, 160),                             # cross-attention
    (64, 64, 160), (1024, 77, 80),                              # mid block, cross d80
])
def test_attention(sdg, cuda, gen, Sq, Sk, d):
    B, heads = 2, 8
    C = heads * d
    q = rnd(B * Sq, C, g=gen).half()
    k = rnd(B * Sk, C, g=gen).half()
    v = rnd(B * Sk, C, g=gen).half()
    vt_ld = (Sk + 7) // 8 * 8
    o = sdg.attention(sdg.heads_layout(q, B, Sq, heads, d), sdg.heads_layout(k, B, Sk, heads, d),
                      sdg.heads_layout(v, B, Sk, heads, d, transpose=True, s_pad=vt_ld), B, heads, Sq, Sk, d, vt_ld)
    torch.cuda.synchronize()
    ref = R.attention(q.float().view(B, Sq, C), k.float().view(B, Sk, C), v.float().view(B, Sk, C), heads)
    assert rel(o, ref) < TOL


# ---------------------------------------------------------------- elementwise
def test_upsample_concat_add(sdg, cuda, gen):
    B, C, H = 2, 640, 16
    x = rnd(B, C, H, H, g=gen).half()
    y = sdg.upsample2x(nhwc(x))
    torch.cuda.synchronize()
    assert torch.equal(nchw(y).float().cpu(), R.upsample2x(x.float()).cpu())
    a = rnd(B, H, H, 320, g=gen).half()
    b = rnd(B, H, H, 640, g=gen).half()
    c = sdg.concat(a, b)
    torch.cuda.synchronize()
    assert torch.equal(c, torch.cat([a, b], -1))
    s = sdg.add(a, a)
    torch.cuda.synchronize()
    assert torch.equal(s, a + a)


# ---------------------------------------------------------------- upsample block as one folded GEMM
@pytest.mark.parametrize("B,C,H,W,ws", [
    (2, 1280, 8, 8, False), (2, 1280, 16, 16, False), (2, 640, 32, 32, False),   # the UNet's three upsamplers
    (2, 1280, 8, 8, True), (2, 1280, 16, 16, True),                              # with a split-K workspace
    (1, 64, 1, 1, False), (4, 128, 2, 2, False), (1, 192, 4, 4, True), (3, 64, 16, 8, False),  # small / ragged
])
def test_upsample_conv3x3_matches_upsample_then_conv(sdg, cuda, gen, B, C, H, W, ws):
    """vk_engine.cpp:693-697 (upsample_f32.comp nearest 2x, then the 3x3 pad-1 conv) against the
    folded phase GEMM, which reads the H x W input directly."""
    Co = C
    x = rnd(B, C, H, W, g=gen).half()
    w = rnd(Co, C, 3, 3, std=1 / math.sqrt(9 * C), g=gen).half()
    b = rnd(Co, std=0.1, g=gen).float()
    wp = torch.from_numpy(sdg.pack_upsample_conv_weight(w.cpu().numpy())).to(cuda)
    work = torch.empty(32 * B * H * W * 4 * Co, dtype=torch.float32, device=cuda) if ws else None
    y = sdg.upsample_conv3x3(nhwc(x), wp, b.repeat(4), workspace=work)
    torch.cuda.synchronize()
    ref = F.conv2d(R.upsample2x(x.float()), w.float(), b, padding=1)
    assert y.shape == (B, 2 * H, 2 * W, Co)
    assert rel(nchw(y), ref) < TOL


# ---------------------------------------------------------------- split-K (deep levels: small M, large K)
@pytest.mark.parametrize("M,N,K,resid", [(128, 1280, 11520, True), (512, 1280, 5120, False), (154, 640, 768, True),
                                         (300, 320, 2880, False)])
def test_linear_splitk(sdg, cuda, gen, M, N, K, resid):
    x = rnd(M, K, g=gen).half()
    w = rnd(N, K, std=1 / math.sqrt(K), g=gen).half()
    b = rnd(N, std=0.1, g=gen).float()
    r = rnd(M, N, g=gen).half() if resid else None
    ws = torch.empty(32 * M * N, dtype=torch.float32, device=cuda)
    y = sdg.linear(x, w, b, residual=r, workspace=ws)
    torch.cuda.synchronize()
    ref = x.float() @ w.float().T + b + (r.float() if resid else 0)
    assert rel(y, ref) < TOL


@pytest.mark.parametrize("B,C,H", [(2, 1280, 8), (2, 1280, 16), (2, 640, 32), (1, 2560, 8)])
def test_conv3x3_splitk_rowbias_residual(sdg, cuda, gen, B, C, H):
    Co = 1280 if C == 2560 else C
    x = rnd(B, C, H, H, g=gen).half()
    w = rnd(Co, C, 3, 3, std=1 / math.sqrt(9 * C), g=gen).half()
    b = rnd(Co, std=0.1, g=gen).float()
    rb = rnd(B, Co, std=0.5, g=gen).float()
    res = rnd(B, Co, H, H, g=gen).half()
    ws = torch.empty(32 * B * H * H * Co, dtype=torch.float32, device=cuda)
    y = sdg.conv2d(nhwc(x), sdg.pack_conv_weight(w), b, Co, k=3, rowbias=rb, residual=nhwc(res), workspace=ws)
    torch.cuda.synchronize()
    ref = F.conv2d(x.float(), w.float(), b, padding=1) + rb[:, :, None, None] + res.float()
    assert rel(nchw(y), ref) < TOL


# ---------------------------------------------------------------- every K-split path of the tile chooser
# (M, N, K): UNet GEMM / conv3x3 shapes (a conv's K is 9 * Cin; the chooser sees only M, N, K)
SPLIT_SHAPES = [(128, 1280, 1280), (128, 1280, 11520), (512, 1280, 5120), (512, 1280, 11520), (2048, 640, 5760),
                (154, 640, 768), (8192, 320, 320), (128, 1280, 23040)]


def _plan_kind(pl):
    return "cluster" if pl["csplit"] > 1 else ("workspace" if pl["splits"] > 1 else "single")


def test_gemm_plan_covers_every_split_path(sdg, cuda):
    kinds = {_plan_kind(sdg.gemm_plan(M, N, K)) for M, N, K in SPLIT_SHAPES}
    assert kinds == {"cluster", "workspace", "single"}, kinds
    for M, N, K in SPLIT_SHAPES:  # without a workspace the chooser never asks for one
        assert sdg.gemm_plan(M, N, K, workspace=False)["splits"] == 1


@pytest.mark.parametrize("with_ws", [True, False])
@pytest.mark.parametrize("M,N,K", SPLIT_SHAPES)
def test_linear_every_split_path(sdg, cuda, gen, M, N, K, with_ws):
    x = rnd(M, K, g=gen).half()
    w = rnd(N, K, std=1 / math.sqrt(K), g=gen).half()
    b = rnd(N, std=0.1, g=gen).float()
    r = rnd(M, N, g=gen).half()
    ws = torch.empty(32 * M * N, dtype=torch.float32, device=cuda) if with_ws else None
    y = sdg.linear(x, w, b, residual=r, workspace=ws)
    torch.cuda.synchronize()
    ref = x.float() @ w.float().T + b + r.float()
    err = rel(y, ref)
    assert err < TOL, (err, sdg.gemm_plan(M, N, K, workspace=with_ws))
