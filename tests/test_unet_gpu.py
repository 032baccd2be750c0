"""Full-path parity of the CUDA engine against the fp32 oracle.

* Block KATs: the reference's own PyTorch goldens (assets/rb, assets/tf) run
  through the C-ABI op surface, composed like the reference's block harnesses
  (vk_engine.cpp:423-480, 931-1012). Reference bars: 0.03 / 0.06; ours 3e-3.
* Full UNet (BASELINE config 0 and smaller latents): relErr <= 3e-3 vs the
  oracle on identical seeded inputs and fp16-rounded seeded weights.
* Batch-CFG, B=2 self-test semantics (vk_engine.cpp:823-839), the tproj entry
  point, the device-pointer entry point, and the 4-step LCM loop (config 3).
"""
import math

import numpy as np
import pytest
import torch

from oracle import fixtures as fx
from oracle import lcm as LCM
from oracle import unet_ref as R
from oracle import weights as W

pytestmark = pytest.mark.gpu
UNET_TOL = 3e-3


def rel(got, ref):
    return R.rel_err_l1(torch.as_tensor(got).float().cpu(), torch.as_tensor(ref).float().cpu())


def nhwc_tokens(x):  # [1,C,H,W] -> [1, H*W, C]
    B, C, H, W_ = x.shape
    return x.permute(0, 2, 3, 1).reshape(B, H * W_, C).contiguous()


# ---------------------------------------------------------------- block KATs via the op surface
def test_resnet_block_kat_via_ops(sdg, cuda):
    x, temb, w, y = fx.load_rb()
    dev = lambda t: t.to(cuda)
    C, H = 320, 64
    xt = dev(nhwc_tokens(x))
    h = sdg.groupnorm(xt, dev(w["rb.norm1.weight"].float()), dev(w["rb.norm1.bias"].float()), 1e-5, True)
    # time projection: SiLU(temb) @ W^T + b through the tensor-core linear
    ts = torch.nn.functional.silu(temb.float()).half().to(cuda)
    tp = sdg.linear(ts, dev(w["rb.time_emb_proj.weight"]), dev(w["rb.time_emb_proj.bias"].float()))
    h2 = sdg.conv2d(h.view(1, H, H, C), dev(sdg.pack_conv_weight(w["rb.conv1.weight"])), dev(w["rb.conv1.bias"].float()),
                    C, rowbias=tp.float())
    h3 = sdg.groupnorm(h2.view(1, H * H, C), dev(w["rb.norm2.weight"].float()), dev(w["rb.norm2.bias"].float()), 1e-5, True)
    out = sdg.conv2d(h3.view(1, H, H, C), dev(sdg.pack_conv_weight(w["rb.conv2.weight"])), dev(w["rb.conv2.bias"].float()),
                     C, residual=xt.view(1, H, H, C))
    torch.cuda.synchronize()
    got = out.permute(0, 3, 1, 2).float().cpu()
    assert rel(got, y) < UNET_TOL


def test_transformer_block_kat_via_ops(sdg, cuda):
    x, ctx, w, y = fx.load_tf()
    dev = lambda t: t.to(cuda)
    C, H, heads, d = 320, 64, 8, 40
    S, M = H * H, H * H
    b = "tf.transformer_blocks.0"
    f32 = lambda k: dev(w[k].float())
    lin_w = lambda k: dev(w[k])
    xt = dev(nhwc_tokens(x)).view(M, C)
    g = sdg.groupnorm(xt.view(1, S, C), f32("tf.norm.weight"), f32("tf.norm.bias"), 1e-6, False).view(M, C)
    t = sdg.linear(g, dev(w["tf.proj_in.weight"].reshape(C, C)), f32("tf.proj_in.bias"))
    hn = sdg.layernorm(t, f32(b + ".norm1.weight"), f32(b + ".norm1.bias"))
    q = sdg.linear(hn, lin_w(b + ".attn1.to_q.weight"))
    k = sdg.linear(hn, lin_w(b + ".attn1.to_k.weight"))
    v = sdg.linear(hn, lin_w(b + ".attn1.to_v.weight"))
    o = sdg.attention(sdg.heads_layout(q, 1, S, heads, d), sdg.heads_layout(k, 1, S, heads, d),
                      sdg.heads_layout(v, 1, S, heads, d, transpose=True), 1, heads, S, S, d, S).view(M, C)
    t = sdg.linear(o, lin_w(b + ".attn1.to_out.0.weight"), f32(b + ".attn1.to_out.0.bias"), residual=t)
    hn = sdg.layernorm(t, f32(b + ".norm2.weight"), f32(b + ".norm2.bias"))
    q = sdg.linear(hn, lin_w(b + ".attn2.to_q.weight"))
    c16 = dev(ctx.view(77, 768))
    kc = sdg.linear(c16, lin_w(b + ".attn2.to_k.weight"))
    vc = sdg.linear(c16, lin_w(b + ".attn2.to_v.weight"))
    o = sdg.attention(sdg.heads_layout(q, 1, S, heads, d), sdg.heads_layout(kc, 1, 77, heads, d),
                      sdg.heads_layout(vc, 1, 77, heads, d, transpose=True, s_pad=80), 1, heads, S, 77, d, 80).view(M, C)
    t = sdg.linear(o, lin_w(b + ".attn2.to_out.0.weight"), f32(b + ".attn2.to_out.0.bias"), residual=t)
    hn = sdg.layernorm(t, f32(b + ".norm3.weight"), f32(b + ".norm3.bias"))
    wp, bp = sdg.pack_geglu_weight(lin_w(b + ".ff.net.0.proj.weight"), f32(b + ".ff.net.0.proj.bias"))
    gg = sdg.linear(hn, wp, bp, act=2)
    t = sdg.linear(gg, lin_w(b + ".ff.net.2.weight"), f32(b + ".ff.net.2.bias"), residual=t)
    out = sdg.linear(t, dev(w["tf.proj_out.weight"].reshape(C, C)), f32("tf.proj_out.bias"), residual=xt)
    torch.cuda.synchronize()
    got = out.view(1, H, H, C).permute(0, 3, 1, 2).float().cpu()
    assert rel(got, y) < UNET_TOL


# ---------------------------------------------------------------- full UNet
def oracle_forward(w, lat, t, ctx):
    with torch.no_grad():
        return R.unet_forward(torch.as_tensor(lat), torch.as_tensor(t), torch.as_tensor(ctx), w).numpy()


@pytest.mark.parametrize("B,H", [(2, 64), (2, 32), (1, 16), (4, 8)])
def test_unet_forward_matches_oracle(engine, unet_weights, B, H):
    lat, t, ctx = W.make_inputs(B, H, H, seed=H + B)
    got = engine.forward(lat.numpy(), t.numpy(), ctx.numpy())
    ref = oracle_forward(unet_weights, lat, t, ctx)
    err = rel(got, ref)
    print(f"UNet B={B} {H}x{H}: relErr {err:.3e}")
    assert np.isfinite(got).all()
    assert err < UNET_TOL


def test_unet_layernorm_affine_folded(sdg, cuda, unet_weights):
    """Default init leaves every LayerNorm at gamma = 1, beta = 0, so the other full-UNet cases never
    exercise the LayerNorm affine; here the transformer LayerNorms get random gamma and beta."""
    g = torch.Generator().manual_seed(21)
    w = dict(unet_weights)
    for k, v in unet_weights.items():
        if ".transformer_blocks.0.norm" in k:
            noise = torch.randn(v.shape, generator=g) * 0.3
            w[k] = ((1.0 + noise) if k.endswith(".weight") else noise).half()
    e = sdg.Engine(0)
    try:
        e.upload_weights(W.iter_reference_blobs(w))
        e.prepare()
        lat, t, ctx = W.make_inputs(2, 64, 64, seed=22)
        got = e.forward(lat.numpy(), t.numpy(), ctx.numpy())
    finally:
        e.release()
    ref = oracle_forward(w, lat, t, ctx)
    err = rel(got, ref)
    print(f"UNet B=2 64x64, LayerNorm affines: relErr {err:.3e}")
    assert np.isfinite(got).all() and err < UNET_TOL


def test_unet_shared_timestep_and_tproj_entry(engine):
    lat, t, ctx = W.make_inputs(2, 32, 32, seed=5)
    a = engine.forward(lat.numpy(), np.array([999.0], np.float32), ctx.numpy())
    tp = R.timestep_embedding(torch.tensor([999.0])).numpy()          # the reference caller's 320-d input
    b = engine.forward_tproj(lat.numpy(), tp, ctx.numpy())
    assert rel(b, a) < 1e-5


def test_b2_selftest_semantics_and_cfg_entry(engine):
    # vk_engine.cpp:823-839: the same input in both batch slots gives the B=1 output twice.
    # Inside one batch the two images take identical arithmetic (bit-identical); B=1 may
    # pick another split-K partition, i.e. another fp32 summation order, so it agrees
    # only to the fp16 noise floor (the parity bar).
    lat, t, ctx = W.make_inputs(1, 32, 32, seed=9)
    one = engine.forward(lat.numpy(), t.numpy(), ctx.numpy())
    both = engine.forward(np.repeat(lat.numpy(), 2, 0), np.repeat(t.numpy(), 2), np.repeat(ctx.numpy(), 2, 0))
    assert np.array_equal(both[0], both[1])
    assert rel(both[0], one[0]) < UNET_TOL
    # unetForward2: [cond ; uncond] for one latent
    _, _, unc = W.make_inputs(1, 32, 32, seed=10)
    out2 = engine.forward_cfg(lat.numpy()[0], 999.0, ctx.numpy()[0], unc.numpy()[0])
    ref = engine.forward(np.repeat(lat.numpy(), 2, 0), np.array([999.0], np.float32),
                         np.concatenate([ctx.numpy(), unc.numpy()], 0))
    assert rel(out2, ref) < 1e-5
    # context sensitivity (vk_engine.cpp:840-849): cond and uncond must differ
    assert np.abs(out2[0] - out2[1]).mean() > 1e-4


def test_device_entry_point(engine, cuda):
    lat, t, ctx = W.make_inputs(2, 32, 32, seed=3)
    host = engine.forward(lat.numpy(), t.numpy(), ctx.numpy())
    dl, dt, dc = lat.to(cuda), t.to(cuda), ctx.to(cuda)
    out = torch.empty_like(dl)
    engine.forward_device(dl, dt, dc, out)
    torch.cuda.synchronize()
    assert rel(out.cpu(), host) < 1e-5


def test_lcm_denoise_matches_oracle_loop(engine, unet_weights):
    n, H, steps = 2, 16, 4
    g = torch.Generator().manual_seed(77)
    lat0 = torch.randn((n, 4, H, H), generator=g).numpy()
    cond = torch.nn.functional.layer_norm(torch.randn((n, 77, 768), generator=g), (768,)).numpy()
    unc = torch.nn.functional.layer_norm(torch.randn((n, 77, 768), generator=g), (768,)).numpy()
    noise = torch.randn((steps - 1, n, 4, H, H), generator=g).numpy()
    got = engine.lcm_denoise(lat0, cond, unc, noise, steps=steps, cfg=1.5)
    ref = LCM.cfg_denoise(lambda l, t, c: oracle_forward(unet_weights, l, np.full((l.shape[0],), t, np.float32), c),
                          lat0, cond, unc, noise, steps=steps, cfg=1.5)
    err = rel(got, ref)
    print(f"LCM 4-step trajectory relErr {err:.3e}")
    assert err < 1e-2


@pytest.mark.parametrize("cfg_steps,cfg", [(2, 1.5), (0, 1.5), (4, 1.0)])
def test_lcm_cfg_only_first_steps_matches_oracle(engine, unet_weights, cfg_steps, cfg):
    # TpuUnetPipeline.kt:75-112: guidance on the first cfg_steps steps, cond-only forwards after them
    n, H, steps = 2, 16, 4
    g = torch.Generator().manual_seed(91 + cfg_steps)
    lat0 = torch.randn((n, 4, H, H), generator=g).numpy()
    cond = torch.nn.functional.layer_norm(torch.randn((n, 77, 768), generator=g), (768,)).numpy()
    unc = torch.nn.functional.layer_norm(torch.randn((n, 77, 768), generator=g), (768,)).numpy()
    noise = torch.randn((steps - 1, n, 4, H, H), generator=g).numpy()
    got = engine.lcm_denoise(lat0, cond, unc, noise, steps=steps, cfg=cfg, cfg_steps=cfg_steps)
    ref = LCM.cfg_denoise(lambda l, t, c: oracle_forward(unet_weights, l, np.full((l.shape[0],), t, np.float32), c),
                          lat0, cond, unc, noise, steps=steps, cfg=cfg, cfg_steps=cfg_steps)
    err = rel(got, ref)
    print(f"LCM cfg_steps={cfg_steps} cfg={cfg}: relErr {err:.3e}")
    assert err < 1e-2


def test_cached_context_graph_matches_full_forward(engine):
    # a denoise call leaves the pair plan's cross-attention K/V cached; a plain forward with another
    # context afterwards must recompute them (full graph), and agree with a fresh evaluation
    lat, t, ctx = W.make_inputs(2, 16, 16, seed=21)
    before = engine.forward(lat.numpy(), t.numpy(), ctx.numpy())
    g = torch.Generator().manual_seed(5)
    other = torch.nn.functional.layer_norm(torch.randn((1, 77, 768), generator=g), (768,)).numpy()
    engine.lcm_denoise(lat.numpy()[:1], other, other, np.zeros((3, 1, 4, 16, 16), np.float32), steps=4, cfg=1.5)
    after = engine.forward(lat.numpy(), t.numpy(), ctx.numpy())
    assert np.array_equal(before, after)


def test_bad_shape_and_missing_weight_are_reported(sdg, cuda, engine):
    lat = np.zeros((1, 4, 12, 12), np.float32)
    with pytest.raises(sdg.SdgError) as ei:
        engine.forward(lat, np.array([1.0], np.float32), np.zeros((1, 77, 768), np.float32))
    assert ei.value.code == 3                                   # SDG_ERR_SHAPE
    e2 = sdg.Engine(0)
    e2.upload_weight("conv_in.bias", np.zeros(320, np.float16), (320,))
    with pytest.raises(sdg.SdgError) as ei:
        e2.prepare()
    assert ei.value.code == 4 and "missing" in str(ei.value)   # SDG_ERR_MISSING_WEIGHT
    e2.release()


def test_profile_categories(engine):
    prof = engine.profile(2, 32, 32)
    assert {"GN", "CONV3", "GEMM", "ATTN"} <= set(prof)
    assert all(ms > 0 for ms, _, _, _ in prof.values())
    assert prof["CONV3"][2] > 0 and prof["GN"][3] > 0          # algorithmic FLOPs / bytes accounted
