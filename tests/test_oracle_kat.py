"""Pin the CPU oracle against the reference's own golden vectors (CPU only)."""
import math

import numpy as np
import torch

from oracle import fixtures as fx
from oracle import lcm
from oracle import unet_ref as R
from oracle import weights as W


def test_resnet_block_matches_reference_golden():
    # assets/rb: PyTorch ResnetBlock2D output (VulkanBench.kt:54-64); the
    # reference's own bar is relErr < 0.03, the fp16 rounding floor is ~2.3e-4
    x, temb, w, y = fx.load_rb()
    out = R.resnet_block(x.float(), temb.float(), w, "rb")
    assert R.rel_err_l1(out, y.float()) < 5e-4


def test_transformer_block_matches_reference_golden():
    # assets/tf: PyTorch Transformer2DModel output (VulkanBench.kt:39-52); bar 0.06
    x, ctx, w, y = fx.load_tf()
    out = R.transformer_block(x.float(), ctx.float(), w, "tf")
    assert R.rel_err_l1(out, y.float()) < 5e-4


def test_fixture_manifest_integrity():
    import hashlib, os
    for line in open(os.path.join(fx.GOLDEN, "MANIFEST.txt")):
        rel, size, sha = line.split()
        data = open(os.path.join(fx.GOLDEN, rel), "rb").read()
        assert len(data) == int(size) and hashlib.sha256(data).hexdigest() == sha, rel


def test_timestep_embedding_matches_kotlin_formula():
    # VulkanUnetPipeline.kt:36-46: cos(t*f_i) then sin(t*f_i), f_i = exp(-ln(1e4) i/160)
    t = 999.0
    e = R.timestep_embedding(torch.tensor([t]))[0].double().numpy()
    for i in (0, 1, 80, 159):
        f = math.exp(-math.log(10000.0) * i / 160)
        assert abs(e[i] - math.cos(t * f)) < 1e-6 and abs(e[160 + i] - math.sin(t * f)) < 1e-6


def test_weight_inventory_matches_sd15():
    inv = W.inventory()
    assert len(inv) == 686
    assert W.param_count() == 859520964
    keys = {k for k, _, _ in inv}
    assert "up_blocks.3.attentions.2.transformer_blocks.0.attn2.to_k.weight" in keys
    assert "down_blocks.1.resnets.0.conv_shortcut.weight" in keys


def test_reference_layout_roundtrip(tmp_path):
    g = torch.Generator().manual_seed(1)
    w = {"a.to_q.weight": torch.randn(4, 6, generator=g).half(), "a.conv.weight": torch.randn(3, 2, 3, 3, generator=g).half(),
         "a.norm.bias": torch.randn(5, generator=g).half()}
    arr = W.to_reference_layout("a.to_q.weight", w["a.to_q.weight"])
    assert arr.shape == (6, 4)                      # Linear stored [in,out]
    back = W.from_reference_layout("a.to_q.weight", arr.reshape(-1), (4, 6))
    assert torch.equal(back, w["a.to_q.weight"])
    conv = W.to_reference_layout("a.conv.weight", w["a.conv.weight"])
    assert conv.shape == (3, 2, 3, 3)               # conv untouched


def test_lcm_schedule_matches_reference():
    # LcmScheduler.kt: 4 steps -> [999, 759, 499, 259]
    s = lcm.LcmScheduler(4)
    assert list(s.timesteps) == [999, 759, 499, 259]
    ac = s.alphas_cumprod
    assert abs(ac[0] - (1 - 0.00085)) < 1e-12 and 0 < ac[-1] < ac[0]


def test_lcm_step_identity_cases():
    s = lcm.LcmScheduler(2)
    lat = np.ones((1, 4, 2, 2), np.float32)
    eps = np.zeros_like(lat)
    noise = np.zeros_like(lat)
    out = s.step(lat.copy(), eps, noise)
    t = s.timesteps[0]
    a = s.alphas_cumprod[t]
    st = t * 10.0
    c_skip = 0.25 / (st * st + 0.25)
    c_out = st / math.sqrt(st * st + 0.25)
    den = c_out / math.sqrt(a) + c_skip
    a_prev = s.alphas_cumprod[s.timesteps[1]]
    assert np.allclose(out, math.sqrt(a_prev) * den, rtol=1e-6)


def test_cfg_only_first_steps_call_pattern():
    # TpuUnetPipeline.kt:97-104: steps idx < cfg_steps run [cond, uncond] pairs, later steps cond only
    calls = []

    def fake_unet(lat, t, ctx):
        calls.append((lat.shape[0], float(ctx[0, 0, 0])))
        return np.full_like(lat, 0.01)

    n, steps = 3, 4
    lat = np.zeros((n, 4, 8, 8), np.float32)
    cond = np.ones((n, 77, 768), np.float32)
    unc = -np.ones((n, 77, 768), np.float32)
    noise = np.zeros((steps - 1, n, 4, 8, 8), np.float32)
    lcm.cfg_denoise(fake_unet, lat, cond, unc, noise, steps=steps, cfg=1.5, cfg_steps=2)
    assert [c[0] for c in calls] == [2 * n, 2 * n, n, n]
    assert calls[2][1] == 1.0                       # cond-only steps see the cond context
    calls.clear()
    lcm.cfg_denoise(fake_unet, lat, cond, None, noise, steps=steps, cfg=1.0, cfg_steps=4)
    assert [c[0] for c in calls] == [n] * steps     # cfg <= 1: no guidance at all
