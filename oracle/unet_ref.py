"""fp32 PyTorch restatement of the reference SD1.5 UNet forward (TEST ORACLE).

Test infrastructure only: imported by ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py``'s CPU-baseline arm. The engine never routes through it.

Layouts follow the reference engine's math, not its memory layout: tensors are
NCHW fp32 here (the reference keeps ``[C, B*HW]``, ``vk_engine.cpp:542``; the
engine keeps NHWC fp16). Weights are a dict keyed by diffusers state-dict names
holding PyTorch-layout tensors (conv ``[Co,Ci,kh,kw]``, linear ``[out,in]``);
``oracle/weights.py`` converts from/to the reference's on-disk layout (linear
weights stored ``[in,out]``).

Every function cites the reference lines it restates.
"""
from __future__ import annotations

import math
from typing import Dict, List, Optional

import torch
import torch.nn.functional as F

Tensor = torch.Tensor
Weights = Dict[str, Tensor]

# SD1.5 UNet2DConditionModel configuration (vk_engine.cpp:721 channels, :727 heads=8).
BLOCK_OUT = (320, 640, 1280, 1280)
HEADS = 8
CTX_DIM = 768
CTX_LEN = 77
TEMB_DIM = 1280
RESNET_EPS = 1e-5        # groupnorm_silu eps (vk_engine.cpp:549)
TRANSFORMER_GN_EPS = 1e-6  # diffusers Transformer2DModel norm eps;
                           # the Vulkan engine hard-codes 1e-5 (vk_engine.cpp:548), the
                           # assets/tf KAT cannot tell the two apart.
LN_EPS = 1e-5            # layernorm eps (vk_engine.cpp:652,658,666)


def _w(w: Weights, key: str) -> Tensor:
    return w[key].float()


# ---------------------------------------------------------------- primitive ops

def timestep_embedding(t: Tensor, dim: int = 320) -> Tensor:
    """Sinusoid, cos first: ``VulkanUnetPipeline.kt:36-46`` (diffusers
    get_timestep_embedding, flip_sin_to_cos=True, shift 0). Computed in float64
    like the Kotlin caller, returned fp32. ``t``: [B] float."""
    half = dim // 2
    i = torch.arange(half, dtype=torch.float64)
    freq = torch.exp(-math.log(10000.0) * i / half)
    a = t.double()[:, None] * freq[None, :]
    return torch.cat([torch.cos(a), torch.sin(a)], dim=1).float()


def groupnorm(x: Tensor, gamma: Tensor, beta: Tensor, eps: float, silu: bool,
              groups: int = 32) -> Tensor:
    """GroupNorm(32) (+SiLU), stats per (image, group):
    ``groupnorm_f32.comp:12-28``, ``groupnorm_silu.comp:12-31``."""
    y = F.group_norm(x, groups, gamma, beta, eps)
    return F.silu(y) if silu else y


def layernorm(x: Tensor, gamma: Tensor, beta: Tensor, eps: float = LN_EPS) -> Tensor:
    """LayerNorm over the last dim: ``layernorm_f32.comp:9-17``."""
    return F.layer_norm(x, (x.shape[-1],), gamma, beta, eps)


def conv2d(x: Tensor, w: Tensor, b: Optional[Tensor], stride: int = 1, pad: Optional[int] = None) -> Tensor:
    """Direct convolution, pad = k//2 (``vk_engine.cpp:578-608``; downsample
    uses 3x3 s2 p1, ``:689-692``)."""
    k = w.shape[-1]
    if pad is None:
        pad = k // 2
    return F.conv2d(x, w, b, stride=stride, padding=pad)


def linear(x: Tensor, w: Tensor, b: Optional[Tensor] = None) -> Tensor:
    """``matmul(act, W[in,out])`` + ``addbias_l`` (``vk_engine.cpp:609-613``);
    here ``w`` is PyTorch ``[out,in]``."""
    return F.linear(x, w, b)


def attention(q: Tensor, k: Tensor, v: Tensor, heads: int) -> Tensor:
    """softmax(Q K^T / sqrt(d)) V per head, keys restricted to the query's own
    image (``attention_f32.comp:22-68``: ``seqQpi/seqKpi``, scale 1/sqrt(d)).
    q: [B, Sq, C], k/v: [B, Sk, C] -> [B, Sq, C]."""
    B, Sq, C = q.shape
    Sk = k.shape[1]
    d = C // heads
    qh = q.view(B, Sq, heads, d).transpose(1, 2)
    kh = k.view(B, Sk, heads, d).transpose(1, 2)
    vh = v.view(B, Sk, heads, d).transpose(1, 2)
    s = torch.matmul(qh, kh.transpose(-1, -2)) * (1.0 / math.sqrt(d))
    p = torch.softmax(s, dim=-1)
    o = torch.matmul(p, vh)
    return o.transpose(1, 2).reshape(B, Sq, C)


def geglu(h: Tensor) -> Tensor:
    """``geglu_f32.comp:11-14``: out = a * gelu_erf(gate), a = first half,
    gate = second half of the FF-proj output."""
    a, gate = h.chunk(2, dim=-1)
    return a * F.gelu(gate)


def upsample2x(x: Tensor) -> Tensor:
    """Nearest 2x, per image: ``upsample_f32.comp:7-11``."""
    return F.interpolate(x, scale_factor=2.0, mode="nearest")


# ---------------------------------------------------------------- blocks

def resnet_block(x: Tensor, temb: Tensor, w: Weights, pf: str) -> Tensor:
    """ResnetBlock2D, ``vk_engine.cpp:623-637``:
    GN+SiLU -> conv3x3+b -> + Linear(SiLU(temb)) -> GN+SiLU -> conv3x3+b ->
    (+ 1x1 shortcut if Cin != Cout) + residual. temb: [B, 1280]."""
    h = groupnorm(x, _w(w, pf + ".norm1.weight"), _w(w, pf + ".norm1.bias"), RESNET_EPS, True)
    h = conv2d(h, _w(w, pf + ".conv1.weight"), _w(w, pf + ".conv1.bias"))
    tp = linear(F.silu(temb), _w(w, pf + ".time_emb_proj.weight"), _w(w, pf + ".time_emb_proj.bias"))
    h = h + tp[:, :, None, None]
    h = groupnorm(h, _w(w, pf + ".norm2.weight"), _w(w, pf + ".norm2.bias"), RESNET_EPS, True)
    h = conv2d(h, _w(w, pf + ".conv2.weight"), _w(w, pf + ".conv2.bias"))
    sc_key = pf + ".conv_shortcut.weight"
    if sc_key in w:
        x = conv2d(x, _w(w, sc_key), _w(w, pf + ".conv_shortcut.bias"))
    return x + h


def transformer_block(x: Tensor, ctx: Tensor, w: Weights, pf: str, heads: int = HEADS,
                      gn_eps: float = TRANSFORMER_GN_EPS) -> Tensor:
    """Transformer2DModel (SpatialTransformer) with one BasicTransformerBlock,
    ``vk_engine.cpp:640-675``: GN -> proj_in 1x1 -> [LN -> self-attn -> out+res]
    -> [LN -> cross-attn(ctx) -> out+res] -> [LN -> GEGLU FF -> out+res] ->
    proj_out 1x1 -> + x. ctx: [B, 77, 768]."""
    B, C, H, W = x.shape
    h = groupnorm(x, _w(w, pf + ".norm.weight"), _w(w, pf + ".norm.bias"), gn_eps, False)
    h = conv2d(h, _w(w, pf + ".proj_in.weight"), _w(w, pf + ".proj_in.bias"))
    t = h.permute(0, 2, 3, 1).reshape(B, H * W, C)          # T_CH (vk_engine.cpp:645)
    b = pf + ".transformer_blocks.0"
    # self-attention (:652-656)
    hn = layernorm(t, _w(w, b + ".norm1.weight"), _w(w, b + ".norm1.bias"))
    q = linear(hn, _w(w, b + ".attn1.to_q.weight"))
    k = linear(hn, _w(w, b + ".attn1.to_k.weight"))
    v = linear(hn, _w(w, b + ".attn1.to_v.weight"))
    a = attention(q, k, v, heads)
    t = t + linear(a, _w(w, b + ".attn1.to_out.0.weight"), _w(w, b + ".attn1.to_out.0.bias"))
    # cross-attention (:658-664)
    hn = layernorm(t, _w(w, b + ".norm2.weight"), _w(w, b + ".norm2.bias"))
    q = linear(hn, _w(w, b + ".attn2.to_q.weight"))
    k = linear(ctx, _w(w, b + ".attn2.to_k.weight"))
    v = linear(ctx, _w(w, b + ".attn2.to_v.weight"))
    a = attention(q, k, v, heads)
    t = t + linear(a, _w(w, b + ".attn2.to_out.0.weight"), _w(w, b + ".attn2.to_out.0.bias"))
    # GEGLU feed-forward (:666-669)
    hn = layernorm(t, _w(w, b + ".norm3.weight"), _w(w, b + ".norm3.bias"))
    g = linear(hn, _w(w, b + ".ff.net.0.proj.weight"), _w(w, b + ".ff.net.0.proj.bias"))
    t = t + linear(geglu(g), _w(w, b + ".ff.net.2.weight"), _w(w, b + ".ff.net.2.bias"))
    # proj_out + residual (:671-674)
    t = t.reshape(B, H, W, C).permute(0, 3, 1, 2)
    po = conv2d(t, _w(w, pf + ".proj_out.weight"), _w(w, pf + ".proj_out.bias"))
    return x + po


def time_mlp(temb_proj: Tensor, w: Weights) -> Tensor:
    """time_embedding MLP, ``vk_engine.cpp:716-717``: Linear 320->1280, SiLU,
    Linear 1280->1280."""
    t1 = F.silu(linear(temb_proj, _w(w, "time_embedding.linear_1.weight"), _w(w, "time_embedding.linear_1.bias")))
    return linear(t1, _w(w, "time_embedding.linear_2.weight"), _w(w, "time_embedding.linear_2.bias"))


# ---------------------------------------------------------------- full graph

def unet_forward(latent: Tensor, timesteps: Tensor, context: Tensor, w: Weights) -> Tensor:
    """Full SD1.5 UNet forward, ``vk_engine.cpp:711-790`` (mode 0).

    latent [B,4,H,W] fp32 (H, W multiples of 8), timesteps [B] or [1],
    context [B,77,768]. Returns eps [B,4,H,W] fp32.
    """
    B = latent.shape[0]
    if timesteps.numel() == 1:
        timesteps = timesteps.reshape(1).expand(B)
    temb = time_mlp(timestep_embedding(timesteps), w)
    x = conv2d(latent, _w(w, "conv_in.weight"), _w(w, "conv_in.bias"))
    skips: List[Tensor] = [x]
    cprev = 320
    for i in range(4):
        cout = BLOCK_OUT[i]
        for r in range(2):
            x = resnet_block(x, temb, w, f"down_blocks.{i}.resnets.{r}")
            if i < 3:
                x = transformer_block(x, context, w, f"down_blocks.{i}.attentions.{r}")
            skips.append(x)
        if i < 3:
            x = conv2d(x, _w(w, f"down_blocks.{i}.downsamplers.0.conv.weight"),
                       _w(w, f"down_blocks.{i}.downsamplers.0.conv.bias"), stride=2, pad=1)
            skips.append(x)
        cprev = cout
    x = resnet_block(x, temb, w, "mid_block.resnets.0")
    x = transformer_block(x, context, w, "mid_block.attentions.0")
    x = resnet_block(x, temb, w, "mid_block.resnets.1")
    for i in range(4):
        for r in range(3):
            skip = skips.pop()
            x = torch.cat([x, skip], dim=1)                     # concat [prev ; skip] (:677-688)
            x = resnet_block(x, temb, w, f"up_blocks.{i}.resnets.{r}")
            if i > 0:
                x = transformer_block(x, context, w, f"up_blocks.{i}.attentions.{r}")
        if i < 3:
            x = upsample2x(x)
            x = conv2d(x, _w(w, f"up_blocks.{i}.upsamplers.0.conv.weight"),
                       _w(w, f"up_blocks.{i}.upsamplers.0.conv.bias"))
    x = groupnorm(x, _w(w, "conv_norm_out.weight"), _w(w, "conv_norm_out.bias"), RESNET_EPS, True)
    return conv2d(x, _w(w, "conv_out.weight"), _w(w, "conv_out.bias"))


def rel_err_l1(got: Tensor, ref: Tensor) -> float:
    """relErr = sum|got-ref| / sum|ref| (``vk_engine.cpp:698-704``,
    ``tools/run_ref.py:46``), over all elements."""
    got = got.double()
    ref = ref.double()
    return float((got - ref).abs().sum() / (ref.abs().sum() + 1e-12))
