"""Readers for the reference's block known-answer fixtures (TEST INFRASTRUCTURE).

``rb``: ResnetBlock2D, C=320 -> 320, 64x64, temb 1280 (``VulkanBench.kt:54-64``,
``vk_engine.cpp:423-480``). ``tf``: Transformer2DModel, C=320, 64x64,
context 77x768, 8 heads (``VulkanBench.kt:39-52``, ``vk_engine.cpp:931-1012``).
All files raw fp16, batch 1, activations ``[C,H,W]``. Linear weights
(``tproj_wT``, ``q1``..``o2``, ``geglu``, ``ffout``) are ``[in,out]``; 1x1 conv
weights (``pin_w``, ``pout_w``) ``[Co,Ci]``; 3x3 conv weights ``[Co,Ci,3,3]``.

Each loader returns a weight dict under a synthetic diffusers-style prefix
(``rb`` / ``tf``) in PyTorch layout, so the same oracle block functions and
the same engine upload path consume it.
"""
from __future__ import annotations

import os
from typing import Dict, Tuple

import numpy as np
import torch

GOLDEN = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "tests", "golden")


def _f16(path: str, shape) -> torch.Tensor:
    a = np.fromfile(path, dtype=np.float16)
    assert a.size == int(np.prod(shape)), (path, a.size, shape)
    return torch.from_numpy(a.reshape(shape).copy())


def load_rb(root: str = GOLDEN, C: int = 320, H: int = 64, W: int = 64, T: int = 1280):
    """-> (x [1,C,H,W], temb [1,T], weights{'rb.*'}, y [1,C,H,W]); fp16 tensors."""
    d = os.path.join(root, "rb")
    f = lambda n, s: _f16(os.path.join(d, n + ".bin"), s)
    w: Dict[str, torch.Tensor] = {
        "rb.norm1.weight": f("norm1_w", (C,)), "rb.norm1.bias": f("norm1_b", (C,)),
        "rb.conv1.weight": f("conv1_w", (C, C, 3, 3)), "rb.conv1.bias": f("conv1_b", (C,)),
        # tproj_wT is [in,out]; the PyTorch layout is its transpose (== tproj_w)
        "rb.time_emb_proj.weight": f("tproj_wT", (T, C)).T.contiguous(),
        "rb.time_emb_proj.bias": f("tproj_b", (C,)),
        "rb.norm2.weight": f("norm2_w", (C,)), "rb.norm2.bias": f("norm2_b", (C,)),
        "rb.conv2.weight": f("conv2_w", (C, C, 3, 3)), "rb.conv2.bias": f("conv2_b", (C,)),
    }
    x = f("x", (1, C, H, W))
    temb = f("temb", (1, T))
    y = f("y", (1, C, H, W))
    return x, temb, w, y


def load_tf(root: str = GOLDEN, C: int = 320, H: int = 64, W: int = 64, n_ctx: int = 77, d_ctx: int = 768):
    """-> (x [1,C,H,W], ctx [1,77,768], weights{'tf.*'}, y [1,C,H,W]); fp16."""
    d = os.path.join(root, "tf")
    f = lambda n, s: _f16(os.path.join(d, n + ".bin"), s)
    lin = lambda n, kin, kout: f(n, (kin, kout)).T.contiguous()   # [in,out] -> [out,in]
    b = "tf.transformer_blocks.0"
    w: Dict[str, torch.Tensor] = {
        "tf.norm.weight": f("gn_w", (C,)), "tf.norm.bias": f("gn_b", (C,)),
        "tf.proj_in.weight": f("pin_w", (C, C, 1, 1)), "tf.proj_in.bias": f("pin_b", (C,)),
        b + ".norm1.weight": f("n1_w", (C,)), b + ".norm1.bias": f("n1_b", (C,)),
        b + ".attn1.to_q.weight": lin("q1", C, C), b + ".attn1.to_k.weight": lin("k1", C, C),
        b + ".attn1.to_v.weight": lin("v1", C, C), b + ".attn1.to_out.0.weight": lin("o1", C, C),
        b + ".attn1.to_out.0.bias": f("o1_b", (C,)),
        b + ".norm2.weight": f("n2_w", (C,)), b + ".norm2.bias": f("n2_b", (C,)),
        b + ".attn2.to_q.weight": lin("q2", C, C), b + ".attn2.to_k.weight": lin("k2", d_ctx, C),
        b + ".attn2.to_v.weight": lin("v2", d_ctx, C), b + ".attn2.to_out.0.weight": lin("o2", C, C),
        b + ".attn2.to_out.0.bias": f("o2_b", (C,)),
        b + ".norm3.weight": f("n3_w", (C,)), b + ".norm3.bias": f("n3_b", (C,)),
        b + ".ff.net.0.proj.weight": lin("geglu", C, 8 * C), b + ".ff.net.0.proj.bias": f("geglu_b", (8 * C,)),
        b + ".ff.net.2.weight": lin("ffout", 4 * C, C), b + ".ff.net.2.bias": f("ffout_b", (C,)),
        "tf.proj_out.weight": f("pout_w", (C, C, 1, 1)), "tf.proj_out.bias": f("pout_b", (C,)),
    }
    x = f("x", (1, C, H, W))
    ctx = f("ctx", (1, n_ctx, d_ctx))
    y = f("y", (1, C, H, W))
    return x, ctx, w, y
