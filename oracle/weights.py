"""SD1.5 UNet weight inventory, seeded init and the reference's on-disk format
(TEST INFRASTRUCTURE: used by tests and bench to make inputs; the engine reads
the same format through its own C++ loader).

Reference format (``vk_engine.cpp:497-507``, ``README.md:293``): one raw
little-endian fp16 file per diffusers state-dict key, ``<dir>/<key>.bin``, no
header. Conv weights ``[Co,Ci,kh,kw]``; norm weights ``[C]``; every Linear
weight is stored TRANSPOSED, ``[in,out]`` (``matmul(act, W[K,N])``,
``vk_engine.cpp:629,653,661,667,669,716-717``; ``assets/rb/tproj_wT.bin`` is
``tproj_w.bin`` transposed).
"""
from __future__ import annotations

import math
import os
from collections import OrderedDict
from typing import Dict, Iterator, List, Tuple

import numpy as np
import torch

from .unet_ref import BLOCK_OUT, CTX_DIM, TEMB_DIM

Shape = Tuple[int, ...]


def _resnet(pf: str, cin: int, cout: int) -> List[Tuple[str, Shape, str]]:
    out = [
        (pf + ".norm1.weight", (cin,), "norm_w"), (pf + ".norm1.bias", (cin,), "norm_b"),
        (pf + ".conv1.weight", (cout, cin, 3, 3), "conv"), (pf + ".conv1.bias", (cout,), "bias:%d" % (cin * 9)),
        (pf + ".time_emb_proj.weight", (cout, TEMB_DIM), "linear"), (pf + ".time_emb_proj.bias", (cout,), "bias:%d" % TEMB_DIM),
        (pf + ".norm2.weight", (cout,), "norm_w"), (pf + ".norm2.bias", (cout,), "norm_b"),
        (pf + ".conv2.weight", (cout, cout, 3, 3), "conv"), (pf + ".conv2.bias", (cout,), "bias:%d" % (cout * 9)),
    ]
    if cin != cout:
        out += [(pf + ".conv_shortcut.weight", (cout, cin, 1, 1), "conv"),
                (pf + ".conv_shortcut.bias", (cout,), "bias:%d" % cin)]
    return out


def _transformer(pf: str, c: int) -> List[Tuple[str, Shape, str]]:
    b = pf + ".transformer_blocks.0"
    out = [
        (pf + ".norm.weight", (c,), "norm_w"), (pf + ".norm.bias", (c,), "norm_b"),
        (pf + ".proj_in.weight", (c, c, 1, 1), "conv"), (pf + ".proj_in.bias", (c,), "bias:%d" % c),
    ]
    for n in ("norm1", "norm2", "norm3"):
        out += [(f"{b}.{n}.weight", (c,), "norm_w"), (f"{b}.{n}.bias", (c,), "norm_b")]
    for a, kv in (("attn1", c), ("attn2", CTX_DIM)):
        out += [(f"{b}.{a}.to_q.weight", (c, c), "linear"),
                (f"{b}.{a}.to_k.weight", (c, kv), "linear"),
                (f"{b}.{a}.to_v.weight", (c, kv), "linear"),
                (f"{b}.{a}.to_out.0.weight", (c, c), "linear"),
                (f"{b}.{a}.to_out.0.bias", (c,), "bias:%d" % c)]
    out += [(f"{b}.ff.net.0.proj.weight", (8 * c, c), "linear"), (f"{b}.ff.net.0.proj.bias", (8 * c,), "bias:%d" % c),
            (f"{b}.ff.net.2.weight", (c, 4 * c), "linear"), (f"{b}.ff.net.2.bias", (c,), "bias:%d" % (4 * c))]
    out += [(pf + ".proj_out.weight", (c, c, 1, 1), "conv"), (pf + ".proj_out.bias", (c,), "bias:%d" % c)]
    return out


def inventory() -> List[Tuple[str, Shape, str]]:
    """Every UNet parameter as (diffusers key, PyTorch shape, kind), in graph
    order (``vk_engine.cpp:711-790``). kind: conv | linear | norm_w | norm_b |
    bias:<fan_in>."""
    inv: List[Tuple[str, Shape, str]] = [
        ("time_embedding.linear_1.weight", (TEMB_DIM, 320), "linear"),
        ("time_embedding.linear_1.bias", (TEMB_DIM,), "bias:320"),
        ("time_embedding.linear_2.weight", (TEMB_DIM, TEMB_DIM), "linear"),
        ("time_embedding.linear_2.bias", (TEMB_DIM,), "bias:%d" % TEMB_DIM),
        ("conv_in.weight", (320, 4, 3, 3), "conv"), ("conv_in.bias", (320,), "bias:36"),
    ]
    cprev = 320
    for i in range(4):
        cout = BLOCK_OUT[i]
        for r in range(2):
            inv += _resnet(f"down_blocks.{i}.resnets.{r}", cprev if r == 0 else cout, cout)
            if i < 3:
                inv += _transformer(f"down_blocks.{i}.attentions.{r}", cout)
        if i < 3:
            inv += [(f"down_blocks.{i}.downsamplers.0.conv.weight", (cout, cout, 3, 3), "conv"),
                    (f"down_blocks.{i}.downsamplers.0.conv.bias", (cout,), "bias:%d" % (cout * 9))]
        cprev = cout
    inv += _resnet("mid_block.resnets.0", 1280, 1280)
    inv += _transformer("mid_block.attentions.0", 1280)
    inv += _resnet("mid_block.resnets.1", 1280, 1280)
    # up path channel bookkeeping (skip LIFO, vk_engine.cpp:748-779)
    skip_ch = [320, 320, 320, 320, 640, 640, 640, 1280, 1280, 1280, 1280, 1280]
    up_out = (1280, 1280, 640, 320)
    cprev = 1280
    for i in range(4):
        cout = up_out[i]
        for r in range(3):
            cs = skip_ch.pop()
            inv += _resnet(f"up_blocks.{i}.resnets.{r}", cprev + cs, cout)
            cprev = cout
            if i > 0:
                inv += _transformer(f"up_blocks.{i}.attentions.{r}", cout)
        if i < 3:
            inv += [(f"up_blocks.{i}.upsamplers.0.conv.weight", (cout, cout, 3, 3), "conv"),
                    (f"up_blocks.{i}.upsamplers.0.conv.bias", (cout,), "bias:%d" % (cout * 9))]
    inv += [("conv_norm_out.weight", (320,), "norm_w"), ("conv_norm_out.bias", (320,), "norm_b"),
            ("conv_out.weight", (4, 320, 3, 3), "conv"), ("conv_out.bias", (4,), "bias:2880")]
    return inv


def make_weights(seed: int = 0) -> "OrderedDict[str, torch.Tensor]":
    """Seeded PyTorch-default init, stored fp16: conv and
    linear weights kaiming_uniform(a=sqrt(5)) == U(-1/sqrt(fan_in), +), biases
    U(-1/sqrt(fan_in), +), norm gamma=1 beta=0. PyTorch layout."""
    g = torch.Generator().manual_seed(seed)
    out: "OrderedDict[str, torch.Tensor]" = OrderedDict()
    for key, shape, kind in inventory():
        if kind == "norm_w":
            t = torch.ones(shape)
        elif kind == "norm_b":
            t = torch.zeros(shape)
        else:
            fan_in = int(kind.split(":")[1]) if kind.startswith("bias:") else int(np.prod(shape[1:]))
            bound = 1.0 / math.sqrt(fan_in)
            t = (torch.rand(shape, generator=g) * 2.0 - 1.0) * bound
        out[key] = t.half()
    return out


def is_linear(key: str, ndim: int) -> bool:
    """True for Linear weights (stored transposed in the reference format)."""
    return ndim == 2 and key.endswith(".weight")


def to_reference_layout(key: str, t: torch.Tensor) -> np.ndarray:
    """PyTorch-layout fp16 tensor -> the array the reference stores in
    ``<key>.bin`` (Linear transposed to ``[in,out]``)."""
    a = t.detach().cpu().half().numpy()
    if is_linear(key, a.ndim):
        a = np.ascontiguousarray(a.T)
    return a


def from_reference_layout(key: str, a: np.ndarray, shape: Shape) -> torch.Tensor:
    """Inverse of :func:`to_reference_layout`; ``shape`` is the PyTorch shape."""
    if len(shape) == 2 and key.endswith(".weight"):
        return torch.from_numpy(a.reshape(shape[1], shape[0]).T.copy())
    return torch.from_numpy(a.reshape(shape).copy())


def save_reference_dir(w: Dict[str, torch.Tensor], d: str) -> None:
    """Write the reference's ``unet_w/`` directory format."""
    os.makedirs(d, exist_ok=True)
    for k, t in w.items():
        to_reference_layout(k, t).tofile(os.path.join(d, k + ".bin"))


def load_reference_dir(d: str) -> "OrderedDict[str, torch.Tensor]":
    out: "OrderedDict[str, torch.Tensor]" = OrderedDict()
    for key, shape, _ in inventory():
        a = np.fromfile(os.path.join(d, key + ".bin"), dtype=np.float16)
        out[key] = from_reference_layout(key, a, shape)
    return out


def iter_reference_blobs(w: Dict[str, torch.Tensor]) -> Iterator[Tuple[str, np.ndarray]]:
    """(key, reference-layout contiguous fp16 array) pairs, for uploading
    through ``sdg_upload_weight`` without touching disk."""
    for k, t in w.items():
        yield k, to_reference_layout(k, t)


def param_count() -> int:
    return int(sum(np.prod(s) for _, s, _ in inventory()))


def make_inputs(B: int = 2, H: int = 64, W: int = 64, seed: int = 0, timestep: float = 999.0):
    """BASELINE config 0 inputs: latent ~N(0,1) [B,4,H,W]; timestep (999);
    context ~N(0,1) [B,77,768] then LayerNorm per token (no affine)."""
    g = torch.Generator().manual_seed(seed)
    latent = torch.randn((B, 4, H, W), generator=g)
    ctx = torch.randn((B, 77, CTX_DIM), generator=g)
    ctx = torch.nn.functional.layer_norm(ctx, (CTX_DIM,))
    t = torch.full((B,), float(timestep))
    return latent, t, ctx
