"""Host logic of the folded upsample block (no GPU): the reference's upsample() is nearest 2x followed by a
3x3 pad-1 conv (vk_engine.cpp:693-697, upsample_f32.comp). The engine runs it as four 2x2 convolutions of
the low-resolution input, one per output phase (py, px), with the 3x3 taps folded per phase by
``sdg_pack_upsample_conv_weights``. Checked here: the C ABI's packing bit for bit against a numpy
restatement, and the folding itself (in fp32, unrounded) against the oracle's upsample + conv."""
import ctypes

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import unet_ref as R

# 3x3 taps (ky or kx) folded into 2x2 tap t of output phase q: output row 2i + q reads input rows
# i + t + q - 1, which the upsampled image holds at rows 2i + q - 1 + k, k = 0, 1, 2
FOLD = {(0, 0): [0], (0, 1): [1, 2], (1, 0): [0, 1], (1, 1): [2]}


def fold_weights(w3: np.ndarray, dtype=np.float32) -> np.ndarray:
    """[Co, Ci, 3, 3] -> [4 phases, Co, 4 taps, Ci], summed in fp32 in (ky, kx) order."""
    Co, Ci = w3.shape[:2]
    w = w3.astype(np.float32)
    out = np.zeros((4, Co, 4, Ci), dtype=np.float32)
    for ph in range(4):
        py, px = ph >> 1, ph & 1
        for tap in range(4):
            ty, tx = tap >> 1, tap & 1
            acc = np.zeros((Co, Ci), dtype=np.float32)
            for ky in FOLD[(py, ty)]:
                for kx in FOLD[(px, tx)]:
                    acc = acc + w[:, :, ky, kx]
            out[ph, :, tap, :] = acc
    return out.astype(dtype)


def phase_conv(x: torch.Tensor, wp: torch.Tensor, bias: torch.Tensor) -> torch.Tensor:
    """The folded computation in fp32: output pixel (2i + py, 2j + px) = sum over the 2x2 taps (ty, tx)
    of wp[ph, :, 2 ty + tx, :] . x[i + ty + py - 1, j + tx + px - 1] (zero outside the input)."""
    B, Ci, H, W = x.shape
    Co = wp.shape[1]
    xp = F.pad(x, (1, 1, 1, 1))
    y = torch.empty(B, Co, 2 * H, 2 * W, dtype=x.dtype)
    for ph in range(4):
        py, px = ph >> 1, ph & 1
        k = wp[ph].reshape(Co, 2, 2, Ci).permute(0, 3, 1, 2)  # [Co, Ci, ty, tx]
        y[:, :, py::2, px::2] = F.conv2d(xp[:, :, py:py + H + 1, px:px + W + 1], k, bias)
    return y


def test_packed_weights_match_restatement_bit_for_bit(sdg):
    g = np.random.default_rng(7)
    for Co, Ci in [(64, 64), (128, 192), (1280, 64)]:
        w3 = (g.standard_normal((Co, Ci, 3, 3)) * 0.05).astype(np.float16)
        got = sdg.pack_upsample_conv_weight(w3)
        want = fold_weights(w3, np.float16)
        assert got.shape == (4, Co, 4, Ci)
        assert np.array_equal(got.view(np.uint16), want.view(np.uint16))


@pytest.mark.parametrize("B,Ci,Co,H,W", [(2, 8, 6, 4, 4), (1, 5, 3, 1, 1), (3, 4, 7, 5, 3)])
def test_phase_folding_equals_upsample_then_conv(B, Ci, Co, H, W):
    g = torch.Generator().manual_seed(B * 100 + H * 10 + W)
    x = torch.randn(B, Ci, H, W, generator=g, dtype=torch.float64)
    w3 = torch.randn(Co, Ci, 3, 3, generator=g, dtype=torch.float64)
    b = torch.randn(Co, generator=g, dtype=torch.float64)
    ref = F.conv2d(R.upsample2x(x), w3, b, padding=1)
    wp = torch.from_numpy(fold_weights(w3.numpy(), np.float64).astype(np.float64))
    # exact identity up to fp64 summation order (the fold sums in fp32 first, so compare loosely)
    got = phase_conv(x, wp, b)
    assert torch.allclose(got, ref, rtol=1e-5, atol=1e-5)


def test_bad_arguments_are_rejected_without_gpu(sdg):
    L = sdg.lib()
    buf = (ctypes.c_uint16 * 64)()
    ERR_ARG, ERR_SHAPE = 2, 3
    assert L.sdg_pack_upsample_conv_weights(None, 4, 4, buf) == ERR_ARG
    assert L.sdg_pack_upsample_conv_weights(buf, 0, 4, buf) == ERR_ARG
    # Ci not a multiple of 64: refused before any device work
    assert L.sdg_upsample_conv3x3(buf, 1, 2, 2, 32, buf, None, 64, buf, None, 0, None, None) == ERR_SHAPE
    assert L.sdg_upsample_conv3x3(None, 1, 2, 2, 64, buf, None, 64, buf, None, 0, None, None) == ERR_ARG
