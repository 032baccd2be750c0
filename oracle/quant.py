"""Weight-only int8 (wo8) restatement — TEST INFRASTRUCTURE (the checker for
the engine's int8 path, never on the product path).

The reference quantises its exported model with ai-edge-quantizer's
``weight_only_wi8_afp32`` recipe (``tools/quantize_wo8.py:42-46``; ai-edge-quantizer
0.8.0 per ``tools/README.md:101`` — a third-party dependency that is not
vendored in the reference). Its per-tensor step, as patched in
``tools/quantize_wo8.py:22-31``: ``q = round(w / scale + zero_point)`` clipped to
the narrow signed range (symmetric 8-bit => [-127, 127]), zero_point 0. The
scale is per output channel, symmetric: ``max|w| / 127``, stored fp16
Rounding is NumPy ``rint`` (round half to even).
Parity of this scheme against the library itself is unpinned (the library is
absent); the tests pin it on hand-worked vectors.

Output channel = the PyTorch weight's first axis (conv ``[Co,Ci,kh,kw]`` and
Linear ``[out,in]``). A zero row gets scale 1 (all q = 0).
"""
from __future__ import annotations

from collections import OrderedDict
from typing import Dict, Tuple

import numpy as np
import torch

from .weights import inventory


def quantize_rows(w: np.ndarray) -> Tuple[np.ndarray, np.ndarray]:
    """[N, ...] float weight -> (q int8 [N, ...], scale float32 [N]) per output row."""
    a = np.asarray(w, dtype=np.float32).reshape(w.shape[0], -1)
    s = (np.abs(a).max(axis=1) / np.float32(127.0)).astype(np.float16).astype(np.float32)
    s[s == 0] = 1.0
    q = np.clip(np.rint(a / s[:, None]), -127, 127).astype(np.int8)
    return q.reshape(w.shape), s


def dequantize_rows(q: np.ndarray, s: np.ndarray) -> np.ndarray:
    return (q.reshape(q.shape[0], -1).astype(np.float32) * s[:, None]).reshape(q.shape)


def quantize_wo8(w: Dict[str, torch.Tensor]) -> "OrderedDict[str, torch.Tensor]":
    """The UNet weights with every conv / linear weight replaced by its
    dequantised wo8 value (fp32); norms and biases unchanged."""
    kinds = {k: kind for k, _, kind in inventory()}
    out: "OrderedDict[str, torch.Tensor]" = OrderedDict()
    for k, t in w.items():
        if kinds.get(k) in ("conv", "linear"):
            q, s = quantize_rows(t.float().numpy())
            out[k] = torch.from_numpy(dequantize_rows(q, s))
        else:
            out[k] = t
    return out
