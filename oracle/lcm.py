"""LCM scheduler + batch-CFG denoise loop (TEST ORACLE for BASELINE config 3).

Restates ``sd/LcmScheduler.kt:13-97`` (diffusers LCMScheduler port:
epsilon prediction, 1000 train steps, 50 original inference steps,
timestep_scaling 10, sigma_data 0.5) and the caller loop of
``sd/VulkanUnetPipeline.kt:76-90`` (one batch-CFG forward per step,
``eps = uncond + cfg * (cond - uncond)``, re-noise between steps).
Arithmetic is float64 like the Kotlin code; latents are float32.
"""
from __future__ import annotations

import math
from typing import Callable, List, Optional

import numpy as np


class LcmScheduler:
    def __init__(self, n_steps: int, n_train: int = 1000, original_steps: int = 50, timestep_scaling: float = 10.0):
        # alphas_cumprod: scaled-linear betas (LcmScheduler.kt:29-38)
        b0, b1 = math.sqrt(0.00085), math.sqrt(0.012)
        ac = np.empty(n_train, dtype=np.float64)
        acc = 1.0
        for i in range(n_train):
            b = (b0 + (b1 - b0) * i / (n_train - 1)) ** 2
            acc *= 1.0 - b
            ac[i] = acc
        self.alphas_cumprod = ac
        # timesteps (LcmScheduler.kt:41-47)
        k = n_train // original_steps
        origin = [(i + 1) * k - 1 for i in range(original_steps)]
        rev = origin[::-1]
        self.timesteps = [rev[int(math.floor(i * len(rev) / n_steps))] for i in range(n_steps)]
        self.n_steps = n_steps
        self.scaling = timestep_scaling
        self.sigma_data = 0.5
        self.step_count = 0

    def coefficients(self, i: int):
        """(c_skip, c_out, sqrt_a, sqrt_b, sqrt_a_prev, sqrt_b_prev, last) of step i
        (LcmScheduler.kt:57-67)."""
        t = self.timesteps[i]
        a = self.alphas_cumprod[t]
        st = t * self.scaling
        sd2 = self.sigma_data ** 2
        c_skip = sd2 / (st * st + sd2)
        c_out = st / math.sqrt(st * st + sd2)
        last = i == self.n_steps - 1
        a_prev = 1.0 if last else self.alphas_cumprod[self.timesteps[i + 1]]
        return c_skip, c_out, math.sqrt(a), math.sqrt(1 - a), math.sqrt(a_prev), math.sqrt(1 - a_prev), last

    def step(self, latents: np.ndarray, eps: np.ndarray, noise: Optional[np.ndarray]) -> np.ndarray:
        """One LCM update (LcmScheduler.kt:68-82)."""
        c_skip, c_out, sa, sb, sap, sbp, last = self.coefficients(self.step_count)
        x = latents.astype(np.float64)
        x0 = (x - sb * eps.astype(np.float64)) / sa
        den = c_out * x0 + c_skip * x
        out = den if last else sap * den + sbp * noise.astype(np.float64)
        self.step_count += 1
        return out.astype(np.float32)


def cfg_denoise(unet: Callable[[np.ndarray, float, np.ndarray], np.ndarray], latents: np.ndarray, cond: np.ndarray,
                uncond: Optional[np.ndarray], step_noise: Optional[np.ndarray], steps: int = 4, cfg: float = 1.5,
                cfg_steps: Optional[int] = None) -> np.ndarray:
    """Batch-CFG LCM loop over n images (VulkanUnetPipeline.kt:76-90).

    unet(lat [B,4,H,W], t, ctx [B,77,768]) -> eps [B,4,H,W]; per image the
    forward batch is [cond, uncond]. step_noise: [steps-1, n, 4, H, W].
    cfg_steps: guidance only on the first cfg_steps steps, cond-only eps after
    them, none at cfg <= 1 (TpuUnetPipeline.kt:97-104); None = every step."""
    n = latents.shape[0]
    sched = LcmScheduler(steps)
    lat = latents.astype(np.float32).copy()
    guided_steps = steps if cfg_steps is None else cfg_steps
    if cfg <= 1.0:
        guided_steps = 0
    for i, t in enumerate(sched.timesteps):
        if i >= guided_steps:
            eps = unet(lat, float(t), cond)
        else:
            lat2 = np.repeat(lat, 2, axis=0)                               # [cond, uncond] per image
            ctx2 = np.stack([cond, uncond], axis=1).reshape((2 * n,) + cond.shape[1:])
            eps2 = unet(lat2, float(t), ctx2).reshape((n, 2) + lat.shape[1:])
            eps = eps2[:, 1] + np.float32(cfg) * (eps2[:, 0] - eps2[:, 1])
        noise = None if i == steps - 1 else step_noise[i]
        lat = sched.step(lat, eps, noise)
    return lat
