"""Data-parallel image generation across GPUs.

The workload shards by image: every rank (one process per GPU) holds a full
weight copy, denoises a contiguous slice of the batch with the 4-step LCM loop
(``Engine.lcm_denoise``: batch-CFG forwards, CFG combine and LCM update on the
device), and the final latents are all-gathered once — the only collective,
NCCL over NVLink/NVSwitch on GPUs (gloo on CPU in tests). The reference runs
the same loop for one image on one device (``sd/VulkanUnetPipeline.kt:76-90``).

Failure handling: the process group is created with a short timeout by the
caller; a rank that fails raises before the gather, so the others' gather
ends with a timeout error instead of hanging (no device-side waits involved).
"""
from __future__ import annotations

from typing import Callable, Optional, Tuple

import numpy as np


def shard(n: int, world: int, rank: int) -> Tuple[int, int]:
    """(start, count) of rank's contiguous share of n images; the first
    n % world ranks take one extra image."""
    if world <= 0 or not (0 <= rank < world) or n < 0:
        raise ValueError("bad shard arguments")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, base + (1 if rank < extra else 0)


def gather_latents(local: "np.ndarray", n_total: int, group=None, device=None) -> "np.ndarray":
    """All-gather the per-rank latents [count, ...] into [n_total, ...] on
    every rank (ranks pad to the largest shard; padding is dropped)."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    per = [shard(n_total, world, r)[1] for r in range(world)]
    cap = max(per)
    item = local.shape[1:]
    buf = torch.zeros((cap,) + tuple(item), dtype=torch.float32, device=device)
    if local.shape[0]:
        buf[: local.shape[0]] = torch.as_tensor(local, dtype=torch.float32, device=device)
    outs = [torch.empty_like(buf) for _ in range(world)]
    dist.all_gather(outs, buf, group=group)
    parts = [outs[r][: per[r]].cpu().numpy() for r in range(world)]
    out = np.concatenate(parts, axis=0)
    assert out.shape[0] == n_total and rank >= 0
    return out


def lcm_generate(denoise: Callable[..., "np.ndarray"], latents: "np.ndarray", cond: "np.ndarray",
                 uncond: "np.ndarray", step_noise: Optional["np.ndarray"], steps: int = 4, cfg: float = 1.5,
                 group=None, device=None, chunk: int = 32, timings: Optional[dict] = None) -> "np.ndarray":
    """Denoise this rank's shard of the batch and gather every image's final latent.

    ``denoise(latents, cond, uncond, step_noise, steps=, cfg=)`` is normally
    ``Engine.lcm_denoise`` (which takes at most 32 images per call; larger
    shards are processed in chunks). ``latents``/``cond``/``uncond`` hold the
    whole batch; ``step_noise`` is [steps-1, n, 4, H, W] (host-generated per
    image so every rank count yields identical results). When ``timings`` is
    a dict it receives this rank's host wall-clock seconds of the denoise
    (``denoise_s``) and of the gather (``gather_s``)."""
    import time
    import torch.distributed as dist
    n = latents.shape[0]
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    s, c = shard(n, world, rank)
    t0 = time.perf_counter()
    outs = []
    for a in range(s, s + c, chunk):
        b = min(s + c, a + chunk)
        nz = None if step_noise is None else np.ascontiguousarray(step_noise[:, a:b])
        outs.append(denoise(latents[a:b], cond[a:b], uncond[a:b], nz, steps=steps, cfg=cfg))
    local = np.concatenate(outs, 0) if outs else np.zeros((0,) + latents.shape[1:], np.float32)
    t1 = time.perf_counter()
    out = local if world == 1 else gather_latents(local, n, group=group, device=device)
    if timings is not None:
        timings["denoise_s"] = t1 - t0
        timings["gather_s"] = time.perf_counter() - t1
    return out
