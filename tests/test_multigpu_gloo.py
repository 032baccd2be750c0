"""Batch sharding and the final-latent gather on CPU
ranks with the gloo backend (world size 2 and 3), plus the failure path: a
rank that dies before the gather makes the others' gather fail with an error
(short process-group timeout) instead of hanging."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from conftest import load_pkg


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _fake_denoise(lat, cond, unc, noise, steps=4, cfg=1.5):
    # stands in for Engine.lcm_denoise: any per-image deterministic function
    return (lat * 0.5 + cond.mean(axis=(1, 2))[:, None, None, None] - cfg * unc.mean(axis=(1, 2))[:, None, None, None]
            + (0 if noise is None else noise.sum(0))).astype(np.float32)


def _inputs(n, H=8):
    g = np.random.default_rng(5)
    lat = g.standard_normal((n, 4, H, H)).astype(np.float32)
    cond = g.standard_normal((n, 77, 16)).astype(np.float32)
    unc = g.standard_normal((n, 77, 16)).astype(np.float32)
    noise = g.standard_normal((3, n, 4, H, H)).astype(np.float32)
    return lat, cond, unc, noise


def _worker(rank, world, port, n, q, fail_rank):
    import datetime
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=15))
    mg = load_pkg().multigpu
    lat, cond, unc, noise = _inputs(n)
    try:
        if rank == fail_rank:
            raise RuntimeError("injected failure before the gather")
        out = mg.lcm_generate(_fake_denoise, lat, cond, unc, noise, chunk=2)
        q.put((rank, "ok", out))
    except Exception as e:  # report instead of hanging the test
        q.put((rank, "error", repr(e)))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(world, n, fail_rank=-1):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, n, q, fail_rank)) for r in range(world)]
    for p in ps:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in ps:
        p.join(timeout=60)
    return sorted(res, key=lambda r: r[0])


def test_shard_covers_batch_exactly():
    mg = load_pkg().multigpu
    for n in (0, 1, 7, 8, 16, 64):
        for w in (1, 2, 3, 4, 8):
            parts = [mg.shard(n, w, r) for r in range(w)]
            assert sum(c for _, c in parts) == n
            assert all(parts[r][0] + parts[r][1] == parts[r + 1][0] for r in range(w - 1))
            assert max(c for _, c in parts) - min(c for _, c in parts) <= 1


@pytest.mark.parametrize("world,n", [(2, 8), (3, 7)])
def test_gather_matches_single_process(world, n):
    res = _run(world, n)
    lat, cond, unc, noise = _inputs(n)
    ref = _fake_denoise(lat, cond, unc, noise)
    for rank, status, out in res:
        assert status == "ok", out
        assert np.allclose(out, ref)


def test_rank_failure_surfaces_as_error():
    res = _run(2, 4, fail_rank=1)
    assert res[1][1] == "error" and "injected" in res[1][2]
    assert res[0][1] == "error"          # the survivor's gather ended with an error, not a hang
