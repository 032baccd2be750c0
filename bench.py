"""Benchmark of the SD1.5 UNet forward on B200 (driver contract).

One step = one UNet forward at BASELINE config 0: B=2 (a CFG cond/uncond
pair), 64x64 latent, 77x768 context, timestep 999, seeded default-init fp16
weights, synthetic seeded inputs. Each rank holds a full weight copy and runs
its own B=2 forwards (data parallel by batch, no collective on the hot path);
`value` is whole-job forwards/s over all ranks (max-over-ranks device time).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Under torchrun each rank binds cuda:LOCAL_RANK; NCCL is used only for the
barrier and the max-over-ranks reduction of the timing.
The reference arm (--impl reference) times the CPU oracle port of the
reference forward on the host cores (the reference's own Vulkan engine
cannot run on this box: no graphics stack).
"""
from __future__ import annotations

import argparse
import importlib
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "UNet fwd/s (B=2 CFG, 64×64 latent) at 1/2/4/8 B200; % dense-fp16 tensor peak"
UNIT = "fwd/s"
B, H, W = 2, 64, 64
FLOPS_PER_FWD = 1.606e12          # algorithmic FLOPs per B=2 64x64 forward (direct-conv count)
# DRAM bytes (read + write) per gemm_tc_kernel launch, averaged over the 210 GEMM launches (and 3 split-K
# reduce launches) of one B=2 64x64 forward, from a one-pass ncu launch list of this bench
# (dram__bytes_read.sum + dram__bytes_write.sum; profiles/forward_launches_b2_64x64.md): 2.73 GB per forward
GEMM_TRAFFIC_PER_LAUNCH = 12.98e6
GEMM_TRAFFIC_NOTE = ("ncu dram__bytes_read.sum + dram__bytes_write.sum of every GEMM launch of one forward "
                     "(split-K reduce launches included) / 210 GEMM launches; serialised replay, cold caches")
L2_FLUSH_BYTES = 256 << 20        # > 126 MB L2


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d.get("hbm_gbs", 6650.0), d.get("bf16_tflops", 1590.0), d.get("bf16_tflops_sustained", 1400.0), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons during the timed region."""

    FIELDS = "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active," \
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown," \
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.lines = []  # (arrival time, csv line)
        self.t = None
        self.t0 = self.t1 = 0.0

    def _read(self):
        for ln in iter(self.proc.stdout.readline, ""):
            self.lines.append((time.time(), ln))

    def start(self):
        """Start sampling every 50 ms; returns once the first sample has arrived (at most 3 s), so
        the samples kept (those arriving between start() and stop()) cover the timed region."""
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            deadline = time.time() + 3.0
            while not self.lines and time.time() < deadline:
                time.sleep(0.01)
        except FileNotFoundError:
            self.proc = None
        self.t0 = time.time()

    def stop(self):
        self.t1 = time.time()
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.t.join(timeout=2)
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ts, ln in self.lines:
            if ts < self.t0 or ts > self.t1 + 0.06:
                continue
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


def make_engine(sdg, device, wo8=False):
    from oracle import weights as Wt
    w = Wt.make_weights(0)
    eng = sdg.Engine(device)
    eng.upload_weights(Wt.iter_reference_blobs(w))
    if wo8:
        eng.quantize_wo8()
    eng.prepare()
    return eng, w


def cpu_oracle_forward_rate(w, threads, runs=3):
    """Time the fp32 oracle forward (config 0) on host cores: 1 warm-up forward, then the median
    of `runs` timed forwards; returns (fwd/s, sample str)."""
    import torch
    from oracle import unet_ref as R
    from oracle import weights as Wt
    torch.set_num_threads(threads)
    lat, t, ctx = Wt.make_inputs(B, H, W, seed=0)
    wf = {k: v.float() for k, v in w.items()}   # fp16-rounded weights held in fp32
    times = []
    with torch.no_grad():
        R.unet_forward(lat, t, ctx, wf)          # warm-up
        for _ in range(runs):
            t0 = time.perf_counter()
            R.unet_forward(lat, t, ctx, wf)
            times.append(time.perf_counter() - t0)
    med = statistics.median(times)
    return 1.0 / med, (f"median of {runs} full B=2 64x64 fp32 oracle forwards after 1 warm-up "
                       f"({', '.join(f'{x:.2f}' for x in times)} s)")


def run_reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    import torch
    from oracle import weights as Wt
    from oracle import unet_ref as R
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    w = Wt.make_weights(0)
    wf = {k: v.float() for k, v in w.items()}
    lat, t, ctx = Wt.make_inputs(B, H, W, seed=0)
    budget = float(os.environ.get("SDG_REF_BUDGET_S", "150"))
    with torch.no_grad():
        t0 = time.perf_counter()
        R.unet_forward(lat, t, ctx, wf)                      # one warm-up forward
        per = time.perf_counter() - t0
        steps = max(1, min(args.steps, int(budget / max(per, 1e-3))))
        t0 = time.perf_counter()
        for _ in range(steps):
            R.unet_forward(lat, t, ctx, wf)
        el = time.perf_counter() - t0
    v = steps / el
    sample = f"{steps} of {args.steps} requested steps (1 warm-up), each a full B=2 64x64 fp32 forward"
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": args.gpus, "steps": steps,
        "warmup": 1, "ms_per_step": 1000.0 * el / steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded, BASELINE config 0)",
        "config": reference_config(),
        "cpu_baseline": {"value": v, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "reference Vulkan engine unavailable on this box (no graphics stack); timed arm = CPU restatement "
                "of vk_engine.cpp runGraph (oracle/unet_ref.py) in PyTorch fp32 on all host threads",
    }))
    return 0


def reference_config():
    """The work the reference arm actually does: one B=2 forward per step in one CPU process (rank 0;
    under torchrun the other ranks exit without work)."""
    return {"workload": "SD1.5 UNet forward, B=2 CFG pair, 64x64 latent, 77x768 context, t=999 (BASELINE config 0)",
            "global_batch": 2, "latent": [H, W], "context": [77, 768],
            "parallelism": "one CPU process on rank 0, all host threads (other ranks do no work)"}


def config3_inputs(n, H3=64, steps=4):
    """BASELINE config 3 inputs for n images, identical on every rank: per-image seeded latent
    ~N(0,1), per-image seeded conditional context, one shared unconditional context (LayerNorm per
    token), and host-generated per-image noise for the re-noising between LCM steps."""
    lat = np.empty((n, 4, H3, H3), np.float32)
    cond = np.empty((n, 77, 768), np.float32)
    noise = np.empty((steps - 1, n, 4, H3, H3), np.float32)
    for i in range(n):
        g = np.random.default_rng(1000 + i)
        lat[i] = g.standard_normal((4, H3, H3), dtype=np.float32)
        c = g.standard_normal((77, 768), dtype=np.float32)
        cond[i] = (c - c.mean(-1, keepdims=True)) / np.sqrt(c.var(-1, keepdims=True) + 1e-5)
        noise[:, i] = g.standard_normal((steps - 1, 4, H3, H3), dtype=np.float32)
    u = np.random.default_rng(999).standard_normal((77, 768), dtype=np.float32)
    u = (u - u.mean(-1, keepdims=True)) / np.sqrt(u.var(-1, keepdims=True) + 1e-5)
    unc = np.ascontiguousarray(np.broadcast_to(u, (n, 77, 768)))
    return lat, cond, unc, noise


def run_config3(eng, sdg, dev, world, rank, sizes=(8, 16, 64), steps=4, cfg=1.5):
    """BASELINE config 3 across the ranks: batches of 8/16/64 images, each rank denoises its shard with
    the 4-step LCM loop through the host API (Engine.lcm_denoise: batch-CFG forwards, CFG combine and
    LCM update on the device, H2D/D2H of its shard included) and the final latents are all-gathered
    over NCCL (multigpu.lcm_generate). Host wall clock per rank between barriers, max over ranks; the
    gather's own time is reported beside. Rank 0 then recomputes every rank's shard alone (same
    chunking) and checks the gathered latents bit for bit."""
    import torch
    import torch.distributed as dist
    mg = sdg.multigpu
    out = {"timing": "host wall clock per rank (denoise via the host API from pinned host buffers + NCCL "
                     "all_gather), max over ranks, median of 3 runs after 1 warm-up",
           "steps": steps, "cfg": cfg, "forwards_per_image": 2 * steps, "batches": {}}
    def pinned(a):  # host inputs in page-locked memory, as the e2e leg uses (asynchronous H2D copies)
        t = torch.empty(a.shape, dtype=torch.float32, pin_memory=True)
        t.numpy()[...] = a
        return t.numpy()

    for n in sizes:
        lat, cond, unc, noise = (pinned(a) for a in config3_inputs(n, H, steps))
        mg.lcm_generate(eng.lcm_denoise, lat, cond, unc, noise, steps=steps, cfg=cfg, device=dev)  # warm-up
        runs = []  # three timed runs (every rank takes the same steps); the median run is reported
        for _ in range(3):
            if world > 1:
                dist.barrier()
            tm = {}
            t0 = time.perf_counter()
            got = mg.lcm_generate(eng.lcm_denoise, lat, cond, unc, noise, steps=steps, cfg=cfg, device=dev,
                                  timings=tm)
            tot = time.perf_counter() - t0
            v = torch.tensor([tot, tm["denoise_s"], tm["gather_s"]], dtype=torch.float64, device=dev)
            vmin = v.clone()
            if world > 1:
                dist.all_reduce(v, op=dist.ReduceOp.MAX)
                dist.all_reduce(vmin, op=dist.ReduceOp.MIN)
            runs.append((float(v[0]), float(v[1]), float(v[2]), float(vmin[1]), float(vmin[2])))
        runs.sort()
        tot, den, gat, den_min, gat_min = runs[1]
        # a rank's gather time = waiting for the slowest rank's denoise + the transfer itself: the
        # fastest rank's wait minus the spread of the denoise times bounds the transfer
        rec = {"images": n, "images_per_gpu": mg.shard(n, world, 0)[1], "s": tot, "images_per_s": n / tot,
               "s_runs": [round(r[0], 4) for r in runs],
               "unet_fwd_per_s": n * steps / tot, "denoise_s_max": den, "denoise_s_min": den_min,
               "gather_s_max": gat, "gather_s_min": gat_min, "gather_share": gat / tot,
               "limiter": ("straggler (denoise spread across ranks)" if world > 1 and den - den_min > gat_min
                           else ("gather" if world > 1 else "none (1 rank)"))}
        if rank == 0:
            ref = []
            for r in range(world):          # each rank's shard, recomputed here with the same chunking
                s0, c = mg.shard(n, world, r)
                for a in range(s0, s0 + c, 32):
                    b = min(s0 + c, a + 32)
                    ref.append(eng.lcm_denoise(lat[a:b], cond[a:b], unc[a:b], np.ascontiguousarray(noise[:, a:b]),
                                               steps=steps, cfg=cfg))
            ref = np.concatenate(ref, 0)
            rec["gathered_bit_identical_to_1gpu"] = bool(got.shape == ref.shape and np.array_equal(got, ref))
        out["batches"][str(n)] = rec
        if world > 1:
            dist.barrier()
    return out


def config_dict(n, wo8=False):
    wl = "SD1.5 UNet forward, B=2 CFG pair, 64x64 latent, 77x768 context, t=999 (BASELINE config 0)"
    if wo8:
        wl = wl.replace("config 0)", "config 4: weight-only int8, per-output-channel scales)")
    return {"workload": wl,
            "global_batch": 2 * n, "latent": [H, W], "context": [77, 768], "parallelism": f"dp{n} (weights replicated)",
            "l2": "256 MB L2 flush (memset) between timed steps, outside the timed events; weights 1.72 GB > L2"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--wo8", action="store_true", help="weight-only int8 engine (BASELINE config 4)")
    ap.add_argument("--no-config3", action="store_true", help="skip the config-3 LCM batches (8/16/64 images)")
    args = ap.parse_args()
    if args.impl == "reference":
        return run_reference_arm(args)

    import torch
    import torch.distributed as dist
    sdg = importlib.import_module("sd-vulkan-pixel10-tensor-g5_b200")
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)

    eng, wts = make_engine(sdg, local, args.wo8)
    from oracle import weights as Wt
    lat, t, ctx = Wt.make_inputs(B, H, W, seed=rank)
    d_lat, d_t, d_ctx = lat.to(dev), t.to(dev), ctx.to(dev)
    d_out = torch.empty_like(d_lat)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    stream = torch.cuda.Stream(device=dev)          # non-default stream: events and forwards share it
    torch.cuda.set_stream(stream)

    def step():
        eng.forward_device(d_lat, d_t, d_ctx, d_out, stream.cuda_stream)

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()

    # ---- timed region: K device-resident forwards, CUDA events per step, L2 flushed between steps
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    clocks = ClockSampler(local)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks.start()
    for i in range(args.steps):
        flush.zero_()
        starts[i].record(stream)
        step()
        ends[i].record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clk = clocks.stop()
    dev_ms = sum(s.elapsed_time(e) for s, e in zip(starts, ends))
    t_max = torch.tensor([dev_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t_max, op=dist.ReduceOp.MAX)
    dev_ms = float(t_max.item())
    ms_per_step = dev_ms / args.steps
    value = world * args.steps / (dev_ms / 1000.0)

    # ---- e2e: the public host API (pinned host inputs, H2D + forward + D2H per step)
    p_lat = torch.empty(lat.shape, dtype=torch.float32).pin_memory()
    p_ctx = torch.empty(ctx.shape, dtype=torch.float32).pin_memory()
    p_t = torch.empty(t.shape, dtype=torch.float32).pin_memory()
    p_lat.copy_(lat); p_ctx.copy_(ctx); p_t.copy_(t)
    n_lat, n_ctx, n_t = p_lat.numpy(), p_ctx.numpy(), p_t.numpy()
    for _ in range(2):
        eng.forward(n_lat, n_t, n_ctx)
    if world > 1:
        dist.barrier()
    e2e_steps = max(5, args.steps // 2)
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        out_host = eng.forward(n_lat, n_t, n_ctx)
    e2e_s = time.perf_counter() - t0
    te = torch.tensor([e2e_s], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_value = world * e2e_steps / float(te.item())
    h2d = n_lat.nbytes + n_ctx.nbytes + n_t.nbytes
    d2h = out_host.nbytes

    # ---- roofline of the dominant kernel, gemm_tc_kernel (every conv / linear launch of the forward, with
    # its split-K reduce launches): the forward's launches of a category are recorded with their arguments
    # and replayed alone as a CUDA graph, back to back, between two CUDA events on the engine's stream
    # (sdg_profile_category) -- no per-launch events; algorithmic FLOPs = 2*M*N*K per launch
    hbm, tc_burst, tc_sust, src = peaks()
    cats = {}
    for c in ("CONV3+GEMM", "CONV3", "GEMM", "ATTN", "GN", "LN", "GEMV", "MISC"):
        try:
            cats[c] = eng.profile_category(c, B, H, W, reps=10)
        except sdg.SdgError:
            pass
    g_ms, g_n, g_fl, g_by = cats["CONV3+GEMM"]
    achieved = g_fl / (g_ms / 1000.0) / 1e12
    roofline = {"bound": "tensor", "kernel": "gemm_tc_kernel: every conv3x3 / conv1x1 / linear launch of the forward",
                "achieved": achieved, "peak": tc_burst, "unit": "TFLOP/s", "frac": achieved / tc_burst,
                "peak_source": f"{src} bf16_tflops (burst)",
                "timing": "the forward's GEMM launches replayed alone as a CUDA graph (CUDA events around 10 "
                          "replays), ms per forward " + f"{g_ms:.4f}",
                "traffic": GEMM_TRAFFIC_PER_LAUNCH, "traffic_note": GEMM_TRAFFIC_NOTE,
                "algorithmic_bytes_per_launch": g_by / max(g_n, 1),
                "launches_per_fwd": g_n, "flops_per_launch": g_fl / max(g_n, 1),
                "whole_forward_tflops": FLOPS_PER_FWD / (ms_per_step / 1000.0) / 1e12,
                "whole_forward_frac_of_sustained": FLOPS_PER_FWD / (ms_per_step / 1000.0) / 1e12 / tc_sust,
                "categories_replayed_alone_ms": {k: round(v[0], 4) for k, v in cats.items()},
                "categories_launches": {k: v[1] for k, v in cats.items()}}
    if "CONV3" in cats:
        c_ms, c_n, c_fl, _ = cats["CONV3"]
        roofline["conv3x3"] = {"tflops": c_fl / (c_ms / 1000.0) / 1e12, "frac": c_fl / (c_ms / 1000.0) / 1e12 / tc_burst,
                               "launches_per_fwd": c_n, "ms_per_fwd": c_ms}
    if "ATTN" in cats:
        a_ms, a_n, a_fl, _ = cats["ATTN"]
        roofline["attention"] = {"tflops": a_fl / (a_ms / 1000.0) / 1e12,
                                 "frac": a_fl / (a_ms / 1000.0) / 1e12 / tc_burst, "launches_per_fwd": a_n}
    for c, key in (("GN", "groupnorm"), ("LN", "layernorm")):
        if c in cats and cats[c][0] > 0:
            gbs = cats[c][3] / (cats[c][0] / 1000.0) / 1e9
            roofline[key] = {"gbs": gbs, "frac_of_hbm": gbs / hbm, "launches_per_fwd": cats[c][1]}

    # config 3 (GPU work) before the CPU baseline: after the oracle's multi-threaded fp32 forwards the first
    # timed host-API call measured ~1 s slower than its steady ~0.09 s for 8 images
    cfg3 = None
    if not args.no_config3 and not args.wo8:
        cfg3 = run_config3(eng, sdg, dev, world, rank)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        v, sample = cpu_oracle_forward_rate(wts, threads)
        cpu = {"value": v, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample}

    launches = eng.forward_launches(B, H, W)
    if rank == 0:
        print(json.dumps({
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": max(3, args.warmup), "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "fp16 (int8 weights)" if args.wo8 else "fp16",
            "data": "synthetic (seeded inputs, seeded default-init weights)",
            "config": config_dict(world, args.wo8), "clocks": clk, "roofline": roofline, "cpu_baseline": cpu,
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h)},
            "gpu_launches": launches * args.steps,
            "tensor_peak_frac": FLOPS_PER_FWD / (ms_per_step / 1000.0) / 1e12 / tc_burst,
            "config3_lcm": cfg3,
        }))
    eng.release()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
