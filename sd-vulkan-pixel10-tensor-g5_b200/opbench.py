"""Op microbenchmark at SD1.5 UNet shapes (BASELINE configs 1 and 2).

The counterpart of the reference's on-device microbench (``sd/VulkanBench.kt:66-126``:
matmul / conv / groupnorm / silu / attention at UNet shapes), run through the
C-ABI op surface on one GPU. Each op is timed with CUDA events over one replay
of a CUDA graph holding ``--iters`` launches (after ``--warmup`` eager
launches), so host launch overhead is excluded; inputs are seeded (activations N(0,1), weights
N(0, 0.02)), fp16, fp32 accumulation.

  python opbench.py                       # every op, JSON line each
  python opbench.py --op attn_self_4096_d40 --iters 3 --warmup 2   # one op (e.g. under ncu)
"""
from __future__ import annotations

import argparse
import importlib
import json
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
sys.path.insert(0, ROOT)


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d.get("hbm_gbs", 6650.0), d.get("bf16_tflops", 1590.0)
    return 6650.0, 1590.0


def build_ops(sdg, dev):
    g = torch.Generator().manual_seed(0)
    rn = lambda *s, std=1.0: (torch.randn(*s, generator=g) * std).half().to(dev)
    ops = {}
    B = 2
    for C, H in ((320, 64), (640, 32), (1280, 16), (1280, 8)):           # config 1 conv3x3
        x = rn(B, H, H, C)
        w = rn(C, 9 * C, std=0.02)
        b = torch.zeros(C, device=dev)
        ws = torch.empty(32 * B * H * H * C, dtype=torch.float32, device=dev)
        y = torch.empty_like(x)
        ops[f"conv3x3_{C}_{H}"] = (lambda x=x, w=w, b=b, y=y, ws=ws, C=C: sdg.conv2d(x, w, b, C, out=y, workspace=ws),
                                    2.0 * B * H * H * C * 9 * C, 0.0)
    for M, N, K in ((8192, 320, 2880), (8192, 1280, 1280), (8192, 4096, 4096), (1024, 320, 2880), (2048, 320, 2880),
                    (4096, 320, 2880)):                                     # plain GEMMs vs cuBLAS
        xa = rn(M, K)
        wa = rn(N, K, std=0.02)
        ya = torch.empty((M, N), dtype=torch.float16, device=dev)
        ops[f"linear_{M}_{N}_{K}"] = (lambda xa=xa, wa=wa, ya=ya: sdg.linear(xa, wa, out=ya), 2.0 * M * N * K, 0.0)
        ops[f"cublas_{M}_{N}_{K}"] = (lambda xa=xa, wa=wa, ya=ya: torch.matmul(xa, wa.t(), out=ya), 2.0 * M * N * K, 0.0)
    # the forward's most frequent linear shapes: K=320 out-projection with residual, the GEGLU FF-proj,
    # and the 32x32 / 16x16-level projections
    for M, N, K, act, res in ((8192, 320, 320, 0, True), (8192, 2560, 320, 2, False), (2048, 640, 640, 0, True),
                              (512, 1280, 1280, 0, True), (8192, 320, 1280, 0, True)):
        xa = rn(M, K)
        wa = rn(N, K, std=0.02)
        ba = torch.zeros(N, device=dev)
        ra = rn(M, N) if res else None
        ya = torch.empty((M, N // 2 if act == 2 else N), dtype=torch.float16, device=dev)
        tag = "geglu" if act == 2 else ("linres" if res else "lin")
        ops[f"{tag}_{M}_{N}_{K}"] = (lambda xa=xa, wa=wa, ba=ba, ra=ra, ya=ya, act=act:
                                     sdg.linear(xa, wa, ba, residual=ra, act=act, out=ya), 2.0 * M * N * K, 0.0)
    for C, H in ((1280, 8), (1280, 16), (640, 32)):                         # the upsample blocks (folded)
        xu = rn(B, H, H, C)
        wu = rn(4, C, 4, C, std=0.02)
        bu = torch.zeros(4 * C, device=dev)
        wsu = torch.empty(32 * B * H * H * 4 * C, dtype=torch.float32, device=dev)
        yu = torch.empty((B, 2 * H, 2 * H, C), dtype=torch.float16, device=dev)
        # FLOPs executed by the folded GEMM: 2 * (B H W) * (4 phases * C) * (4 taps * C), i.e. 16/36 of the direct
        # count of a 3x3 conv on the 2H x 2H upsampled input
        ops[f"upconv_{C}_{H}"] = (lambda xu=xu, wu=wu, bu=bu, yu=yu, wsu=wsu: sdg.upsample_conv3x3(xu, wu, bu, out=yu,
                                                                                                   workspace=wsu),
                                  2.0 * B * H * H * (4 * C) * (4 * C), 0.0)
    x = rn(B, 32, 32, 320)                                                  # config 1 conv1x1 skip
    w = rn(640, 320, std=0.02)
    y = torch.empty((B, 32, 32, 640), dtype=torch.float16, device=dev)
    ops["conv1x1_320_640_32"] = (lambda: sdg.conv2d(x, w, None, 640, k=1, out=y), 2.0 * B * 1024 * 320 * 640, 0.0)
    for C, H in ((320, 64), (1280, 16)):                                    # config 1 GroupNorm+SiLU
        xg = rn(B, H * H, C)
        gm = torch.ones(C, device=dev)
        bt = torch.zeros(C, device=dev)
        yg = torch.empty_like(xg)
        st = torch.empty(sdg.lib().sdg_groupnorm_scratch_bytes(B, H * H, C, 32) // 4 + 1, dtype=torch.float32,
                         device=dev)
        ops[f"gn_silu_{C}_{H}"] = (lambda xg=xg, gm=gm, bt=bt, yg=yg, st=st: sdg.groupnorm(xg, gm, bt, 1e-5, True, out=yg,
                                                                                        stats=st),
                                   0.0, 2.0 * 2 * B * H * H * C)
    for M, C in ((8192, 320), (2048, 640), (512, 1280)):                    # transformer LayerNorm
        xl = rn(M, C)
        gl = torch.ones(C, device=dev)
        bl = torch.zeros(C, device=dev)
        yl = torch.empty_like(xl)
        ops[f"layernorm_{M}_{C}"] = (lambda xl=xl, gl=gl, bl=bl, yl=yl: sdg.layernorm(xl, gl, bl, out=yl), 0.0,
                                     2.0 * 2 * M * C)
    xt = rn(64)
    yt = torch.empty_like(xt)
    ops["launch_floor_add64"] = (lambda: sdg.add(xt, xt, out=yt), 0.0, 0.0)   # per-launch floor in a graph
    heads = 8                                                               # config 2 attention
    for name, Sq, Sk, d in (("attn_self_4096_d40", 4096, 4096, 40), ("attn_self_1024_d80", 1024, 1024, 80),
                            ("attn_self_256_d160", 256, 256, 160), ("attn_cross_4096_d40", 4096, 77, 40), ("attn_cross_1024_d80", 1024, 77, 80),
                            ("attn_cross_256_d160", 256, 77, 160)):
        C = heads * d
        q = sdg.heads_layout(rn(B * Sq, C), B, Sq, heads, d)
        k = sdg.heads_layout(rn(B * Sk, C), B, Sk, heads, d)
        vt_ld = (Sk + 7) // 8 * 8
        v = sdg.heads_layout(rn(B * Sk, C), B, Sk, heads, d, transpose=True, s_pad=vt_ld)
        o = torch.empty((B, Sq, C), dtype=torch.float16, device=dev)
        ops[name] = (lambda q=q, k=k, v=v, o=o, Sq=Sq, Sk=Sk, d=d, vt_ld=vt_ld:
                     sdg.attention(q, k, v, B, heads, Sq, Sk, d, vt_ld, out=o),
                     4.0 * B * heads * Sq * Sk * d, 0.0)
    return ops


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--op", default=None)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--eager", action="store_true", help="time eager launches instead of a CUDA-graph replay")
    a = ap.parse_args()
    sdg = importlib.import_module(os.path.basename(HERE))
    dev = torch.device("cuda", 0)
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    ops = build_ops(sdg, dev)
    hbm, tc = peaks()
    names = [a.op] if a.op else list(ops)
    for n in names:
        fn, flops, nbytes = ops[n]
        for _ in range(a.warmup):
            fn()
        torch.cuda.synchronize()
        run = fn
        if not a.eager:
            # replay a captured graph of `iters` launches: device time without host launch gaps
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                for _ in range(a.iters):
                    fn()
            g.replay()
            torch.cuda.synchronize()
            run = g.replay
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        if a.eager:
            for _ in range(a.iters):
                run()
        else:
            run()
        e1.record(stream)
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1000.0 / a.iters
        rec = {"op": n, "us": round(us, 2)}
        if not flops and not nbytes:
            rec["note"] = "per-launch time of a trivial kernel"

        if flops:
            rec["tflops"] = round(flops / us / 1e6, 1)
            rec["frac_of_tensor_peak"] = round(flops / us / 1e6 / tc, 3)
        if nbytes:
            rec["gbs"] = round(nbytes / us / 1e3, 1)
            rec["frac_of_hbm"] = round(nbytes / us / 1e3 / hbm, 3)
        print(json.dumps(rec))


if __name__ == "__main__":
    main()
