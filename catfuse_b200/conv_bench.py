"""Single-layer benchmark of the fused Conv -> BN -> LIF kernel.

    python -m catfuse_b200.conv_bench                      # config 0: T=4 B=32 128->128 32x32
    python -m catfuse_b200.conv_bench --shape 4,64,128,128,16,16,3,1,1 --reps 3
    python -m catfuse_b200.conv_bench --ssa 4,64,64,384,12          # T,B,N,C,heads

Shape = T,B,Cin,Cout,H,W,k,stride,pad.  Inputs are seeded Bernoulli(p) spikes and
Kaiming-scaled weights; BN is the identity affine.  Each timed launch runs inside a
CUDA graph of ``--graph`` back-to-back calls; the line printed per shape gives the
mean time per call, the dense TFLOP/s (2*T*B*Ho*Wo*Cout*Cin*k*k) and the tile
geometry the kernel chose.  ``--reps N`` only runs N eager calls (no timing): the
form used under a profiler.
"""
from __future__ import annotations

import argparse

import torch

from . import ops

CONFIG0 = (4, 32, 128, 128, 32, 32, 3, 1, 1)


def run(shape, p=0.1, graph=20, reps=0, seed=0):
    T, B, Ci, Co, H, W, k, s, pad = shape
    dev = torch.device("cuda", torch.cuda.current_device())
    g = torch.Generator().manual_seed(seed)
    x = (torch.rand(T, B, Ci, H, W, generator=g) < p).float().to(dev)
    w = (torch.randn(Co, Ci, k, k, generator=g) * (2.0 / (Ci * k * k)) ** 0.5).to(dev)
    xp = ops.pack_tbchw(x)
    wp = ops.pack_conv_weight(w, xp.shape[-1])
    sc = torch.ones(Co, device=dev)
    sh = torch.zeros(Co, device=dev)
    Ho = (H + 2 * pad - k) // s + 1
    Wo = (W + 2 * pad - k) // s + 1
    v = torch.empty(B, Ho, Wo, Co, device=dev)
    out = torch.empty(B, Ho, Wo, T, Co, dtype=torch.float16, device=dev)

    def call():
        ops.conv_bn_lif(xp, wp, sc, sh, s, pad, v_out=v, out=out)

    if reps:
        for _ in range(reps):
            call()
        torch.cuda.synchronize()
        return None
    for _ in range(3):
        call()
    torch.cuda.synchronize()
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr):
        for _ in range(graph):
            call()
    gr.replay()
    torch.cuda.synchronize()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record()
    gr.replay()
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / graph
    flops = 2.0 * T * B * Ho * Wo * Co * Ci * k * k
    return {"shape": shape, "us": ms * 1e3, "tflops": flops / ms / 1e9,
            "geometry": ops.conv_geometry(T, B, Ho, Wo, Co)}


def run_ssa(shape, p=0.1, graph=20, seed=0):
    """Time ops.ssa_lif (spiking self-attention + LIF) on seeded token spikes."""
    T, B, N, C, heads = shape
    dev = torch.device("cuda", torch.cuda.current_device())
    g = torch.Generator().manual_seed(seed)
    q, k, v = ((torch.rand(B, N, T, C, generator=g) < p).half().to(dev) for _ in range(3))
    out = torch.empty_like(q)
    vo = torch.empty(B, N, C, device=dev)

    def call():
        ops.ssa_lif(q, k, v, heads, v_out=vo, out=out)

    for _ in range(3):
        call()
    torch.cuda.synchronize()
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr):
        for _ in range(graph):
            call()
    gr.replay()
    torch.cuda.synchronize()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record()
    gr.replay()
    b.record()
    torch.cuda.synchronize()
    us = a.elapsed_time(b) / graph * 1e3
    nbytes = 4 * B * N * T * C * 2 + B * N * C * 4
    return {"shape": shape, "us": us, "gbs": nbytes / us / 1e3, "mb": nbytes / 1e6}


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__,
                                 formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--shape", action="append", default=[],
                    help="T,B,Cin,Cout,H,W,k,stride,pad (repeatable)")
    ap.add_argument("--p", type=float, default=0.1, help="input spike probability")
    ap.add_argument("--graph", type=int, default=20, help="calls per timed graph")
    ap.add_argument("--reps", type=int, default=0, help="eager calls only, no timing")
    ap.add_argument("--ssa", action="append", default=[],
                    help="T,B,N,C,heads: time the spiking self-attention kernel instead")
    args = ap.parse_args(argv)
    for sh in args.ssa:
        r = run_ssa(tuple(int(v) for v in sh.split(",")), p=args.p, graph=args.graph)
        print(f"ssa {r['shape']}: {r['us']:.1f} us, {r['gbs']:.0f} GB/s of algorithmic bytes "
              f"({r['mb']:.1f} MB: q, k, v, spikes, v_T)")
    if args.ssa and not args.shape:
        return 0
    shapes = [tuple(int(v) for v in s.split(",")) for s in args.shape] or [CONFIG0]
    for shp in shapes:
        r = run(shp, p=args.p, graph=args.graph, reps=args.reps)
        if r is not None:
            print(f"{r['shape']}: {r['us']:.1f} us, {r['tflops']:.1f} TFLOP/s, "
                  f"geometry {r['geometry']}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
