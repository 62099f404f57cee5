"""Bandwidth benchmark of the memory-bound kernels at the BASELINE shapes.

    python -m catfuse_b200.hbm_bench [--reps 10]

Each call is captured into a CUDA graph and timed alone with CUDA events
around its replay, after an L2 eviction (a 256 MB write, then a 256 MB read
so that the flush leaves no dirty lines to write back inside the timed call).
Achieved bandwidth = algorithmic bytes / time; the peak is ``hbm_gbs`` of
MEASURED_PEAKS.json when present (a measured copy bandwidth of the GPU model).

Cases (config numbers of BASELINE.json):
* config 0 LIF family on z [T=4, B=32, 128, 32, 32]: lif_fwd (fp32 z -> fp16 /
  u8 / bit-packed spikes), bn_lif, add_lif;
* config 2 prescan over x [B=32, 28, 28, T=4, 256] fp16 (conv-tile masks) and
  the reference-geometry prescan over the per-step NCHW view;
* config 2 sparse conv sweep: Conv3x3-BN-LIF 256->256 at 28x28 with the
  prescan masks, block sparsity s in {0.8, 0.9, 0.95, 0.99, 1.0}; bytes =
  x read once + weights + spikes written + v_T, as a memory-bound kernel.
"""
from __future__ import annotations

import argparse
import json
from pathlib import Path

import torch

from . import ops, workloads
from .timing import L2Flush

ROOT = Path(__file__).resolve().parent.parent


def _peak():
    try:
        return float(json.loads((ROOT / "MEASURED_PEAKS.json").read_text())["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def _time(fn, reps, flush):
    """Mean device time (us) of ``fn``'s launches: captured once into a CUDA
    graph and replayed between two events, each replay after an L2-evicting
    write, so host-side overhead of the Python wrappers is not timed."""
    fn()
    torch.cuda.synchronize()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=side):
        fn()
    torch.cuda.synchronize()
    ev = []
    for _ in range(reps):
        flush()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        g.replay()
        b.record()
        ev.append((a, b))
    torch.cuda.synchronize()
    return sum(a.elapsed_time(b) for a, b in ev) / reps * 1e3  # us


def _time_stream(make, nbytes, reps, min_total=512 << 20):
    """Steady-state device time (us per launch) of back-to-back launches:
    ``make(i)`` returns the call for the i-th of k independent buffer sets,
    k chosen so that the k sets together move more than ``min_total`` bytes
    (four times the L2), so every launch streams its inputs from HBM without
    an explicit flush.  The k launches are captured into one CUDA graph; the
    replay is timed with CUDA events and divided by k, so the launch ramp and
    the event clock's granularity are spread over k launches."""
    k = max(2, -(-min_total // int(nbytes)))
    fns = [make(i) for i in range(k)]
    for f in fns:
        f()
    torch.cuda.synchronize()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=side):
        for f in fns:
            f()
    torch.cuda.synchronize()
    g.replay()
    torch.cuda.synchronize()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        g.replay()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) * 1e3 / (reps * k), k


def stream_table(dev, peak, src, reps):
    """Back-to-back (steady-state) bandwidth of the memory-bound kernels at the
    BASELINE shapes, beside a plain device copy of the same byte count."""
    g = torch.Generator().manual_seed(1)
    rows = []

    def report(name, us, nbytes, k):
        gbs = nbytes / us / 1e3
        rows.append({"kernel": name, "us": us, "MB": nbytes / 1e6, "GBs": gbs,
                     "frac": gbs / peak, "sets": k})
        print(f"{name:58s} {us:8.1f} us {nbytes / 1e6:8.1f} MB {gbs:7.0f} GB/s "
              f"{gbs / peak:6.1%} of {src} {peak:.0f}  (x{k} back to back)")

    T, B, C, H, W = 4, 32, 128, 32, 32
    N = B * C * H * W
    zs, outs = {}, {}

    def z_of(i):
        if i not in zs:
            zs[i] = (torch.randn(T, B, C, H, W, generator=g) * 0.8 + 0.3).to(dev)
            outs[i] = torch.empty(T, B, C, H, W, dtype=torch.float16, device=dev)
        return zs[i], outs[i]

    nb = T * N * 4 + T * N * 2
    # plain device copy of the same byte count (read z fp32 half, write half):
    # the achievable streaming rate at this size
    def mk_copy(i):
        src_ = torch.empty(nb // 8, dtype=torch.float32, device=dev)
        dst = torch.empty_like(src_)
        return lambda: dst.copy_(src_)
    us, k = _time_stream(mk_copy, nb, reps)
    report("device copy (torch), same bytes as lif_fwd fp16", us, nb, k)

    def mk_lif(i):
        z, o = z_of(i)
        return lambda: ops.lif_fwd(z, spike_dtype=torch.float16)
    us, k = _time_stream(mk_lif, nb, reps)
    report("lif_fwd  z fp32 -> spikes fp16  [4,32,128,32,32]", us, nb + 4 * N, k)
    scale = torch.rand(C, generator=g).to(dev) + 0.5
    shift = torch.randn(C, generator=g).to(dev) * 0.1

    def mk_bn(i):
        z, o = z_of(i)
        return lambda: ops.bn_lif(z, scale, shift, spike_dtype=torch.float16)
    us, k = _time_stream(mk_bn, nb, reps)
    report("bn_lif   z fp32 -> spikes fp16", us, nb + 4 * N + 8 * C, k)
    z2s = {}

    def mk_add(i):
        z, o = z_of(i)
        if i not in z2s:
            z2s[i] = torch.randn(T, B, C, H, W, generator=g).to(dev)
        z2 = z2s[i]
        return lambda: ops.add_lif(z, z2, spike_dtype=torch.float16)
    us, k = _time_stream(mk_add, nb + T * N * 4, reps)
    report("add_lif  2 x fp32 -> spikes fp16", us, nb + T * N * 4 + 4 * N, k)
    zs.clear(); outs.clear(); z2s.clear()

    T, B, C, H, W = 4, 32, 256, 28, 28
    xs = {}

    def x_of(i):
        if i not in xs:
            x = workloads.block_sparse_spikes(T, B, C, H, W, 0.9, seed=900 + i).to(dev)
            xp = ops.pack_tbchw(x)
            xr = x.reshape(T * B, C, H, W).half().contiguous()
            del x
            xs[i] = (xp, xr, ops.prescan_conv_tiles(xp, C, 3, 3, 1, 1))
        return xs[i]
    xbytes = T * B * C * H * W * 2

    def mk_pc(i):
        xp, _, m = x_of(i)
        return lambda: ops.prescan_conv_tiles(xp, C, 3, 3, 1, 1, mask_out=m)
    us, k = _time_stream(mk_pc, xbytes, reps)
    report("prescan_conv_tiles  x [32,28,28,4,256] fp16  s=0.9", us, xbytes, k)

    def mk_pr(i):
        _, xr, _ = x_of(i)
        return lambda: ops.prescan(xr, 3, 1, 1, 8, 8, 32)
    us, k = _time_stream(mk_pr, xbytes, reps)
    report("prescan (reference geometry) x [128,256,28,28] fp16", us, xbytes, k)
    print(json.dumps({"hbm_stream": rows, "peak_gbs": peak, "peak_source": src}))
    return rows


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__,
                                 formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--reps", type=int, default=20)
    ap.add_argument("--only", choices=["lif", "prescan", "sweep"], default=None,
                    help="run one group: the LIF family, the two prescans once each on the "
                         "config-2 input (s = 0.9), or the SparseFlow sweep")
    ap.add_argument("--stream", action="store_true",
                    help="steady-state table: each kernel launched back to back over buffer "
                         "sets larger than L2 (no flush), beside a device copy of equal bytes")
    args = ap.parse_args(argv)
    dev = torch.device("cuda", torch.cuda.current_device())
    peak, src = _peak()
    if args.stream:
        stream_table(dev, peak, src, args.reps)
        return 0
    flush = L2Flush(dev)
    g = torch.Generator().manual_seed(0)
    rows = []

    def report(name, us, nbytes):
        gbs = nbytes / us / 1e3
        rows.append((name, us, nbytes / 1e6, gbs, gbs / peak))
        print(f"{name:58s} {us:8.1f} us {nbytes / 1e6:8.1f} MB {gbs:7.0f} GB/s "
              f"{gbs / peak:6.1%} of {src} {peak:.0f}")

    if args.only == "prescan":
        T, B, C, H, W = 4, 32, 256, 28, 28
        x = workloads.block_sparse_spikes(T, B, C, H, W, 0.9, seed=900).to(dev)
        xp = ops.pack_tbchw(x)
        us = _time(lambda: ops.prescan_conv_tiles(xp, C, 3, 3, 1, 1), args.reps, flush)
        report("prescan_conv_tiles  x [32,28,28,4,256] fp16  s=0.9", us, xp.numel() * 2)
        xr = x.reshape(T * B, C, H, W).half().contiguous()
        us = _time(lambda: ops.prescan(xr, 3, 1, 1, 8, 8, 32), args.reps, flush)
        report("prescan (reference geometry) x [128,256,28,28] fp16", us, xr.numel() * 2)
        return 0

    # ---- config 0: LIF family ---------------------------------------------
    T, B, C, H, W = 4, 32, 128, 32, 32
    N = B * C * H * W
    z = (torch.randn(T, B, C, H, W, generator=g) * 0.8 + 0.3).to(dev)
    for sd, sb, name in ((torch.float16, 2, "fp16"), (torch.uint8, 1, "u8"), ("bits", 1 / 8, "bits")):
        us = _time(lambda: ops.lif_fwd(z, spike_dtype=sd), args.reps, flush)
        report(f"lif_fwd  z fp32 -> spikes {name}  [4,32,128,32,32]", us, T * N * 4 + T * N * sb + 4 * N)
    scale = torch.rand(C, generator=g).to(dev) + 0.5
    shift = torch.randn(C, generator=g).to(dev) * 0.1
    us = _time(lambda: ops.bn_lif(z, scale, shift, spike_dtype=torch.float16), args.reps, flush)
    report("bn_lif   z fp32 -> spikes fp16", us, T * N * 4 + T * N * 2 + 4 * N + 8 * C)
    z2 = torch.randn(T, B, C, H, W, generator=g).to(dev)
    us = _time(lambda: ops.add_lif(z, z2, spike_dtype=torch.float16), args.reps, flush)
    report("add_lif  2 x fp32 -> spikes fp16", us, T * N * 8 + T * N * 2 + 4 * N)
    if args.only == "lif":
        return 0

    # ---- config 2: prescan and sparse conv sweep -----------------------------
    T, B, C, H, W = 4, 32, 256, 28, 28
    w = (torch.randn(C, C, 3, 3, generator=g) * (2.0 / (C * 9)) ** 0.5).to(dev)
    sc = torch.ones(C, device=dev)
    sh = torch.zeros(C, device=dev)
    dense_us = None
    sweep = []
    geom = None
    for s in (0.0, 0.8, 0.9, 0.95, 0.99, 1.0):
        x = workloads.block_sparse_spikes(T, B, C, H, W, s, seed=int(s * 1000)).to(dev)
        xp = ops.pack_tbchw(x)
        wp = ops.pack_conv_weight(w, xp.shape[-1])
        xbytes = xp.numel() * 2
        mask = ops.prescan_conv_tiles(xp, C, 3, 3, 1, 1)
        pre_us = _time(lambda: ops.prescan_conv_tiles(xp, C, 3, 3, 1, 1, mask_out=mask),
                       args.reps, flush)
        report(f"prescan_conv_tiles  x [32,28,28,4,256] fp16  s={s}", pre_us,
               xbytes + 4 * mask.numel())
        if geom is None:
            geom = ops.conv_geometry(T, B, H, W, C, xp.shape[-1], 1, True)
        n_kx = xp.shape[-1] // ops.conv_chunk(xp.shape[-1], True)
        active = int(sum(bin(int(m) & ((1 << n_kx) - 1)).count("1") for m in mask.cpu().tolist()))
        frac = active / (geom["n_mtiles"] * n_kx)
        v = torch.empty(B, H, W, C, device=dev)
        out = torch.empty(B, H, W, T, C, dtype=torch.float16, device=dev)
        conv_bytes = xbytes + wp.numel() * 2 + out.numel() * 2 + v.numel() * 4
        if dense_us is None:
            dense_us = _time(lambda: ops.conv_bn_lif(xp, wp, sc, sh, 1, 1, v_out=v, out=out),
                             args.reps, flush)
            flops = 2.0 * T * B * H * W * C * C * 9
            print(f"{'dense conv_bn_lif 256->256 28x28 (reference for the sweep)':58s} "
                  f"{dense_us:8.1f} us  {flops / dense_us / 1e6:7.0f} TFLOP/s dense-equivalent")
        us = _time(lambda: ops.conv_bn_lif(xp, wp, sc, sh, 1, 1, v_out=v, out=out, tile_mask=mask),
                   args.reps, flush)
        report(f"sparse conv_bn_lif (masked, chunk 32) s={s} active={frac:.3f} "
               f"[{us / dense_us:.2f}x dense, +prescan {(us + pre_us) / dense_us:.2f}x]",
               us, conv_bytes)
        # device EGD: dense-chunk masks, the kernel decides
        emask = ops.prescan_conv_tiles(xp, C, 3, 3, 1, 1, egd=True)
        n_kd = xp.shape[-1] // ops.conv_chunk(xp.shape[-1], False)
        efrac = sum(bin(int(m) & ((1 << n_kd) - 1)).count("1") for m in emask.cpu().tolist()) / (
            geom["n_mtiles"] * n_kd)
        emasked = _time(lambda: ops.conv_bn_lif(xp, wp, sc, sh, 1, 1, v_out=v, out=out,
                                                tile_mask=emask, egd_max_active_frac=1.0),
                        args.reps, flush)
        from .hardware import B200
        theta = B200.egd_max_active_frac

        def egd_total():
            ops.prescan_conv_tiles(xp, C, 3, 3, 1, 1, mask_out=emask, egd=True)
            ops.conv_bn_lif(xp, wp, sc, sh, 1, 1, v_out=v, out=out, tile_mask=emask,
                            egd_max_active_frac=theta)
        etot = _time(egd_total, args.reps, flush)
        print(f"{'  device EGD (prescan + conv, max_active ' + str(theta) + ')':58s} {etot:8.1f} us"
              f"  [{etot / dense_us:.2f}x dense]  active(chunk 64)={efrac:.3f}, "
              f"masks forced {emasked:.1f} us")
        sweep.append({"s": s, "active_frac": efrac, "masked_us": emasked, "prescan_us": pre_us,
                      "dense_us": dense_us, "egd_total_us": etot,
                      "active_frac_chunk32": frac, "masked_chunk32_us": us})
    # EGD calibration: masked time ~ a + b * active_frac (least squares over the
    # sweep); SparseFlow pays off while prescan + masked < dense, i.e. below
    # the crossover fraction written out here.
    xs = [r["active_frac"] for r in sweep]
    ys = [r["masked_us"] for r in sweep]
    n = len(xs)
    mx, my = sum(xs) / n, sum(ys) / n
    sxx = sum((a - mx) ** 2 for a in xs)
    b = sum((a - mx) * (c - my) for a, c in zip(xs, ys)) / sxx if sxx > 0 else 0.0
    a0 = my - b * mx
    pre = sum(r["prescan_us"] for r in sweep) / n
    cross = (dense_us - pre - a0) / b if b > 0 else 0.0
    print(json.dumps({"egd_calibration": {"masked_us_fit": [a0, b], "prescan_us": pre,
                                          "dense_us": dense_us,
                                          "crossover_active_frac": cross, "sweep": sweep}}))
    xr = x.reshape(T * B, C, H, W).half().contiguous()
    us = _time(lambda: ops.prescan(xr, 3, 1, 1, 8, 8, 32), args.reps, flush)
    report("prescan (reference geometry) x [128,256,28,28] fp16", us, xr.numel() * 2)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
