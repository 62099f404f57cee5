"""Benchmark: SEW-ResNet-18 (CIFAR shape, T=4) inference samples/s on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = ``functional.reset_net`` + one multi-step forward of SEW-ResNet-18
(B=64 per GPU, 3x32x32 N(0,1) images repeated over T=4,
random-init weights with data-calibrated BN statistics, LIF tau=2, v_th=1,
hard reset, cnf ADD, avgpool -> fc 512->10).  With N GPUs (torchrun, one
process per GPU) every rank runs its own batch of 64 (weak scaling) and the
logits are all-gathered over NCCL at the end of each step.

``value``: samples/s of the whole job with inputs resident in HBM (the
forward is one CUDA-graph replay of fused sm_100a kernels), each step timed
with CUDA events, L2 flushed (256 MB write, then a 256 MB read so no dirty line
is left) between steps outside the timed
events, max over ranks.  ``e2e``: the same metric through the public API
(``optimize``'d model called on a device copy of pinned host images, logits
read back to the host), host<->device copies inside the timed region.
``--impl reference``: the reference's CPU path (SpikingJelly semantics in
PyTorch, restated in ``oracle/``) on the host cores; rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from catfuse_b200.timing import L2Flush  # noqa: E402

METRIC = "SEW-ResNet18 T=4 samples/s"
UNIT = "samples/s"
T_STEPS = 4
BATCH = 64


def _peaks():
    try:
        return json.loads((ROOT / "MEASURED_PEAKS.json").read_text()), "measured"
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def _conv_flops(plan) -> float:
    from catfuse_b200.network import ConvStep
    total = 0.0
    for st in plan.steps:
        if isinstance(st, ConvStep):
            b, ho, wo, t, co = plan.shapes[st.dst]
            spec = st.native.spec
            total += 2.0 * t * b * ho * wo * co * spec.in_channels * spec.kernel_size ** 2
    return total


def _traffic_from_profiles():
    """Per-launch DRAM bytes of the conv kernel from the committed ncu summary
    (a line 'traffic_bytes_per_forward: N'), or None."""
    p = ROOT / "profiles" / "conv_bn_lif_sew_rn18.md"
    try:
        for line in p.read_text().splitlines():
            if line.strip().startswith("traffic_bytes_per_launch_avg:"):
                return float(line.split(":", 1)[1])
    except Exception:
        pass
    return None


class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        fd, name = tempfile.mkstemp(prefix="catfuse_clocks_", suffix=".csv")
        os.close(fd)
        self.path = Path(name)

    def start(self):
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=self.fh, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
            return
        # nvidia-smi takes a moment to start: wait (bounded) for its first
        # sample so that the timed region that follows is covered.
        t_end = time.time() + 5.0
        while time.time() < t_end and self.proc.poll() is None:
            self.fh.flush()
            if self.path.stat().st_size > 0:
                break
            time.sleep(0.05)

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.fh.close()
        text = self.path.read_text()
        try:
            self.path.unlink()
        except OSError:
            pass
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in text.splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def build_model(device, batch, seed=0, precision="fp16"):
    from catfuse_b200 import optimize
    from catfuse_b200.sj import zoo
    net = zoo.init_random_(zoo.build_sew_resnet18_cifar(), seed)
    g = torch.Generator().manual_seed(1000 + seed)
    calib = torch.randn(BATCH, 3, 32, 32, generator=g).unsqueeze(0).repeat(T_STEPS, 1, 1, 1, 1)
    zoo.calibrate_bn_(net, calib)
    model, stats = optimize(net.eval(), device=device, T=T_STEPS, precision=precision)
    return model, stats, net


def time_plan(plan, steps, flush, dist=None, gathered=None):
    """Per-step CUDA-event times (ms) of the graphed forward, L2 flushed
    between steps outside the events; returns the list of step times."""
    def step():
        plan.fresh = True            # reset_net: every step starts from v = 0
        logits = plan.run(use_graph=True)
        if dist is not None:
            dist.all_gather_into_tensor(gathered, logits)
        return logits

    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(steps)]
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    for s, e in evs:
        flush()
        s.record()
        step()
        e.record()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    return [s.elapsed_time(e) for s, e in evs]


def max_over_ranks(x, dev, dist):
    t = torch.tensor([float(x)], device=dev)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def cpu_baseline(batch=BATCH, budget_s=12.0):
    """The reference's CPU path (SJ semantics in PyTorch; oracle restatement)
    on the host cores, a bounded sample of the workload."""
    import oracle
    from catfuse_b200.sj import zoo
    torch.set_num_threads(os.cpu_count() or 1)
    net = zoo.init_random_(zoo.build_sew_resnet18_cifar(), 0)
    g = torch.Generator().manual_seed(1000)
    x = torch.randn(batch, 3, 32, 32, generator=g).unsqueeze(0).repeat(T_STEPS, 1, 1, 1, 1)
    zoo.calibrate_bn_(net, x)
    params = {k: v.detach().float() for k, v in net.state_dict().items()}
    with torch.no_grad():
        oracle.sew_resnet18_forward(x, params)  # warm-up
        n, t0 = 0, time.perf_counter()
        while True:
            oracle.sew_resnet18_forward(x, params)
            n += 1
            el = time.perf_counter() - t0
            if el >= budget_s or n >= 50:
                break
    return {"value": n * batch / el, "unit": UNIT, "cores": torch.get_num_threads(),
            "kind": "port",
            "sample": f"{n} forwards of B={batch} (T=4, 32x32) in {el:.1f}s, fp32 torch CPU "
                      f"(SpikingJelly LIF semantics, oracle/nets.py)"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    # At most 8 bounded CPU samples (~1 minute in total) whatever --steps asks:
    # each step is a multi-second sample of the CPU workload (B=64 forwards,
    # the GPU arm's configuration), not one forward.
    n_ref = max(1, min(args.steps, 8))
    budget = max(2.0, min(20.0, 60.0 / (n_ref + min(args.warmup, 3))))
    for _ in range(min(args.warmup, 3)):
        cpu_baseline(batch=8, budget_s=0.5)
    vals = [cpu_baseline(batch=BATCH, budget_s=budget) for _ in range(n_ref)]
    v = statistics.median(x["value"] for x in vals)
    base = vals[0]
    base["value"] = v
    line = {"metric": METRIC, "value": v, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1000.0 * BATCH / v, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "impl": "reference", "cpu_samples": n_ref,
            "config": {"workload": "SEW-ResNet18 CIFAR T=4 forward (reference CPU path)",
                       "global_batch": BATCH, "seq_len": T_STEPS, "parallelism": "cpu"},
            "cpu_baseline": base,
            "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def egd_report(plan):
    """Device-side EGD of the STFusion sites in the last forward: the active
    (tile, chunk) fraction of each site's prescan masks and what the kernel
    chose with the profile's threshold."""
    from catfuse_b200 import ops
    from catfuse_b200.network import ConvStep
    out = {}
    for st in plan.steps:
        if not isinstance(st, ConvStep) or not st.sparse:
            continue
        cin_p = plan.shapes[st.src][-1]
        n_kx = cin_p // ops.conv_chunk(cin_p, False)   # device-dispatch masks: dense chunk
        bits = (1 << n_kx) - 1
        masks = st.mask.cpu().tolist()
        active = sum(bin(int(m) & bits).count("1") for m in masks) / (len(masks) * n_kx)
        choice = ("StaticZero" if active == 0 else
                  ("SparseFlow" if active <= plan.egd_frac else "DenseKeep"))
        out[st.name] = {"active_frac": round(active, 4), "decision": choice}
    return {"max_active_frac": plan.egd_frac, "sites": out} if out else None


def other_workloads(dev, flush, steps, dist, world):
    """The other BASELINE configurations, same protocol (graph replay, inputs
    resident, L2 flushed between steps, CUDA events, max over ranks):
    config 3 Spiking ResNet-18 224x224 B=32 (dense plan, and every 3x3/s1 conv
    on STFusion with the device EGD deciding per layer and per call from the
    measured masks), config 4 Spikformer B=64."""
    from catfuse_b200 import hardware
    from catfuse_b200.network import CTFNetwork
    from catfuse_b200.sj import spikformer, zoo
    from catfuse_b200.spikformer_net import CTFSpikformer
    from catfuse_b200.substitute import substitute, substitute_sf
    out = {}

    def measure(plan, B, label, flops=None):
        for _ in range(3):
            plan.fresh = True
            plan.run(use_graph=True)
        ms = max_over_ranks(sum(time_plan(plan, steps, flush)), dev, dist) / steps
        r = {"samples_per_s": world * B * 1000.0 / ms, "ms_per_step": ms, "per_gpu_batch": B,
             "steps": steps}
        if flops:
            r["conv_tflops_per_s"] = flops / (ms / 1000.0) / 1e12
        out[label] = r
        return r

    g = torch.Generator().manual_seed(77)
    # config 3: Spiking ResNet-18, ImageNet stem, 224x224, B=32
    B3 = 32
    net = zoo.init_random_(zoo.build_spiking_resnet18_imagenet(num_classes=1000), 0)
    calib = torch.randn(8, 3, 224, 224, generator=g).unsqueeze(0).repeat(T_STEPS, 1, 1, 1, 1)
    zoo.calibrate_bn_(net, calib)
    net.eval()
    x3 = torch.randn(B3, 3, 224, 224, generator=g).to(dev).unsqueeze(0).repeat(T_STEPS, 1, 1, 1, 1)
    m3, _ = substitute(net)
    c3 = CTFNetwork(m3.to(dev), use_sparse=False)
    p3 = c3.plan_for(x3)
    p3.x_in.copy_(x3)
    measure(p3, B3, "spiking_resnet18_224_b32 (config 3, DenseKeep)", _conv_flops(p3))
    del c3, p3
    ms3, st3 = substitute_sf(net, T=T_STEPS, force_sparse=True, hwprof=hardware.B200)
    e3 = CTFNetwork(ms3.to(dev), use_sparse=True)
    pe3 = e3.plan_for(x3)
    pe3.x_in.copy_(x3)
    r = measure(pe3, B3, "spiking_resnet18_224_b32 (config 3, STFusion + device EGD)")
    r["egd"] = egd_report(pe3)
    del e3, pe3, x3
    # config 4: Spikformer, embed 384, 12 heads, 4 blocks, B=64
    sf = zoo.init_random_(spikformer.build_spikformer_cifar(), 0)
    calib = torch.randn(16, 3, 32, 32, generator=g).unsqueeze(0).repeat(T_STEPS, 1, 1, 1, 1)
    zoo.calibrate_bn_(sf, calib)
    sf.eval()
    msf, _ = substitute_sf(sf, T=T_STEPS)
    csf = CTFSpikformer(msf.to(dev))
    x4 = torch.randn(BATCH, 3, 32, 32, generator=g).to(dev).unsqueeze(0).repeat(T_STEPS, 1, 1, 1, 1)
    p4 = csf.plan_for(x4)
    p4.x_in.copy_(x4)
    measure(p4, BATCH, "spikformer_b64 (config 4)")
    return out


def conv_roofline(plan, flush, peaks, peak_src):
    """The forward's conv launches replayed alone as one CUDA graph (same
    inputs, same order, L2 flushed before each replay), plus each launch timed
    alone (eager, L2 flushed before it) for the per-layer fractions."""
    from catfuse_b200.network import ConvStep
    from catfuse_b200 import ops

    def launch(st):
        plan.conv_launch(st, True)

    def layer_flops(st):
        fl = 0.0
        for c in (st, st.dual) if st.dual is not None else (st,):
            b_, ho, wo, t_, co = plan.shapes[c.dst]
            spec = c.native.spec
            fl += 2.0 * t_ * b_ * ho * wo * co * spec.in_channels * spec.kernel_size ** 2
        return fl

    convs = [st for st in plan.steps if isinstance(st, ConvStep) and not st.fused]

    def conv_launches():
        for st in convs:
            launch(st)

    plan.fresh = True
    plan.pack_input()
    conv_launches()                      # warm-up (also fills every activation)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    conv_graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(conv_graph, stream=side):
        conv_launches()
    torch.cuda.synchronize()
    conv_ms = []
    for _ in range(5):
        flush()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        conv_graph.replay()
        b.record()
        torch.cuda.synchronize()
        conv_ms.append(a.elapsed_time(b))
    conv_ms_fwd = sum(conv_ms) / len(conv_ms)
    peak = peaks["bf16_tflops"]
    per_layer = []
    for st in convs:
        fl = layer_flops(st)
        g1 = torch.cuda.CUDAGraph()          # one launch, replayed (no host overhead timed)
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.graph(g1, stream=side):
            launch(st)
        torch.cuda.synchronize()
        ts = []
        for _ in range(20):   # mean of 20: the event clock ticks in ~4 us steps here
            flush()
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record()
            g1.replay()
            b.record()
            ts.append((a, b))
        torch.cuda.synchronize()
        us = 1000.0 * statistics.mean(a.elapsed_time(b) for a, b in ts)
        per_layer.append({"layer": st.name + ("+" + st.dual.name.split(".")[-1] if st.dual else ""),
                          "us": round(us, 2),
                          "tflops": round(fl / us / 1e6, 1),
                          "frac": round(fl / us / 1e6 / peak, 3)})
    flops = _conv_flops(plan)
    achieved = flops / (conv_ms_fwd / 1000.0) / 1e12
    return {"bound": "tensor", "achieved": achieved, "peak": peak,
            "unit": "TFLOP/s", "frac": achieved / peak,
            "traffic": _traffic_from_profiles(), "peak_source": f"{peak_src} bf16_tflops (burst)",
            "kernel": "conv_t_kernel / conv_bn_lif_kernel (the conv launches of one forward, "
                      "replayed as one CUDA graph, L2 flushed before each replay)",
            "flops_per_forward": flops, "conv_ms_per_forward": conv_ms_fwd,
            "launches_per_forward": len(convs), "per_layer": per_layer}


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=500)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--batch", type=int, default=BATCH, help="per-GPU batch")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the fp32-mode and strong-scaling side measurements")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        return run_reference(args)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev)

    from catfuse_b200.sj import functional
    model, stats, _ = build_model(dev, args.batch)
    B = args.batch
    g = torch.Generator().manual_seed(2000 + rank)
    images = torch.randn(B, 3, 32, 32, generator=g)
    x_dev = images.to(dev).unsqueeze(0).repeat(T_STEPS, 1, 1, 1, 1).contiguous()
    plan = model.plan_for(x_dev)
    plan.x_in.copy_(x_dev)
    flush = L2Flush(dev)
    gathered = torch.empty((world, T_STEPS, B, 10), device=dev) if world > 1 else None

    for _ in range(args.warmup):
        plan.fresh = True
        plan.run(use_graph=True)
        if dist is not None:
            dist.all_gather_into_tensor(gathered, plan.logits)
    torch.cuda.synchronize()

    # ---- value: device-resident inputs, per-step CUDA events, L2 flushed ----
    sampler = ClockSampler(local)
    sampler.start()
    step_ms = time_plan(plan, args.steps, flush, dist, gathered)
    clocks = sampler.stop()
    total_ms = max_over_ranks(sum(step_ms), dev, dist)
    ms_per_step = total_ms / args.steps
    value = world * B * args.steps / (total_ms / 1000.0)

    egd = egd_report(plan)
    peaks, peak_src = _peaks()
    roofline = conv_roofline(plan, flush, peaks, peak_src)
    roofline["share_of_step"] = roofline["conv_ms_per_forward"] / ms_per_step

    # ---- e2e through the public API (host buffers, copies inside) -----------
    pinned = images.pin_memory()
    out_host = torch.empty((T_STEPS, B, 10), dtype=torch.float32).pin_memory()

    def e2e_step():
        xd = pinned.to(dev, non_blocking=True)
        x_seq = xd.unsqueeze(0).repeat(T_STEPS, 1, 1, 1, 1)
        functional.reset_net(model)
        logits = model(x_seq)
        if dist is not None:
            dist.all_gather_into_tensor(gathered, logits)
        out_host.copy_(logits, non_blocking=True)
        return logits

    for _ in range(3):
        e2e_step()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(args.steps):
        e2e_step()
    b.record()
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(a.elapsed_time(b), dev, dist)
    e2e_value = world * B * args.steps / (e2e_ms / 1000.0)

    extras = {}
    if not args.no_extras:
        n_side = max(20, min(args.steps, 100))
        # fp32-faithful mode (exact integer weight planes), same protocol
        m32, _, _ = build_model(dev, args.batch, precision="fp32")
        p32 = m32.plan_for(x_dev)
        p32.x_in.copy_(x_dev)
        for _ in range(3):
            p32.fresh = True
            p32.run(use_graph=True)
        t32 = max_over_ranks(sum(time_plan(p32, n_side, flush, dist, gathered)), dev, dist)
        extras["precision_modes"] = {
            "fp16": {"value": value, "note": "fp16 weights (the reference GPU path's TF32/fp16 "
                                             "operand precision)"},
            "fp32": {"value": world * B * n_side / (t32 / 1000.0), "steps": n_side,
                     "note": "fp32-faithful: exact integer weight planes, hi+lo stem"}}
        del m32, p32
        extras["workloads"] = other_workloads(dev, flush, n_side, dist, world)
        if world > 1 and BATCH % world == 0:
            # strong scaling: the global batch of 64 sharded over the ranks
            bs = BATCH // world
            ms, _, _ = build_model(dev, bs)
            xs = x_dev[:, :bs].contiguous()
            ps = ms.plan_for(xs)
            ps.x_in.copy_(xs)
            gs = torch.empty((world, T_STEPS, bs, 10), device=dev)
            for _ in range(3):
                ps.fresh = True
                ps.run(use_graph=True)
                dist.all_gather_into_tensor(gs, ps.logits)
            ts = max_over_ranks(sum(time_plan(ps, n_side, flush, dist, gs)), dev, dist)
            extras["strong_scaling"] = {"global_batch": BATCH, "per_gpu_batch": bs,
                                        "value": BATCH * n_side / (ts / 1000.0),
                                        "ms_per_step": ts / n_side, "steps": n_side}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": {"workload": "SEW-ResNet18 CIFAR T=4 forward (BASELINE config 1)",
                       "model": "sew_resnet18_cifar", "global_batch": world * B,
                       "per_gpu_batch": B, "seq_len": T_STEPS, "parallelism": f"dp{world}",
                       "l2": "flushed between timed steps (256 MB write, then 256 MB read)",
                       "weights": "random init (seed 0), BN statistics calibrated on synthetic data",
                       "operands": "fp16 spikes/weights, fp32 accumulate + LIF",
                       "precision": "fp16"},
            "gpu_launches": plan.launches() * args.steps,
            "roofline": roofline,
            "e2e": {"value": e2e_value, "unit": UNIT,
                    "h2d_bytes_per_step": pinned.numel() * 4,
                    "d2h_bytes_per_step": out_host.numel() * 4},
            "clocks": clocks,
            "routing": {k: v for k, v in stats["patterns_matched"].items()},
            "egd": egd,
        }
        line.update(extras)
        if not args.no_cpu_baseline and world == 1:
            line["cpu_baseline"] = cpu_baseline()
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
