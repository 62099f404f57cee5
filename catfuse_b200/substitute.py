"""Graph rewrite: find fusible Conv/Linear -> BN -> LIF subgraphs in a
SpikingJelly-style model and swap in CTF patterns.

Follows the reference's matching rules (``catfuse/substitute.py``):

* ``substitute(model)`` (``:193-330``): SEW / Spiking ResNet BasicBlocks and
  Bottlenecks (recognised by class name and the SEW ``cnf`` attribute) become
  block patterns; ``nn.Sequential`` triples (Conv2d, BatchNorm2d, LIF) and
  pairs (Conv2d, LIF), (Linear, LIF) become fused patterns.
* ``substitute_sf(model, T)`` (``:362-797``): attribute-name triples
  ``conv{i}/bn{i}/sn{i}``, ``downsample`` + ``downsample_sn``,
  ``X/X_bn/X_lif|X_sn``, ``conv{i}/bn{i}/lif{i}``, ``rpe_conv/rpe_bn/rpe_lif``
  and Sequential triples, each routed by :func:`catfuse_b200.policy.get_policy`
  to ``STFusionConvBNLIF`` (SparseFlow) or ``PartialFusionConvBNLIF``
  (DenseKeep); matched BN / LIF slots become ``nn.Identity``.

Deliberate differences (each fixes a hazard of the reference):

* a standard Spiking ResNet BasicBlock / Bottleneck (residual added before the
  last LIF) is rewritten as a whole block pattern in ``substitute_sf`` too;
  matching its ``conv2/bn2/sn2`` triple would move the LIF before the add;
* ``Linear -> BatchNorm1d -> LIF`` is fused (BN folded into the epilogue)
  instead of being skipped;
* the duplicated phases of the reference run once.
"""
from __future__ import annotations

import copy

import torch.nn as nn

from .patterns import (CTFSEWBasicBlock, CTFSEWBottleneck, CTFSpikingBasicBlock,
                       CTFSpikingBottleneck, FusedLinearLIF, PartialFusionConvBNLIF,
                       PartialFusionConvLIF, STFusionConvBNLIF)
from .policy import SpatialBackend, get_policy
from .sj.neuron import is_lif as _is_lif


def _is_conv(m):
    return isinstance(m, nn.Conv2d)


def _is_bn2d(m):
    return isinstance(m, nn.BatchNorm2d)


def _is_bn1d(m):
    return isinstance(m, nn.BatchNorm1d)


def _is_linear(m):
    return isinstance(m, nn.Linear)


def _is_sew_basic_block(m):
    return type(m).__name__ == "BasicBlock" and getattr(m, "cnf", None) is not None


def _is_spiking_basic_block(m):
    return type(m).__name__ == "BasicBlock" and not hasattr(m, "cnf")


def _is_sew_bottleneck(m):
    return type(m).__name__ == "Bottleneck" and getattr(m, "cnf", None) is not None


def _is_spiking_bottleneck(m):
    return type(m).__name__ == "Bottleneck" and not hasattr(m, "cnf")


def _count_lif(model):
    return sum(1 for _, m in model.named_modules() if _is_lif(m))


def _k_s(c):
    ks = c.kernel_size[0] if isinstance(c.kernel_size, tuple) else c.kernel_size
    st = c.stride[0] if isinstance(c.stride, tuple) else c.stride
    return ks, st


# ---------------------------------------------------------------------------
# substitute()
# ---------------------------------------------------------------------------

def _rewrite_sequential(seq: nn.Sequential):
    children = list(seq)
    out, reps = [], []
    i, n = 0, len(children)
    while i < n:
        c = children[i]
        if i + 2 < n and _is_conv(c) and _is_bn2d(children[i + 1]) and _is_lif(children[i + 2]):
            out.append(PartialFusionConvBNLIF.from_sj_modules(c, children[i + 1], children[i + 2]))
            reps.append(("PartialFusionConvBNLIF", (i, i + 1, i + 2)))
            i += 3
            continue
        if i + 2 < n and _is_linear(c) and _is_bn1d(children[i + 1]) and _is_lif(children[i + 2]):
            out.append(FusedLinearLIF.from_sj_modules(c, children[i + 2], children[i + 1]))
            reps.append(("FusedLinearLIF", (i, i + 1, i + 2)))
            i += 3
            continue
        if i + 1 < n and _is_conv(c) and _is_lif(children[i + 1]):
            out.append(PartialFusionConvLIF.from_sj_modules(c, children[i + 1]))
            reps.append(("PartialFusionConvLIF", (i, i + 1)))
            i += 2
            continue
        if i + 1 < n and _is_linear(c) and _is_lif(children[i + 1]):
            out.append(FusedLinearLIF.from_sj_modules(c, children[i + 1]))
            reps.append(("FusedLinearLIF", (i, i + 1)))
            i += 2
            continue
        out.append(c)
        i += 1
    return nn.Sequential(*out), reps


_BLOCK_RULES = (
    (_is_sew_basic_block, CTFSEWBasicBlock, "CTFSEWBasicBlock", "SEWBasicBlock",
     lambda b: 3 if b.downsample is not None else 2),
    (_is_spiking_basic_block, CTFSpikingBasicBlock, "CTFSpikingBasicBlock", "SpikingBasicBlock",
     lambda b: 2),
    (_is_sew_bottleneck, CTFSEWBottleneck, "CTFSEWBottleneck", "SEWBottleneck",
     lambda b: 4 if b.downsample is not None else 3),
    (_is_spiking_bottleneck, CTFSpikingBottleneck, "CTFSpikingBottleneck", "SpikingBottleneck",
     lambda b: 3),
)


def substitute(sj_model: nn.Module, verbose: bool = False):
    model = copy.deepcopy(sj_model)
    stats = {"total_lif_nodes": _count_lif(model), "fused_lif_nodes": 0, "patterns_matched": {},
             "substituted_sequentials": [], "unsupported_structures": []}

    def bump(name, n=1):
        stats["patterns_matched"][name] = stats["patterns_matched"].get(name, 0) + 1
        stats["fused_lif_nodes"] += n

    def walk(parent, path=""):
        for name, child in list(parent.named_children()):
            cpath = f"{path}.{name}" if path else name
            done = False
            for pred, cls, pname, tag, nlif in _BLOCK_RULES:
                if pred(child):
                    setattr(parent, name, cls.from_sj_block(child))
                    bump(pname, nlif(child))
                    stats["substituted_sequentials"].append(f"{cpath}:{tag}")
                    if verbose:
                        print(f"  [substitute] {cpath}: {pname}")
                    done = True
                    break
            if done:
                continue
            if isinstance(child, nn.Sequential):
                new_seq, reps = _rewrite_sequential(child)
                if reps:
                    setattr(parent, name, new_seq)
                    stats["substituted_sequentials"].append(cpath)
                    for pname, idx in reps:
                        bump(pname)
                        if verbose:
                            print(f"  [substitute] {cpath}: {pname} @ indices {idx}")
                    walk(new_seq, cpath)
                else:
                    walk(child, cpath)
            else:
                walk(child, cpath)

    walk(model)
    stats["coverage_pct"] = (100.0 * stats["fused_lif_nodes"] / stats["total_lif_nodes"]
                             if stats["total_lif_nodes"] else 0.0)
    return model, stats


# ---------------------------------------------------------------------------
# substitute_sf()
# ---------------------------------------------------------------------------

def _h_est(cin):
    # The reference estimates the spatial size from the channel count
    # (catfuse/substitute.py:395); kept for routing parity.
    return 32 if cin <= 64 else (16 if cin <= 128 else 8)


def substitute_sf(sj_model, T=16, verbose=False, force_sparse=False, hwprof=None):
    model = copy.deepcopy(sj_model)
    stats = {"total_lif_nodes": _count_lif(model), "fused_lif_nodes": 0, "patterns_matched": {},
             "routing": []}
    done = set()

    def record(name, pattern, shape, backend, K):
        stats["fused_lif_nodes"] += 1
        stats["patterns_matched"][pattern] = stats["patterns_matched"].get(pattern, 0) + 1
        stats["routing"].append({"name": name, "pattern": pattern, "shape": shape,
                                 "backend": backend, "K": K})
        if verbose:
            print(f"  [substitute_sf] {name}: {pattern} ({shape}, backend={backend}, K={K})")

    def fuse_conv(c, b, l):
        cin, cout = c.in_channels, c.out_channels
        ks, st = _k_s(c)
        row = get_policy("Conv3x3_BN_LIF", C_in=cin, C_out=cout, H=_h_est(cin), W=_h_est(cin),
                         kernel_size=ks, T=T, hwprof=hwprof)
        use_sparse = force_sparse or row.spatial_backend == SpatialBackend.SPARSE_FLOW
        if use_sparse and ks == 3 and st == 1:
            b.eval()
            return (STFusionConvBNLIF.from_sj_modules(c, b, l, K=row.K), "STFusionConvBNLIF",
                    f"{cin}->{cout}, k={ks}, s={st}", row.spatial_backend, row.K)
        return (PartialFusionConvBNLIF.from_sj_modules(c, b, l), "PartialFusionConvBNLIF",
                f"{cin}->{cout}, k={ks}, s={st}", SpatialBackend.DENSE_KEEP, row.K)

    # Phase 0: standard Spiking ResNet blocks (add before the last LIF) are
    # rewritten as whole blocks so the LIF stays after the residual add.
    def walk_blocks(parent, path=""):
        for name, child in list(parent.named_children()):
            cpath = f"{path}.{name}" if path else name
            for pred, cls, pname, _, nlif in _BLOCK_RULES[1::2]:
                if pred(child):
                    for _, m in child.named_modules():
                        if _is_lif(m):
                            done.add(id(m))
                    blk = cls.from_sj_block(child)
                    n_rec = nlif(child)
                    if cls is CTFSpikingBasicBlock:
                        # the block's first Conv-BN-LIF is routed like any other
                        # (SparseFlow with the runtime EGD where the policy says so)
                        fused, pat, shape, backend, K = fuse_conv(child.conv1, child.bn1,
                                                                  child.sn1)
                        blk.fused_first = fused
                        record(cpath + ".conv1", pat, shape, backend, K)
                        n_rec -= 1
                    setattr(parent, name, blk)
                    for _ in range(n_rec):
                        record(cpath, pname, "block", SpatialBackend.DENSE_KEEP, T)
                    break
            else:
                walk_blocks(child, cpath)

    walk_blocks(model)

    # Phase 1: conv{i}/bn{i}/sn{i} triples
    for pname_, pmod in list(model.named_modules()):
        for i in ("1", "2", "3"):
            c, b, l = (getattr(pmod, f"conv{i}", None), getattr(pmod, f"bn{i}", None),
                       getattr(pmod, f"sn{i}", None))
            if not (_is_conv(c) and _is_bn2d(b) and _is_lif(l)) or id(l) in done:
                continue
            fused, pat, shape, backend, K = fuse_conv(c, b, l)
            setattr(pmod, f"conv{i}", fused)
            setattr(pmod, f"bn{i}", nn.Identity())
            setattr(pmod, f"sn{i}", nn.Identity())
            done.add(id(l))
            record(f"{pname_}.conv{i}" if pname_ else f"conv{i}", pat, shape, backend, K)

    # Phase 1b: SEW downsample = Sequential(Conv, BN) + downsample_sn
    for pname_, pmod in list(model.named_modules()):
        ds, ds_sn = getattr(pmod, "downsample", None), getattr(pmod, "downsample_sn", None)
        if not isinstance(ds, nn.Sequential) or len(ds) < 2 or not _is_lif(ds_sn) or id(ds_sn) in done:
            continue
        c, b = ds[0], ds[1]
        if not (_is_conv(c) and _is_bn2d(b)):
            continue
        fused = PartialFusionConvBNLIF.from_sj_modules(c, b, ds_sn)
        pmod.downsample = nn.Sequential(fused, nn.Identity())
        pmod.downsample_sn = nn.Identity()
        done.add(id(ds_sn))
        ks, st = _k_s(c)
        record(f"{pname_}.downsample" if pname_ else "downsample", "PartialFusionConvBNLIF",
               f"{c.in_channels}->{c.out_channels}, k={ks}, s={st}", SpatialBackend.DENSE_KEEP, T)

    # Phase 1c/1d: X/X_bn/X_lif|X_sn, conv{i}/bn{i}/lif{i}, rpe_conv/rpe_bn/rpe_lif
    for pname_, pmod in list(model.named_modules()):
        names = {n for n, _ in pmod.named_children()}
        triples = []
        for n in sorted(names):
            for suf in ("_bn", "_lif", "_sn"):
                if n.endswith(suf):
                    base = n[:-len(suf)]
                    lif_name = base + "_lif" if base + "_lif" in names else base + "_sn"
                    triples.append((base, base + "_bn", lif_name))
        triples += [(f"conv{i}", f"bn{i}", f"lif{i}") for i in range(10)]
        triples.append(("rpe_conv", "rpe_bn", "rpe_lif"))
        seen = set()
        for cn, bn_, ln in triples:
            if (cn, ln) in seen:
                continue
            seen.add((cn, ln))
            c, b, l = getattr(pmod, cn, None), getattr(pmod, bn_, None), getattr(pmod, ln, None)
            if c is None or b is None or not _is_lif(l) or id(l) in done:
                continue
            full = f"{pname_}.{cn}" if pname_ else cn
            if _is_conv(c) and _is_bn2d(b):
                if cn == "rpe_conv":
                    fused = PartialFusionConvBNLIF.from_sj_modules(c, b, l)
                    pat, shape, backend, K = ("PartialFusionConvBNLIF",
                                              f"{c.in_channels}->{c.out_channels}",
                                              SpatialBackend.DENSE_KEEP, T)
                else:
                    fused, pat, shape, backend, K = fuse_conv(c, b, l)
            elif _is_linear(c) and _is_bn1d(b):
                fused = FusedLinearLIF.from_sj_modules(c, l, b)
                pat, shape, backend, K = ("FusedLinearLIF", f"{c.in_features}->{c.out_features}",
                                          SpatialBackend.DENSE_KEEP, T)
            else:
                continue
            setattr(pmod, cn, fused)
            setattr(pmod, bn_, nn.Identity())
            setattr(pmod, ln, nn.Identity())
            done.add(id(l))
            record(full, pat, shape, backend, K)

    # Phase 2: Sequential triples / pairs
    for pname_, pmod in list(model.named_modules()):
        for name, child in list(pmod.named_children()):
            if not isinstance(child, nn.Sequential):
                continue
            kids = list(child)
            new, changed, i = [], False, 0
            while i < len(kids):
                c = kids[i]
                full = f"{pname_}.{name}.{i}" if pname_ else f"{name}.{i}"
                if (i + 2 < len(kids) and _is_conv(c) and _is_bn2d(kids[i + 1])
                        and _is_lif(kids[i + 2]) and id(kids[i + 2]) not in done):
                    fused, pat, shape, backend, K = fuse_conv(c, kids[i + 1], kids[i + 2])
                    new.append(fused)
                    done.add(id(kids[i + 2]))
                    record(full, pat, shape, backend, K)
                    changed = True
                    i += 3
                    continue
                if (i + 2 < len(kids) and _is_linear(c) and _is_bn1d(kids[i + 1])
                        and _is_lif(kids[i + 2]) and id(kids[i + 2]) not in done):
                    new.append(FusedLinearLIF.from_sj_modules(c, kids[i + 2], kids[i + 1]))
                    done.add(id(kids[i + 2]))
                    record(full, "FusedLinearLIF", f"{c.in_features}->{c.out_features}",
                           SpatialBackend.DENSE_KEEP, T)
                    changed = True
                    i += 3
                    continue
                if (i + 1 < len(kids) and _is_linear(c) and _is_lif(kids[i + 1])
                        and id(kids[i + 1]) not in done):
                    new.append(FusedLinearLIF.from_sj_modules(c, kids[i + 1]))
                    done.add(id(kids[i + 1]))
                    record(full, "FusedLinearLIF", f"{c.in_features}->{c.out_features}",
                           SpatialBackend.DENSE_KEEP, T)
                    changed = True
                    i += 2
                    continue
                new.append(c)
                i += 1
            if changed:
                setattr(pmod, name, nn.Sequential(*new))

    stats["coverage_pct"] = 100.0 * stats["fused_lif_nodes"] / max(stats["total_lif_nodes"], 1)
    return model, stats


def print_coverage_report(stats: dict, title: str = "Coverage report"):
    print(f"\n{'=' * 70}\n{title}\n{'=' * 70}")
    print(f"  total LIF nodes      : {stats['total_lif_nodes']}")
    print(f"  fused LIF nodes      : {stats['fused_lif_nodes']}")
    print(f"  coverage             : {stats['coverage_pct']:.2f}%")
    print("\n  patterns matched:")
    for pattern, count in sorted(stats["patterns_matched"].items()):
        print(f"    {pattern:<30} {count} instance(s)")
    for path in stats.get("substituted_sequentials", []):
        print(f"    {path}")


def print_routing_table(stats):
    print(f"\n{'layer':<28} {'pattern':<24} {'shape':<24} {'backend':<12} K")
    for r in stats.get("routing", []):
        print(f"{r['name']:<28} {r['pattern']:<24} {r['shape']:<24} {r['backend']:<12} {r['K']}")


__all__ = ["substitute", "substitute_sf", "print_coverage_report", "print_routing_table"]
