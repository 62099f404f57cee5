"""Batch-sharded inference with a logits all-gather, as world_size-2 gloo
process groups on the CPU (the host-side logic of the multi-GPU path), plus
the failure path: a rank that dies before the collective makes the survivor's
gather fail with a timeout error instead of hanging.  No GPU involved."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, mode, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world))
    import torch.distributed as dist
    from catfuse_b200.distributed import ShardedInference, init_inference_group
    try:
        init_inference_group("gloo", timeout_s=20.0 if mode == "ok" else 4.0)
        torch.manual_seed(0)
        W = torch.randn(10, 3 * 8 * 8)

        def fwd(x):  # stand-in per-sample model: [T, b, 3, 8, 8] -> [T, b, 10]
            return x.flatten(2) @ W.T

        x = torch.randn(4, 7, 3, 8, 8, generator=torch.Generator().manual_seed(1))
        if mode == "dead" and rank == 1:
            q.put((rank, "exited"))
            q.close()
            q.join_thread()
            os._exit(0)  # leaves between steps, never joins the collective
        out = ShardedInference(fwd)(x)
        q.put((rank, bool(torch.allclose(out, fwd(x), atol=1e-5))))
        dist.destroy_process_group()
    except Exception as e:  # noqa: BLE001
        q.put((rank, f"error:{type(e).__name__}"))


def _run(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(60)
        if p.is_alive():
            p.kill()
    res = {}
    while not q.empty():
        r, v = q.get()
        res[r] = v
    return res


def test_sharded_inference_gather_matches_full_batch():
    res = _run("ok")
    assert res == {0: True, 1: True}, res


def test_lost_rank_surfaces_as_error():
    res = _run("dead")
    assert res.get(1) == "exited"
    assert isinstance(res.get(0), str) and res[0].startswith("error:"), res
