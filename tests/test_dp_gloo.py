"""CPU, world size 2 (gloo): the data-parallel reduction the training bench
uses.  Each rank computes gradients of the mean loss of its own batch; a SUM
all-reduce followed by grad_scale = 1/world (what ne_adamw_step applies)
must equal the gradient of the mean loss over the concatenated global batch,
and the max-over-ranks timing reduction must return the slowest rank."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import sys
        sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
        from oracle import model as om
        from oracle import train as ot
        cfg = om.tiny(head_dim=16, qk_norm=True)
        layers, rf, emb, qk = om.init_weights(cfg, seed=5, std=0.1)
        tok_all = om.prompt_tokens(cfg.vocab, 9, 6, batch=2 * world)
        mine = tok_all[2 * rank:2 * rank + 2]
        _, g = ot.loss_and_grads(cfg, layers, rf, emb, qk, mine)
        flat = torch.tensor(np.concatenate([g["embed"].ravel(), g["layers"][1]["W2"].ravel(),
                                            g["qk"][0][0].ravel()]))
        dist.all_reduce(flat, op=dist.ReduceOp.SUM)
        flat /= world
        t = torch.tensor([1.0 + rank])
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        if rank == 0:
            _, gg = ot.loss_and_grads(cfg, layers, rf, emb, qk, tok_all)
            ref = np.concatenate([gg["embed"].ravel(), gg["layers"][1]["W2"].ravel(),
                                  gg["qk"][0][0].ravel()])
            q.put((float(np.abs(flat.numpy() - ref).max()), float(np.abs(ref).max()),
                   float(t.item())))
    finally:
        dist.destroy_process_group()


def test_dp_allreduce_equals_global_batch_gradient():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    err, scale, tmax = q.get(timeout=5)
    assert err <= 1e-9 * max(scale, 1.0), (err, scale)
    assert tmax == 2.0


def _leaver(rank, port, q):
    """Rank 1 joins the coordination group and leaves between steps (nothing
    in flight); rank 0's next max-over-ranks must end with an error, not wait."""
    import sys
    import time
    from datetime import timedelta
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=timedelta(seconds=5))
    if rank == 1:
        os._exit(0)
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import bench
    t0 = time.time()
    try:
        bench.allmax(1.0, 2)
        q.put(("returned", time.time() - t0, ""))
    except Exception as e:
        q.put(("raised", time.time() - t0, repr(e)))
    os._exit(0)


def test_rank_that_leaves_ends_the_others_coordination():
    """bench.py's coordination group (gloo, a short timeout): a rank that
    exits between steps makes the next max-over-ranks raise on the others
    within the timeout, so no bench rank waits for good."""
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_leaver, args=(r, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    kind, took, msg = q.get(timeout=120)
    for p in ps:
        p.join(timeout=30)
    assert kind == "raised", (kind, took, msg)
    assert took < 60, took
