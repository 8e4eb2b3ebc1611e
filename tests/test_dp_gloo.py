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
